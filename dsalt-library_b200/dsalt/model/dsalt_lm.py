"""DSALT causal language model (reference ``dsalt/model/dsalt_lm.py``).

Same constructor, module tree, parameter names and initialisation order as the
reference, so a seeded construction and reference checkpoints give identical
weights.  The attention layers run the B200 CUDA ops.  The loss: on CUDA in
16-bit compute every ``loss_fn`` runs the fused chunked loss of
``kernels/fused_ce.py`` (loss and gradient per chunk in one pass over the
logits), the B200 counterpart of the reference's Triton fused linear
cross-entropy (``"liger"``); elsewhere the reference's chunked loss.  ``"auto"``
(the reference measures chunked against Liger once per device) therefore
resolves to the same computation.
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..kernels.RMSENorm import RMSENorm
from ..kernels import _ext
from ..kernels.fused_ce import fused_chunked_cross_entropy
from ..modules.dsalt_transformer import DSALTTransformerBlock
from .config import DSALTConfig


def _chunked_cross_entropy(x: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                           chunk_size: int = 512) -> torch.Tensor:
    """Mean CE over non-ignored labels, the LM head applied chunk by chunk (reference :19-39)."""
    total = x.shape[0]
    loss_acc = torch.zeros((), device=x.device, dtype=torch.float32)
    valid_acc = torch.zeros((), device=x.device, dtype=torch.float32)
    for start in range(0, total, chunk_size):
        end = min(start + chunk_size, total)
        y = labels[start:end]
        logits = F.linear(x[start:end], weight)
        loss_acc = loss_acc + F.cross_entropy(logits, y, ignore_index=-100, reduction="sum")
        valid_acc = valid_acc + (y != -100).sum()
    return loss_acc / valid_acc.clamp(min=1.0)


def _fused_ce_dtype(x: torch.Tensor, weight: torch.Tensor):
    """The 16-bit dtype of the chunk logits for the fused loss; None: the torch path."""
    return _ext.half_compute_dtype(x, weight)


_LOSS_FN = {"auto": None, "liger": None, "chunked": _chunked_cross_entropy}


class DSALTLMHeadModel(nn.Module):
    """Causal LM: embedding → DSALT blocks → RMSNorm → (tied) LM head (reference :64-285)."""

    def __init__(self, vocab_size, d_model, n_layers, n_heads, n_min, n_max, k_lmk, max_seq_len, d_ff=None,
                 dropout=0.0, yarn_scale=1.0, tie_weights=True, padding_idx=None, lm_head_chunk_size=2048,
                 loss_fn="chunked", aux_loss_weight=0.0, n_kv_heads=None, qkv_bias=False, rope_base=10000.0):
        super().__init__()
        assert loss_fn in _LOSS_FN, f"loss_fn must be one of {list(_LOSS_FN)}"
        self.d_model = d_model
        self.n_layers = n_layers
        self.vocab_size = vocab_size
        self.lm_head_chunk_size = lm_head_chunk_size
        self._cu_host = None  # (cu_seqlens, version, host list): see _host_cu
        self.loss_fn = loss_fn
        self.aux_loss_weight = aux_loss_weight
        if d_ff is None:
            hidden = int(8 / 3 * d_model)
            d_ff = ((hidden + 127) // 128) * 128
        self.embed_tokens = nn.Embedding(vocab_size, d_model, padding_idx=padding_idx)
        self.embed_dropout = nn.Dropout(dropout)
        self.layers = nn.ModuleList([
            DSALTTransformerBlock(d_model=d_model, n_heads=n_heads, n_min=n_min, n_max=n_max, k_lmk=k_lmk,
                                  max_seq_len=max_seq_len, d_ff=d_ff, dropout=dropout, yarn_scale=yarn_scale,
                                  layer_idx=i, n_kv_heads=n_kv_heads, qkv_bias=qkv_bias, rope_base=rope_base)
            for i in range(n_layers)
        ])
        self.final_norm = RMSENorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab_size, bias=False)
        if tie_weights:
            self.lm_head.weight = self.embed_tokens.weight
        self._init_weights()

    @classmethod
    def from_config(cls, config: DSALTConfig) -> "DSALTLMHeadModel":
        return cls(**config.to_dict())

    def _init_weights(self):
        nn.init.normal_(self.embed_tokens.weight, std=0.02)
        residual_std = 0.02 / math.sqrt(2 * self.n_layers)
        for name, module in self.named_modules():
            if isinstance(module, nn.Linear):
                std = residual_std if any(k in name for k in ("out_proj", "down_proj")) else 0.02
                nn.init.normal_(module.weight, std=std)
                if module.bias is not None:
                    nn.init.zeros_(module.bias)

    def _compute_loss(self, x: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        flat_x = x.reshape(-1, self.d_model)
        flat_labels = labels.reshape(-1).long()
        dt = _fused_ce_dtype(flat_x, self.lm_head.weight)
        if dt is not None:
            return fused_chunked_cross_entropy(flat_x, self.lm_head.weight, flat_labels, self.lm_head_chunk_size, dt)
        return _chunked_cross_entropy(flat_x, self.lm_head.weight, flat_labels, self.lm_head_chunk_size)

    @staticmethod
    def _to_autocast_dtype(x: torch.Tensor) -> torch.Tensor:
        dev = x.device.type
        if torch.is_autocast_enabled(dev):
            dt = torch.get_autocast_dtype(dev)
            return x.to(dt) if x.dtype != dt else x
        return x

    def _host_cu(self, cu_seqlens: torch.Tensor) -> list:
        """Host copy of ``cu_seqlens``.  While the same tensor object comes back with
        an unchanged version counter (no in-place write since), the previous copy is
        reused, so a fixed packing costs no device-to-host sync per step."""
        c = self._cu_host
        if c is not None and c[0] is cu_seqlens and c[1] == cu_seqlens._version:
            return c[2]
        lst = cu_seqlens.detach().to("cpu").tolist()
        self._cu_host = (cu_seqlens, cu_seqlens._version, lst)
        return lst

    def _packed_rope_meta(self, cu_seqlens: torch.Tensor, total_len: int, attn0):
        """RoPE cos/sin gathered per packed position and a host copy of cu_seqlens (reference :218-235)."""
        device = cu_seqlens.device
        cu_list = self._host_cu(cu_seqlens)
        cu = cu_seqlens.long()
        lens = cu[1:] - cu[:-1]
        seq_ids = torch.repeat_interleave(torch.arange(cu.shape[0] - 1, device=device), lens,
                                          output_size=int(cu_list[-1]))
        pos_ids = torch.arange(total_len, device=device) - cu[:-1][seq_ids]
        rope_cs = (attn0.rope_cos.to(device)[pos_ids], attn0.rope_sin.to(device)[pos_ids])
        if torch.is_autocast_enabled(device.type):
            # every layer casts the rows to the compute dtype: do it once
            dt = torch.get_autocast_dtype(device.type)
            rope_cs = (rope_cs[0].to(dt), rope_cs[1].to(dt))
        return rope_cs, cu_list

    def forward(self, input_ids, cu_seqlens=None, max_seqlen=None, labels=None, gradient_checkpointing=False,
                padding_mask=None) -> dict:
        if max_seqlen is None:
            max_seqlen = input_ids.shape[-1]
        x = self.embed_dropout(self.embed_tokens(input_ids))
        x = self._to_autocast_dtype(x)
        aux_loss = torch.zeros((), device=input_ids.device, dtype=x.dtype)
        rope_cs = cu_list = None
        if cu_seqlens is not None:
            rope_cs, cu_list = self._packed_rope_meta(cu_seqlens, input_ids.shape[0], self.layers[0].attn)
        # each block leaves its last residual add (x + ffn_out) to the next RMSNorm,
        # which fuses it: the next block's attn_norm, or final_norm
        pending = None
        for layer in self.layers:
            x, layer_aux, pending = layer(x, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen,
                                          gradient_checkpointing=gradient_checkpointing, rope_cs=rope_cs,
                                          cu_list=cu_list, pending=pending, defer=True)
            aux_loss = aux_loss + layer_aux
        x = self.final_norm(x) if pending is None else self.final_norm.add_forward(x, pending)[1]
        if labels is not None:
            loss = self._compute_loss(x, labels) + self.aux_loss_weight * aux_loss
            return {"loss": loss, "logits": None, "aux_loss": aux_loss.detach()}
        return {"loss": None, "logits": self.lm_head(x), "aux_loss": None}

    def num_parameters(self, trainable_only: bool = True) -> int:
        if trainable_only:
            return sum(p.numel() for p in self.parameters() if p.requires_grad)
        return sum(p.numel() for p in self.parameters())
