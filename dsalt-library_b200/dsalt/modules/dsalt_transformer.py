"""Pre-norm transformer block with DSALT attention (reference dsalt/modules/dsalt_transformer.py)."""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F
import torch.utils.checkpoint

from ..kernels import _ext
from ..kernels import swiglu as swiglu_cuda
from ..kernels.RMSENorm import RMSENorm
from .dsalt_attention import DSALTAttention


class SwiGLUFFN(nn.Module):
    """``down(silu(gate(x)) * up(x))`` (reference :10-21).

    On CUDA in 16-bit compute (autocast, or 16-bit input and weights) the block
    runs as ``kernels/swiglu.py``'s fused function: one gate+up GEMM, the CUDA
    activation each way, one GEMM per gradient.  Elsewhere the reference's ops.
    """

    def __init__(self, d_model: int, d_ff: int, dropout: float = 0.0):
        super().__init__()
        self.gate_proj = nn.Linear(d_model, d_ff, bias=False)
        self.up_proj = nn.Linear(d_model, d_ff, bias=False)
        self.down_proj = nn.Linear(d_ff, d_model, bias=False)
        self.drop = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w_g, w_u, w_d = self.gate_proj.weight, self.up_proj.weight, self.down_proj.weight
        dt = _ext.half_compute_dtype(x, w_g, w_u, w_d)
        if dt is not None and swiglu_cuda.supported(x, w_g):
            return self.drop(swiglu_cuda.swiglu_ffn(x, w_g, w_u, w_d, dt))
        return self.drop(self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x)))


class DSALTTransformerBlock(nn.Module):
    """RMSNorm → DSALTAttention → residual, RMSNorm → SwiGLU → residual (reference :24-86)."""

    def __init__(self, d_model, n_heads, n_min, n_max, k_lmk, max_seq_len, d_ff, dropout=0.0,
                 yarn_scale=1.0, layer_idx=0, n_kv_heads=None, qkv_bias=False, rope_base=10000.0):
        super().__init__()
        self.layer_idx = layer_idx
        self.attn_norm = RMSENorm(d_model)
        self.ffn_norm = RMSENorm(d_model)
        self.attn = DSALTAttention(d_model=d_model, n_heads=n_heads, n_min=n_min, n_max=n_max, k_lmk=k_lmk,
                                   max_seq_len=max_seq_len, dropout=dropout, yarn_scale=yarn_scale,
                                   layer_idx=layer_idx, n_kv_heads=n_kv_heads, qkv_bias=qkv_bias,
                                   rope_base=rope_base)
        self.ffn = SwiGLUFFN(d_model=d_model, d_ff=d_ff, dropout=dropout)

    def forward(self, x, cu_seqlens=None, max_seqlen=None, gradient_checkpointing=False, rope_cs=None,
                cu_list=None, pending=None, defer=False):
        """``(x, aux)`` as the reference block.  ``pending`` / ``defer`` let the model
        fuse each residual add into the RMSNorm after it: with ``pending`` the block
        first forms ``x + pending``; with ``defer`` it returns ``(x, aux, ffn_out)``
        and leaves the final ``x + ffn_out`` to the caller."""
        if not (gradient_checkpointing and self.training):
            if pending is not None:
                x, h = self.attn_norm.add_forward(x, pending)
            else:
                h = self.attn_norm(x)
            x_attn, aux = self.attn(h, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen, rope_cs=rope_cs,
                                    cu_list=cu_list)
            x, h = self.ffn_norm.add_forward(x, x_attn)
            f = self.ffn(h)
            return (x, aux, f) if defer else (x + f, aux)
        if pending is not None:
            x = x + pending
        x, aux = self._forward_checkpointed(x, cu_seqlens, max_seqlen, rope_cs, cu_list)
        return (x, aux, None) if defer else (x, aux)

    def _forward_checkpointed(self, x, cu_seqlens, max_seqlen, rope_cs, cu_list):
        """The reference's checkpointed path: attention and FFN recomputed in the backward."""
        aux_box = []

        def attn_fn(h):
            out, a = self.attn(h, cu_seqlens=cu_seqlens, max_seqlen=max_seqlen, rope_cs=rope_cs,
                               cu_list=cu_list)
            aux_box.append(a)
            return out
        x = x + torch.utils.checkpoint.checkpoint(attn_fn, self.attn_norm(x), use_reentrant=False)
        x = x + torch.utils.checkpoint.checkpoint(self.ffn, self.ffn_norm(x), use_reentrant=False)
        aux = aux_box[-1] if aux_box else torch.zeros((), device=x.device, dtype=x.dtype)
        return x, aux

