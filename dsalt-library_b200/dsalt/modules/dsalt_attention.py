"""DSALT sparse attention module on B200 (drop-in for the reference module).

Reference: ``dsalt/modules/dsalt_attention.py``.  Same constructor, parameter
names (``q_proj``, ``k_proj``, ``v_proj``, ``out_proj``, ``win_gate``,
``alpha_w``) and ``forward(x, cu_seqlens, max_seqlen, rope_cs, cu_list) ->
(out, aux)`` contract, so reference checkpoints load unchanged.  Query ``i``
attends ``A(i) = W(i) ∪ L(i)``: the adaptive causal window predicted by
``win_gate`` and the per-head top-k landmarks of its sequence chosen by the
hybrid score.

Every attention computation runs on the hand-written sm_100a kernels:
window gate (``dsalt_win_gate``), hybrid score + top-k (``dsalt_hybrid_scores``,
``dsalt_select_topk``) and the training / inference attention ops.  There is
no dense SDPA fallback; CPU tensors raise.

Deliberate differences from the reference:
  * ``[B, T, d]`` input goes through the packed op (``B`` sequences of ``T``);
    the reference's batched path is a dense reference that only accepts B = 1
    (dsalt_attention.py:382, 391-401);
  * ``_last_P`` (the dense attention matrix of the first sequence, an eval-mode
    diagnostic, :636-702) is only built when ``_collect_last_P`` is set to True.
"""

from __future__ import annotations

import math
import warnings

import torch
import torch.nn as nn

from ..kernels import _ext
from ..kernels.rope_gqa import qkv_rope, rope_gqa
from ..kernels.window_utils import build_rope_cache
from ..kernels.landmark_tokens_ker import hybrid_scores_per_head
from ..kernels.selectors import select_topk, _compute_landmark_indices
from ..kernels.window_gate import window_continuous
from ..kernels.dsalt_triton_attn import dsalt_triton_attention
from ..kernels.dsalt_triton_train import dsalt_triton_train_attention

_TRITON_OK = True        # names kept: the CUDA ops take the Triton ops' place
_TRITON_TRAIN_OK = True


def _dynamo_opaque(fn):
    disable = getattr(getattr(torch, "_dynamo", None), "disable", None)
    return disable(fn) if disable is not None else fn


class DSALTAttention(nn.Module):
    """DSALT sparse attention: adaptive local window plus landmark tokens (reference :147-703)."""

    def __init__(
        self,
        d_model:     int,
        n_heads:     int,
        n_min:       int,
        n_max:       int,
        k_lmk:       int,
        max_seq_len: int,
        dropout:     float = 0.0,
        yarn_scale:  float = 1.0,
        layer_idx:   int   = 0,
        n_kv_heads:  int | None = None,
        qkv_bias:    bool   = False,
        rope_base:   float  = 10000.0,
    ):
        super().__init__()
        assert d_model % n_heads == 0
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.n_kv_heads = n_kv_heads if n_kv_heads is not None else n_heads
        assert n_heads % self.n_kv_heads == 0, "n_heads must be a multiple of n_kv_heads"
        self.n_rep = n_heads // self.n_kv_heads
        self.kv_dim = self.n_kv_heads * self.head_dim
        self.n_min = n_min
        self.n_max = n_max
        self.k_lmk = k_lmk
        self.max_seq_len = max_seq_len
        self.dropout = dropout
        self.yarn_scale = yarn_scale
        self.rope_base = rope_base
        self.layer_idx = layer_idx

        self.q_proj = nn.Linear(d_model, d_model, bias=qkv_bias)
        self.k_proj = nn.Linear(d_model, self.kv_dim, bias=qkv_bias)
        self.v_proj = nn.Linear(d_model, self.kv_dim, bias=qkv_bias)
        self.out_proj = nn.Linear(d_model, d_model, bias=False)
        self.win_gate = nn.Linear(d_model, 1, bias=True)
        self.alpha_w = nn.Parameter(torch.full((n_heads,), math.log(0.6 / 0.4)))

        self.tau_win = 1.0
        self.tau_lmk = 2.0
        self.win_edge = 4

        self._last_P: torch.Tensor | None = None
        self._collect_last_P = False

        cos, sin = build_rope_cache(max_seq_len, self.head_dim, torch.device("cpu"), base=rope_base,
                                    scale=yarn_scale)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)

    # ------------------------------------------------------------ helpers
    def _alpha(self) -> torch.Tensor:
        return torch.sigmoid(self.alpha_w)

    def _apply_out_proj(self, out: torch.Tensor) -> torch.Tensor:
        # under autocast the linear casts its input itself (a 16-bit output of the
        # op then goes in unchanged)
        if torch.is_autocast_enabled(out.device.type):
            return self.out_proj(out)
        return self.out_proj(out.to(self.out_proj.weight.dtype))

    def _op_out_dtype(self, q: torch.Tensor):
        """The dtype the attention op may return O in: q's 16-bit dtype when out_proj
        computes in it (autocast, or 16-bit weights), so that the fp32 output and its
        casts are skipped; None (the reference's fp32 output) otherwise."""
        if q.dtype == torch.float32:
            return None
        dev = q.device.type
        if torch.is_autocast_enabled(dev) and torch.get_autocast_dtype(dev) == q.dtype:
            return q.dtype
        return q.dtype if self.out_proj.weight.dtype == q.dtype else None

    def _repeat_kv(self, t: torch.Tensor) -> torch.Tensor:
        if self.n_rep == 1:
            return t
        if t.dim() == 3:
            T, _, D = t.shape
            return t.unsqueeze(2).expand(T, self.n_kv_heads, self.n_rep, D).reshape(T, self.n_heads, D)
        B, _, T, D = t.shape
        return t.unsqueeze(2).expand(B, self.n_kv_heads, self.n_rep, T, D).reshape(B, self.n_heads, T, D)

    def _window_continuous(self, x: torch.Tensor) -> torch.Tensor:
        """``w̃(i) = n_min + σ(win_gate(x_i))·(n_max − n_min)``, ``[T]`` (reference :270-275)."""
        return window_continuous(x, self.win_gate, self.n_min, self.n_max)

    @torch.no_grad()
    def _window_sizes(self, x: torch.Tensor, floor: bool) -> torch.Tensor:
        """Discrete window: floor at inference, round otherwise, at least 1 (reference :277-284)."""
        w = self._window_continuous(x)
        w = w.floor() if floor else w.round()
        return w.clamp(min=1)

    @torch.no_grad()
    def _rope(self, n: int, device: torch.device):
        if n <= self.rope_cos.shape[0]:
            return self.rope_cos[:n].to(device), self.rope_sin[:n].to(device)
        return self.rope_cos.to(device), self.rope_sin.to(device)

    def _aux_zero(self, device, dtype):
        return torch.zeros((), device=device, dtype=dtype)

    @torch.no_grad()
    def warmup(self, device: torch.device) -> None:
        was = self.training
        self.eval()
        T = max(self.n_min * 2, 16)
        x = torch.randn(T, self.d_model, device=device)
        cu = torch.tensor([0, T], dtype=torch.int32, device=device)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            self._packed(x, cu, T, device, None, [0, T])
        if device.type == "cuda":
            torch.cuda.synchronize(device)
        self.train(was)

    # ------------------------------------------------------------ forward
    def forward(self, x, cu_seqlens=None, max_seqlen=None, rope_cs=None, cu_list=None):
        if cu_seqlens is not None:
            return self._packed(x, cu_seqlens, x.shape[0], x.device, rope_cs, cu_list)
        B, T, _ = x.shape
        return self._batched(x, B, T, x.device)

    def _batched(self, x, B, T, device):
        """``[B, T, d]`` input, run as ``B`` packed sequences of length ``T``."""
        cu_list = [b * T for b in range(B + 1)]
        cu = torch.tensor(cu_list, dtype=torch.int32, device=device)
        out, aux = self._packed(x.reshape(B * T, self.d_model), cu, B * T, device, None, cu_list)
        return out.view(B, T, self.d_model), aux

    def _project_qkv(self, x, total_len, cos, sin):
        """``(q, k, v, xwv)``: the projections with RoPE on q and k (reference
        apply_rotary_emb, bitwise equal at equal projections), k and v with their
        ``n_kv_heads`` heads: the attention ops read the kv head of each query head in
        place instead of the reference's _repeat_kv expansion (:254-268); and the value
        projection x·W_Vᵀ for the landmark scorer (v carries no RoPE), or None with a v
        bias.  Bias-free in 16-bit compute on CUDA the three projections run as one GEMM
        feeding the prologue kernel (``qkv_rope``)."""
        wq, wk, wv = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight
        no_bias = self.q_proj.bias is None and self.k_proj.bias is None and self.v_proj.bias is None
        dt = _ext.half_compute_dtype(x, wq, wk, wv) if no_bias else None
        if dt is not None:
            return qkv_rope(x, wq, wk, wv, cos, sin, self.n_heads, self.n_kv_heads, self.head_dim, dt, expand=False)
        q = self.q_proj(x).view(total_len, self.n_heads, self.head_dim)
        k = self.k_proj(x).view(total_len, self.n_kv_heads, self.head_dim)
        v = self.v_proj(x).view(total_len, self.n_kv_heads, self.head_dim)
        xwv = v.view(total_len, self.kv_dim) if self.v_proj.bias is None else None
        q, k, v = rope_gqa(q, k, v, cos.to(q.dtype), sin.to(q.dtype), expand=False)
        return q, k, v, xwv

    def _packed_train_triton(self, q, k, v, x, cu_seqlens, total_len, device, cu_list=None, xwv=None):
        """Training attention on the CUDA op, carrying the window and α gradients (reference :440-455)."""
        w_cont, lmk_pos, lmk_logw = self._train_selectors(x, cu_seqlens, total_len, device, cu_list, xwv)
        return dsalt_triton_train_attention(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens,
                                            tau_win=self.tau_win, win_edge=float(self.win_edge),
                                            n_max=self.n_max, cu_list=cu_list, out_dtype=self._op_out_dtype(q))

    @_dynamo_opaque
    def _train_selectors(self, x, cu_seqlens, total_len, device, cu_list=None, xwv=None):
        """``(w_cont [T], lmk_pos [H,S,k], lmk_logw [H,S,k])`` (reference :457-487).

        The hybrid score is computed once: its detached value drives the hard top-k
        (the reference recomputes the identical values under no_grad) and its graph
        carries the landmark-weight gradient to ``alpha_w``, ``x`` and ``v_proj``.
        """
        w_cont = self._window_continuous(x)
        alpha = self._alpha()
        scores, _, _ = hybrid_scores_per_head(x, self.v_proj.weight, alpha, self.n_heads, self.head_dim, xwv=xwv)
        cu_h = cu_list if cu_list is not None else cu_seqlens.detach().to("cpu").tolist()
        max_len = max((cu_h[b + 1] - cu_h[b] for b in range(len(cu_h) - 1)), default=0)
        with torch.no_grad():
            w_disc = w_cont.detach().float().floor().clamp(min=1)
            lmk_pos = select_topk(scores.detach(), w_disc, cu_seqlens, self.k_lmk, max_len)
        starts = cu_seqlens[:-1].to(device).long()
        abs_pos = starts[None, :, None] + lmk_pos.clamp(min=0)
        head_ix = torch.arange(self.n_heads, device=device)[:, None, None]
        # scores[abs_pos, head_ix] as a flat gather, whose backward is a scatter-add
        # instead of index_put's sort: a (position, head) pair repeats only for
        # padding slots (lmk_pos = -1), whose gradient is exactly zero, so the sum
        # does not depend on the order of the additions
        s_sel = scores.reshape(-1).gather(0, (abs_pos * self.n_heads + head_ix).reshape(-1)).view(abs_pos.shape)
        lmk_logw = torch.log(torch.sigmoid(s_sel / self.tau_lmk).clamp(min=1e-20))
        lmk_logw = torch.where(lmk_pos >= 0, lmk_logw, torch.full_like(lmk_logw, float("-inf")))
        return w_cont, lmk_pos, lmk_logw

    def _packed(self, x, cu_seqlens, total_len, device, rope_cs=None, cu_list=None):
        if rope_cs is None:
            num_seqs = cu_seqlens.shape[0] - 1
            cu = cu_seqlens.to(device).long()
            lens = cu[1:] - cu[:-1]
            seq_ids = torch.repeat_interleave(torch.arange(num_seqs, device=device), lens)
            pos_ids = torch.arange(total_len, device=device) - cu[:-1][seq_ids]
            cos = self.rope_cos.to(device)[pos_ids]
            sin = self.rope_sin.to(device)[pos_ids]
        else:
            cos, sin = rope_cs
        q, k, v, xwv = self._project_qkv(x, total_len, cos, sin)
        aux = self._aux_zero(x.device, x.dtype)

        if self.training:
            self._last_P = None
            out = self._packed_train_triton(q, k, v, x, cu_seqlens, total_len, device, cu_list, xwv)
            return self._apply_out_proj(out.view(total_len, self.d_model)), aux

        w_sizes = self._window_sizes(x, floor=True)
        alpha = self._alpha()
        lmk_indices, _, _ = _compute_landmark_indices(
            x.detach(), self.v_proj.weight.detach(), alpha.detach().float(), w_sizes, cu_seqlens,
            self.k_lmk, self.n_min, total_len, cu_list, head_dim=self.head_dim,
            xwv=None if xwv is None else xwv.detach())
        lmk_bias = torch.zeros_like(lmk_indices, dtype=torch.float32)
        out = dsalt_triton_attention(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens)
        self._last_P = self._dense_first_sequence(q, k, w_sizes, lmk_indices, cu_seqlens) \
            if self._collect_last_P else None
        return self._apply_out_proj(out.view(total_len, self.d_model)), aux

    @torch.no_grad()
    def _dense_first_sequence(self, q, k, w_sizes, lmk_indices, cu_seqlens):
        """Dense ``[H, T0, T0]`` attention of the first sequence under the hard mask (reference :643-702)."""
        s0, e0 = int(cu_seqlens[0]), int(cu_seqlens[1])
        T0 = e0 - s0
        rows = torch.arange(T0, device=q.device)
        w0 = w_sizes[s0:e0].long()
        in_win = (rows[None, :] >= rows[:, None] - w0[:, None] + 1) & (rows[None, :] <= rows[:, None])
        in_lmk = torch.zeros(self.n_heads, T0, T0, dtype=torch.bool, device=q.device)
        for h in range(self.n_heads):
            vp = lmk_indices[h, 0]
            vp = vp[vp >= 0]
            if vp.numel():
                col = torch.zeros(T0, dtype=torch.bool, device=q.device)
                col[vp] = True
                in_lmk[h] = col[None, :] & (rows[None, :] <= rows[:, None])
        mask = in_win[None] | in_lmk
        k = self._repeat_kv(k)  # k arrives with its kv heads
        sc = torch.matmul(q[s0:e0].transpose(0, 1).float(), k[s0:e0].transpose(0, 1).float().transpose(-2, -1))
        sc = sc / math.sqrt(self.head_dim)
        return torch.softmax(sc.masked_fill(~mask, float("-inf")), dim=-1)
