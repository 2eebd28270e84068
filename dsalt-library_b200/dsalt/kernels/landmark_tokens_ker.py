"""Hybrid-energy landmark score on B200 (module name kept from the reference).

Reference: ``dsalt/kernels/landmark_tokens_ker.py:19-61``.  For token ``j`` and
head ``h``::

    s = α_h · z(‖x_j W_Vᵀ‖_(kv-head of h)) + (1 − α_h) · z(‖x_j‖)

with ``z`` standardising over ALL packed tokens (unbiased std clamped at 1e-6).
The ``x @ W_Vᵀ`` projection is a plain library GEMM (torch/cuBLAS); the norms,
the global statistics and the per-head mix run in one CUDA pipeline
(``dsalt_hybrid_scores``: warp-per-token norms, a single-CTA fp64 reduction,
an elementwise mix).  The result is differentiable in ``x``, ``W_V`` and ``α``
through an analytic backward, as the reference's autograd graph is.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _ext


def _scale_rows(x: torch.Tensor, coef: torch.Tensor, groups: int) -> torch.Tensor:
    """``(coef[:, g, None] · x.float().view(T, groups, -1)).to(x.dtype)`` in one CUDA pass."""
    T, width = x.shape[0], x.shape[1] // groups
    out = torch.empty_like(x)
    p = _ext.ScaleRowsParams(x=_ext.ptr(x), coef=_ext.ptr(coef), out=_ext.ptr(out), T=T, groups=groups,
                             width=width, dtype=_ext.dtype_code(x.dtype))
    _ext.call("dsalt_scale_rows", p)
    return out


class _HybridScore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, xwv, alpha, n_heads: int, n_kv: int, dh: int):
        _ext.require_cuda(x, "x")
        T, d_model = x.shape
        dev = x.device
        x_c = x.contiguous()
        xv = xwv.contiguous().to(x_c.dtype)
        a = alpha.detach().to(device=dev, dtype=torch.float32).contiguous()
        scores = torch.empty(T, n_heads, dtype=torch.float32, device=dev)
        z_x = torch.empty(T, dtype=torch.float32, device=dev)
        z_v = torch.empty(T, n_heads, dtype=torch.float32, device=dev)
        stats = torch.empty(2 + 2 * n_kv, dtype=torch.float32, device=dev)
        norms = torch.empty(1 + n_kv, T, dtype=torch.float32, device=dev)  # column-major (library layout)
        if T > 0:
            p = _ext.ScoreParams(x=_ext.ptr(x_c), xwv=_ext.ptr(xv), alpha=_ext.ptr(a),
                                 scores=_ext.ptr(scores), z_x=_ext.ptr(z_x), z_v=_ext.ptr(z_v),
                                 stats=_ext.ptr(stats), norms=_ext.ptr(norms), T=T,
                                 d_model=d_model, H=n_heads, n_kv=n_kv, dh=dh,
                                 dtype=_ext.dtype_code(x_c.dtype))
            _ext.call("dsalt_hybrid_scores", p)
        ctx.save_for_backward(x_c, xv, a, norms, stats, z_x, z_v)
        ctx.shape = (n_heads, n_kv, dh)
        ctx.alpha_dtype = alpha.dtype
        ctx.mark_non_differentiable(z_x, z_v)
        return scores, z_x, z_v

    @staticmethod
    def backward(ctx, g_s, g_zx, g_zv):
        x_c, xv, a, norms_cm, stats, z_x, z_v = ctx.saved_tensors
        H, n_kv, dh = ctx.shape
        T = x_c.shape[0]
        dev = x_c.device
        if T == 0:
            return None, None, torch.zeros(H, dtype=ctx.alpha_dtype, device=dev), None, None, None
        g = (g_s.float().contiguous() if g_s is not None else torch.zeros(T, H, device=dev))
        # the chain through the z-scores in one CUDA pass pair (dsalt_hybrid_scores_bwd):
        # d alpha and the per-row coefficients of d‖r‖/dr = r/‖r‖
        d_alpha = torch.empty(H, dtype=torch.float32, device=dev)
        coef_x = torch.empty(T, dtype=torch.float32, device=dev)
        coef_v = torch.empty(T, n_kv, dtype=torch.float32, device=dev)
        sums = torch.empty(2 * (1 + n_kv), dtype=torch.float32, device=dev)
        parts = torch.empty((T + _ext.SCORE_BWD_TOKENS - 1) // _ext.SCORE_BWD_TOKENS, 2 * (1 + n_kv) + H,
                            dtype=torch.float32, device=dev)
        p = _ext.ScoreBwdParams(g_s=_ext.ptr(g), alpha=_ext.ptr(a), z_x=_ext.ptr(z_x), z_v=_ext.ptr(z_v),
                                norms=_ext.ptr(norms_cm), stats=_ext.ptr(stats), sums=_ext.ptr(sums),
                                partials=_ext.ptr(parts), d_alpha=_ext.ptr(d_alpha), coef_x=_ext.ptr(coef_x),
                                coef_v=_ext.ptr(coef_v), T=T, H=H, n_kv=n_kv)
        _ext.call("dsalt_hybrid_scores_bwd", p)
        dx = dxwv = None
        # each row (group) of x / x·W_Vᵀ scaled by its coefficient, the fp32 product
        # rounded once to the dtype (dsalt_scale_rows)
        if ctx.needs_input_grad[0]:
            dx = _scale_rows(x_c, coef_x, 1)
        if ctx.needs_input_grad[1]:
            dxwv = _scale_rows(xv, coef_v, n_kv)
        return dx, dxwv, d_alpha.to(ctx.alpha_dtype), None, None, None


def hybrid_scores_per_head(
    x:       torch.Tensor,
    W_V:     torch.Tensor,
    alpha:   torch.Tensor,
    n_heads: int,
    dh:      int,
    xwv:     torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Per-head hybrid score and the standardised signals (reference :19-61).

    Returns ``(scores [T, n_heads], z_x [T], z_v [T, n_heads])`` in fp32.  Under
    GQA (``W_V`` has ``n_kv_heads·dh`` rows) the kv-head value norm is shared by
    the query heads of its group.  ``xwv`` (``[T, n_kv·dh]``) may pass the value
    projection the caller already has: without a bias ``x·W_Vᵀ`` is exactly the
    pre-RoPE ``v``, so the ``T·d·n_kv·dh`` GEMM is not repeated.
    """
    n_kv = W_V.shape[0] // dh
    if n_heads % n_kv != 0:
        raise ValueError(f"n_heads={n_heads} is not a multiple of n_kv={n_kv}")
    if xwv is None:
        xwv = x @ W_V.T.to(x.dtype)  # library GEMM; autocast gives the reference's bf16 product
    elif xwv.shape != (x.shape[0], W_V.shape[0]):
        raise ValueError(f"xwv must be [T, {W_V.shape[0]}], got {tuple(xwv.shape)}")
    return _HybridScore.apply(x, xwv, alpha, n_heads, n_kv, dh)


def compute_hybrid_scores(x: torch.Tensor, W_V: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
    """Historical ``(x, W_V, alpha)`` signature (reference :64-85)."""
    if alpha.ndim == 0:
        x_norm = x.norm(dim=-1)
        xwv = (x @ W_V.T).norm(dim=-1)
        mu_x, std_x = x_norm.mean(), x_norm.std().clamp(min=1e-6)
        mu_v, std_v = xwv.mean(), xwv.std().clamp(min=1e-6)
        return alpha * (xwv - mu_v) / std_v + (1.0 - alpha) * (x_norm - mu_x) / std_x
    n_heads = alpha.shape[0]
    dh = W_V.shape[0] // n_heads
    scores, _, _ = hybrid_scores_per_head(x, W_V, alpha, n_heads, dh)
    return scores


def select_landmarks(scores: torch.Tensor, k: int, exclude_mask: torch.Tensor | None = None) -> torch.Tensor:
    """Top-k landmarks from the scores, optionally excluding the local window (reference :88-104)."""
    if exclude_mask is not None:
        scores = scores.masked_fill(exclude_mask, float("-inf"))
    n_valid = int((scores != float("-inf")).sum())
    k_actual = min(k, n_valid)
    if k_actual == 0:
        return torch.empty(0, dtype=torch.long, device=scores.device)
    _, indices = torch.topk(scores, k=k_actual, dim=-1, sorted=False)
    return indices


def soft_landmark_weights(scores: torch.Tensor, k: int, exclude_mask: torch.Tensor | None = None,
                          temperature: float = 1.0) -> torch.Tensor:
    """Temperature-scaled softmax weights over the candidates (reference :107-117)."""
    if exclude_mask is not None:
        scores = scores.masked_fill(exclude_mask, float("-inf"))
    return torch.softmax(scores / temperature, dim=-1)


class HybridEnergyLandmarkSelector(nn.Module):
    """Landmark selector with a learnable ``alpha`` ``[n_layers, n_heads]`` (reference :120-147)."""

    def __init__(self, n_layers: int, n_heads: int):
        super().__init__()
        self.alpha = nn.Parameter(torch.full((n_layers, n_heads), torch.logit(torch.tensor(0.6)).item()))

    def forward(self, x, W_V, layer_idx, head_idx, k, window_mask):
        alpha = torch.sigmoid(self.alpha[layer_idx, head_idx])
        scores = compute_hybrid_scores(x, W_V, alpha)
        in_win = window_mask.any(dim=0)
        indices = select_landmarks(scores, k=k, exclude_mask=in_win)
        weights = soft_landmark_weights(scores, k=k, exclude_mask=in_win)
        return indices, weights
