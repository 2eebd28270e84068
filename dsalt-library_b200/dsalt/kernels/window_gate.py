"""Adaptive window gate ``w̃ = n_min + σ(x·W + b)·(n_max − n_min)`` on B200.

Reference: ``DSALTAttention._window_continuous`` (dsalt/modules/dsalt_attention.py:270-275),
an ``nn.Linear(d_model, 1)`` followed by torch elementwise ops.  Here one CUDA
kernel (``dsalt_win_gate``: one warp per token, fp32 accumulation) computes the
logit and the whole elementwise chain with the rounding torch applies under
autocast (each op rounded to the compute dtype), so the window equals the
reference's bit for bit at equal logits.  The backward is analytic:
``∂w̃/∂logit = (n_max − n_min)·σ·(1 − σ)``; in 16-bit compute the rank-one
products ``dx = dl ⊗ w`` and ``dW = Σ_t dl·x`` run as one CUDA pass
(``dsalt_win_gate_bwd``).
"""

from __future__ import annotations

import torch

from . import _ext


def _compute_dtype(x: torch.Tensor) -> torch.dtype:
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


class _WinGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, n_min: float, n_max: float):
        _ext.require_cuda(x, "x")
        dt = _compute_dtype(x)
        T, d = x.shape
        xc = x.contiguous().to(dt)
        wc = weight.reshape(-1).contiguous().to(dt)
        bc = (bias.reshape(-1) if bias is not None else torch.zeros(1, device=x.device)).contiguous().to(dt)
        w_cont = torch.empty(T, dtype=dt, device=x.device)
        logits = torch.empty(T, dtype=torch.float32, device=x.device)
        if T > 0:
            p = _ext.WinGateParams(x=_ext.ptr(xc), weight=_ext.ptr(wc), bias=_ext.ptr(bc),
                                   w_cont=_ext.ptr(w_cont), w_f32=0, w_disc=0, logits=_ext.ptr(logits),
                                   T=T, d_model=d, n_min=float(n_min), n_max=float(n_max),
                                   dtype=_ext.dtype_code(dt))
            _ext.call("dsalt_win_gate", p)
        ctx.save_for_backward(xc, wc, logits)
        ctx.span = float(n_max - n_min)
        ctx.dtypes = (x.dtype, weight.dtype, bias.dtype if bias is not None else None)
        ctx.has_bias = bias is not None
        return w_cont

    @staticmethod
    def backward(ctx, g):
        xc, wc, logits = ctx.saved_tensors
        sg = torch.sigmoid(logits)
        dl = g.float() * ctx.span * sg * (1.0 - sg)                      # [T]
        need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        T, d = xc.shape
        if xc.dtype != torch.float32 and d % 8 == 0 and T > 0 and (need_dx or need_dw):
            # one CUDA pass: dx = dl ⊗ w rounded to the dtype, dW as row-block partials
            dl = dl.contiguous()
            dx = torch.empty_like(xc) if need_dx else None
            parts = (torch.empty((T + _ext.WIN_GATE_ROWS_PER_PART - 1) // _ext.WIN_GATE_ROWS_PER_PART, d,
                                 dtype=torch.float32, device=xc.device) if need_dw else None)
            p = _ext.WinGateBwdParams(x=_ext.ptr(xc), weight=_ext.ptr(wc), dl=_ext.ptr(dl),
                                      dx=_ext.ptr(dx) if need_dx else 0, dw_part=_ext.ptr(parts) if need_dw else 0,
                                      T=T, d_model=d, dtype=_ext.dtype_code(xc.dtype))
            _ext.call("dsalt_win_gate_bwd", p)
            dx = dx.to(ctx.dtypes[0]) if need_dx else None
            dw = parts.sum(0, keepdim=True).to(ctx.dtypes[1]) if need_dw else None
        else:
            dx = (dl[:, None] * wc.float()[None, :]).to(ctx.dtypes[0]) if need_dx else None
            dw = (dl[None, :] @ xc.float()).to(ctx.dtypes[1]) if need_dw else None
        db = dl.sum().reshape(1).to(ctx.dtypes[2]) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
        return dx, dw, db, None, None


def window_continuous(x: torch.Tensor, linear: torch.nn.Linear, n_min: float, n_max: float) -> torch.Tensor:
    """``[T]`` continuous window in the compute dtype, differentiable in ``x`` and ``linear``."""
    return _WinGate.apply(x, linear.weight, linear.bias, float(n_min), float(n_max))
