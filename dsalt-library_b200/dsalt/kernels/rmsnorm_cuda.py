"""CUDA RMSNorm (``dsalt_rmsnorm_fwd`` / ``_bwd`` in ``csrc/rmsnorm.cu``) for the model blocks.

Replaces ``F.rms_norm`` in ``RMSENorm`` (reference ``dsalt/kernels/RMSENorm.py``)
on CUDA tensors with d in ``SUPPORTED_D``: one kernel each way instead of the
fp32 casts, products and reductions torch runs, with the same fp32 arithmetic
(the result rounded once to the input dtype).  The weight gradient is summed
from fixed per-CTA partials (deterministic).  ``add_rms_norm`` also folds in the
residual add in front of the norm (``x + res``, rounded like torch's add) and,
in the backward, the sum of the residual stream's gradient with the norm's.
"""

from __future__ import annotations

import torch

from . import _ext

SUPPORTED_D = (256, 512, 768, 1024)


def _fwd(x2, res2, w32, eps):
    T, d = x2.shape
    y = torch.empty_like(x2)
    rstd = torch.empty(T, dtype=torch.float32, device=x2.device)
    x_sum = torch.empty_like(x2) if res2 is not None else None
    p = _ext.RmsNormParams(x=_ext.ptr(x2), res=_ext.ptr(res2), x_sum=_ext.ptr(x_sum), w=_ext.ptr(w32),
                           y=_ext.ptr(y), rstd=_ext.ptr(rstd), T=T, d=d, eps=float(eps),
                           dtype=_ext.dtype_code(x2.dtype))
    _ext.call("dsalt_rmsnorm_fwd", p)
    return y, rstd, x_sum


def _bwd(xn, w32, rstd, dy, dres, need_dw):
    """(dx, dw fp32 or None) for the normalised input ``xn``; ``dres`` is added to dx."""
    T, d = xn.shape
    dy2 = dy.contiguous().view(-1, d).to(xn.dtype)
    dres2 = dres.contiguous().view(-1, d).to(xn.dtype) if dres is not None else None
    dx = torch.empty_like(xn)
    parts = torch.empty((T + _ext.RMSNORM_ROWS_PER_PART - 1) // _ext.RMSNORM_ROWS_PER_PART, d,
                        dtype=torch.float32, device=xn.device)
    dw = None
    if need_dw:  # zeros for an empty batch (the library then launches nothing)
        dw = torch.empty(d, dtype=torch.float32, device=xn.device) if T > 0 else torch.zeros(d, device=xn.device)
    p = _ext.RmsNormParams(x=_ext.ptr(xn), w=_ext.ptr(w32), rstd=_ext.ptr(rstd), dy=_ext.ptr(dy2),
                           dres=_ext.ptr(dres2), dx=_ext.ptr(dx), dw_part=_ext.ptr(parts), dw=_ext.ptr(dw),
                           T=T, d=d, eps=0.0, dtype=_ext.dtype_code(xn.dtype))
    _ext.call("dsalt_rmsnorm_bwd", p)
    return dx, dw


class RMSNormFunction(torch.autograd.Function):
    """``(x [..., d], weight [d], eps) -> y [..., d]`` in x's dtype."""

    @staticmethod
    def forward(ctx, x, weight, eps: float):
        _ext.require_cuda(x, "x")
        d = x.shape[-1]
        x2 = x.contiguous().view(-1, d)
        w32 = weight.detach().float().contiguous()
        y, rstd, _ = _fwd(x2, None, w32, eps)
        ctx.save_for_backward(x2, w32, rstd)
        ctx.x_shape = x.shape
        ctx.w_dtype = weight.dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w32, rstd = ctx.saved_tensors
        dx, dw = _bwd(x2, w32, rstd, dy, None, ctx.needs_input_grad[1])
        return dx.view(ctx.x_shape), (dw.to(ctx.w_dtype) if dw is not None else None), None


class AddRMSNormFunction(torch.autograd.Function):
    """``(x, res, weight, eps) -> (x + res, rms_norm(x + res))``, both in x's dtype."""

    @staticmethod
    def forward(ctx, x, res, weight, eps: float):
        _ext.require_cuda(x, "x")
        d = x.shape[-1]
        x2 = x.contiguous().view(-1, d)
        r2 = res.contiguous().view(-1, d)
        w32 = weight.detach().float().contiguous()
        y, rstd, x_sum = _fwd(x2, r2, w32, eps)
        ctx.save_for_backward(x_sum, w32, rstd)
        ctx.x_shape = x.shape
        ctx.w_dtype = weight.dtype
        return x_sum.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, d_sum, dy):
        x_sum, w32, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(x_sum)
        dx, dw = _bwd(x_sum, w32, rstd, dy, d_sum, ctx.needs_input_grad[2])
        dx = dx.view(ctx.x_shape)
        return dx, dx, (dw.to(ctx.w_dtype) if dw is not None else None), None


def supported(x: torch.Tensor) -> bool:
    return x.is_cuda and x.shape[-1] in SUPPORTED_D and x.dtype in (torch.bfloat16, torch.float16, torch.float32)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return RMSNormFunction.apply(x, weight, eps)


def add_rms_norm(x: torch.Tensor, res: torch.Tensor, weight: torch.Tensor, eps: float):
    """``(x + res, rms_norm(x + res))`` with one kernel each way (x and res of one dtype and shape)."""
    return AddRMSNormFunction.apply(x, res, weight, eps)
