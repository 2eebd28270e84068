"""CUDA RMSNorm (``dsalt_rmsnorm_fwd`` / ``_bwd`` in ``csrc/rmsnorm.cu``) for the model blocks.

Replaces ``F.rms_norm`` in ``RMSENorm`` (reference ``dsalt/kernels/RMSENorm.py``)
on CUDA tensors with d in ``SUPPORTED_D``: one kernel each way instead of the
fp32 casts, products and reductions torch runs, with the same fp32 arithmetic
(the result rounded once to the input dtype).  The weight gradient is summed
from fixed per-CTA partials (deterministic).
"""

from __future__ import annotations

import torch

from . import _ext

SUPPORTED_D = (256, 512, 768, 1024)


class RMSNormFunction(torch.autograd.Function):
    """``(x [..., d], weight [d], eps) -> y [..., d]`` in x's dtype."""

    @staticmethod
    def forward(ctx, x, weight, eps: float):
        _ext.require_cuda(x, "x")
        d = x.shape[-1]
        x2 = x.contiguous().view(-1, d)
        T = x2.shape[0]
        w32 = weight.detach().float().contiguous()
        y = torch.empty_like(x2)
        rstd = torch.empty(T, dtype=torch.float32, device=x.device)
        p = _ext.RmsNormParams(x=_ext.ptr(x2), w=_ext.ptr(w32), y=_ext.ptr(y), rstd=_ext.ptr(rstd), T=T, d=d,
                               eps=float(eps), dtype=_ext.dtype_code(x.dtype))
        _ext.call("dsalt_rmsnorm_fwd", p)
        ctx.save_for_backward(x2, w32, rstd)
        ctx.x_shape = x.shape
        ctx.w_dtype = weight.dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w32, rstd = ctx.saved_tensors
        T, d = x2.shape
        dy2 = dy.contiguous().view(-1, d).to(x2.dtype)
        dx = torch.empty_like(x2)
        parts = torch.empty((T + _ext.RMSNORM_ROWS_PER_PART - 1) // _ext.RMSNORM_ROWS_PER_PART, d,
                            dtype=torch.float32, device=x2.device)
        p = _ext.RmsNormParams(x=_ext.ptr(x2), w=_ext.ptr(w32), rstd=_ext.ptr(rstd), dy=_ext.ptr(dy2),
                               dx=_ext.ptr(dx), dw_part=_ext.ptr(parts), T=T, d=d, eps=0.0,
                               dtype=_ext.dtype_code(x2.dtype))
        _ext.call("dsalt_rmsnorm_bwd", p)
        dw = parts.sum(0).to(ctx.w_dtype) if ctx.needs_input_grad[1] else None
        return dx.view(ctx.x_shape), dw, None


def supported(x: torch.Tensor) -> bool:
    return x.is_cuda and x.shape[-1] in SUPPORTED_D and x.dtype in (torch.bfloat16, torch.float16, torch.float32)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return RMSNormFunction.apply(x, weight, eps)
