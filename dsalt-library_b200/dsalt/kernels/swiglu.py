"""SwiGLU feed-forward block with one gate+up GEMM and a CUDA activation.

The reference block (``dsalt/modules/dsalt_transformer.py:10-21``) computes
``down_proj(silu(gate_proj(x)) * up_proj(x))``: under autocast two GEMMs, then
``silu``, a product, and in the backward the two products, ``silu_backward``, two
input-gradient GEMMs and their sum.  Here the gate and up weights are stacked
into one ``[2F, d]`` operand, so the forward is one GEMM giving ``[T, 2F]``
(gate half, up half) and the backward one GEMM for ``dx`` and one for both weight
gradients; the activation and its gradient are one CUDA pass each
(``dsalt_swiglu_fwd`` / ``dsalt_swiglu_bwd`` in ``csrc/swiglu.cu``, torch's
rounding of the replaced elementwise ops).  The weight gradients come out of the
GEMMs in fp32 (the reference rounds them to the compute dtype first); ``dx`` is
one GEMM over ``K = 2F`` instead of the sum of two rounded halves.
"""

from __future__ import annotations

import torch

from . import _ext


def _act(gu: torch.Tensor, F: int) -> torch.Tensor:
    T = gu.shape[0]
    h = torch.empty(T, F, dtype=gu.dtype, device=gu.device)
    p = _ext.SwigluParams(g=_ext.ptr(gu), u=_ext.ptr(gu[:, F:]), h=_ext.ptr(h), T=T, F=F, ld_in=2 * F, ld_out=2 * F,
                          dtype=_ext.dtype_code(gu.dtype))
    _ext.call("dsalt_swiglu_fwd", p)
    return h


def _act_bwd(gu: torch.Tensor, dh: torch.Tensor, F: int) -> torch.Tensor:
    T = gu.shape[0]
    dgu = torch.empty_like(gu)
    p = _ext.SwigluParams(g=_ext.ptr(gu), u=_ext.ptr(gu[:, F:]), dh=_ext.ptr(dh), dg=_ext.ptr(dgu),
                          du=_ext.ptr(dgu[:, F:]), T=T, F=F, ld_in=2 * F, ld_out=2 * F,
                          dtype=_ext.dtype_code(gu.dtype))
    _ext.call("dsalt_swiglu_bwd", p)
    return dgu


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """``R(R(silu(g))·u)`` for 16-bit ``[T, F]`` tensors (forward only, no autograd)."""
    _ext.require_cuda(g, "g")
    if g.shape != u.shape or g.dtype != u.dtype or g.dim() != 2:
        raise ValueError("g and u must be [T, F] tensors of one dtype")
    gu = torch.cat([g, u], dim=1)
    return _act(gu, g.shape[1])


class SwiGLUFFNFunction(torch.autograd.Function):
    """``(x [T, d], w_gate [F, d], w_up [F, d], w_down [d, F], dtype) -> [T, d]`` in ``dtype``."""

    @staticmethod
    def forward(ctx, x, w_gate, w_up, w_down, dtype: torch.dtype):
        _ext.require_cuda(x, "x")
        F, d = w_gate.shape
        lead = x.shape[:-1]
        x2 = x.reshape(-1, d).to(dtype).contiguous()
        w_gu = torch.empty(2 * F, d, dtype=dtype, device=x.device)
        w_gu[:F].copy_(w_gate.detach())
        w_gu[F:].copy_(w_up.detach())
        w_d = w_down.detach().to(dtype)
        gu = torch.mm(x2, w_gu.t())
        h = _act(gu, F)
        out = torch.mm(h, w_d.t())
        ctx.save_for_backward(x2, w_gu, w_d, gu, h)
        ctx.lead, ctx.F = lead, F
        ctx.dtypes = (x.dtype, w_gate.dtype, w_up.dtype, w_down.dtype)
        return out.view(*lead, d)

    @staticmethod
    def backward(ctx, dout):
        x2, w_gu, w_d, gu, h = ctx.saved_tensors
        F = ctx.F
        d = x2.shape[1]
        x_dt, wg_dt, wu_dt, wd_dt = ctx.dtypes
        dout2 = dout.reshape(-1, d).to(x2.dtype).contiguous()
        dh = torch.mm(dout2, w_d)
        dgu = _act_bwd(gu, dh, F)
        dx = dw_g = dw_u = dw_d = None
        if ctx.needs_input_grad[0]:
            dx = torch.mm(dgu, w_gu).to(x_dt).view(*ctx.lead, d)
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            dw_gu = torch.mm(dgu.t(), x2, out_dtype=torch.float32)
            dw_g, dw_u = dw_gu[:F].to(wg_dt), dw_gu[F:].to(wu_dt)
        if ctx.needs_input_grad[3]:
            dw_d = torch.mm(dout2.t(), h, out_dtype=torch.float32).to(wd_dt)
        return dx, dw_g, dw_u, dw_d, None


def supported(x: torch.Tensor, w_gate: torch.Tensor) -> bool:
    """CUDA input and an intermediate width that splits into 16-byte pieces."""
    return x.is_cuda and w_gate.shape[0] % 8 == 0


def swiglu_ffn(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor,
               dtype: torch.dtype) -> torch.Tensor:
    """``down(silu(gate(x)) * up(x))`` computed in ``dtype`` (f16 / bf16), bias-free."""
    return SwiGLUFFNFunction.apply(x, w_gate, w_up, w_down, dtype)
