"""Fused attention prologue: RoPE on q and k plus the GQA expansion of k and v.

One CUDA pass (``dsalt_rope_gqa_fwd`` / ``dsalt_rope_gqa_bwd`` in ``csrc/rope.cu``)
replaces, on the packed path of ``DSALTAttention``, the reference's
``apply_rotary_emb`` (``dsalt/kernels/window_utils.py:73-88``) on q and k and
``_repeat_kv`` (``dsalt/modules/dsalt_attention.py:254-268``) on k and v.  The
forward rounds like those tensor ops (bitwise equal results); the backward
returns the gradients of the same expressions.  There is no CPU path: CPU
tensors raise.
"""

from __future__ import annotations

import torch

from . import _ext


def _params(rows, kv_rows, cos, sin, **bufs) -> _ext.RopeParams:
    """Sizes from ``rows`` ([T, H, D]) and ``kv_rows`` ([T, Hkv, D]); ``bufs`` name the pointers."""
    T, H, D = rows.shape
    p = _ext.RopeParams(cos=_ext.ptr(cos), sin=_ext.ptr(sin), T=T, H=H, Hkv=kv_rows.shape[1], D=D,
                        dtype=_ext.dtype_code(rows.dtype))
    for name, t in bufs.items():
        setattr(p, name, _ext.ptr(t))
    return p


class RopeGqaFunction(torch.autograd.Function):
    """``(q [T,H,D], k [T,Hkv,D], v [T,Hkv,D], cos [T,D], sin [T,D]) -> (q_rot, k_rot [T,H,D], v [T,H,D])``."""

    @staticmethod
    def forward(ctx, q, k, v, cos, sin):
        for name, t in (("q", q), ("k", k), ("v", v), ("cos", cos), ("sin", sin)):
            _ext.require_cuda(t, name)
        if not (q.dtype == k.dtype == v.dtype == cos.dtype == sin.dtype):
            raise TypeError("q, k, v, cos and sin must share one dtype")
        T, H, D = q.shape
        Hkv = k.shape[1]
        if k.shape != (T, Hkv, D) or v.shape != k.shape or cos.shape != (T, D) or sin.shape != (T, D):
            raise ValueError("expected q [T,H,D], k/v [T,Hkv,D], cos/sin [T,D]")
        if H % Hkv != 0:
            raise ValueError("H must be a multiple of the number of kv heads")
        q, k, v, cos, sin = (t.contiguous() for t in (q, k, v, cos, sin))
        q_out = torch.empty_like(q)
        k_out = torch.empty(T, H, D, dtype=k.dtype, device=k.device)
        expand = H != Hkv
        v_out = torch.empty(T, H, D, dtype=v.dtype, device=v.device) if expand else None
        p = _params(q, k, cos, sin, q=q, k=k, v=v if expand else None, q_out=q_out, k_out=k_out, v_out=v_out)
        _ext.call("dsalt_rope_gqa_fwd", p)
        ctx.save_for_backward(cos, sin)
        ctx.hkv = Hkv
        ctx.expand = expand
        # without expansion v passes through unchanged, as in the reference
        return q_out, k_out, (v_out if expand else v.view_as(v))

    @staticmethod
    def backward(ctx, dq_out, dk_out, dv_out):
        cos, sin = ctx.saved_tensors
        T, D = cos.shape
        ref = dq_out if dq_out is not None else dk_out
        H = ref.shape[1]
        dev, dt = cos.device, cos.dtype
        dq_out = torch.zeros(T, H, D, dtype=dt, device=dev) if dq_out is None else dq_out.contiguous()
        dk_out = torch.zeros(T, H, D, dtype=dt, device=dev) if dk_out is None else dk_out.contiguous()
        dq = torch.empty(T, H, D, dtype=dt, device=dev)
        dk = torch.empty(T, ctx.hkv, D, dtype=dt, device=dev)
        dv = None
        if ctx.expand:
            dv_out = torch.zeros(T, H, D, dtype=dt, device=dev) if dv_out is None else dv_out.contiguous()
            dv = torch.empty(T, ctx.hkv, D, dtype=dt, device=dev)
            p = _params(dq_out, dk, cos, sin, dq_out=dq_out, dk_out=dk_out, dv_out=dv_out, dq=dq, dk=dk, dv=dv)
        else:
            dv = dv_out
            p = _params(dq_out, dk, cos, sin, dq_out=dq_out, dk_out=dk_out, dq=dq, dk=dk)
        _ext.call("dsalt_rope_gqa_bwd", p)
        return dq, dk, dv, None, None


def rope_gqa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """RoPE on q and k and the expansion of k and v to q's heads, fused (see the module docstring)."""
    return RopeGqaFunction.apply(q, k, v, cos, sin)
