"""Fused attention prologue: RoPE on q and k plus (optionally) the GQA expansion of k and v.

With ``expand=False`` k and v keep their ``H_kv`` heads: the attention op reads
the kv head of each query head in place (``DsaltAttnParams.H_kv``), so the
expansion is never written.

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
    """``(q [T,H,D], k [T,Hkv,D], v [T,Hkv,D], cos [T,D], sin [T,D]) -> (q_rot, k_rot [T,H,D], v [T,H,D])``,
    or with ``expand=False`` ``(q_rot, k_rot [T,Hkv,D], v)``."""

    @staticmethod
    def forward(ctx, q, k, v, cos, sin, expand_kv: bool = True):
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
        expand = H != Hkv and expand_kv
        k_out = torch.empty(T, H if expand else Hkv, D, dtype=k.dtype, device=k.device)
        v_out = torch.empty(T, H, D, dtype=v.dtype, device=v.device) if expand else None
        p = _params(q, k, cos, sin, q=q, k=k, v=v if expand else None, q_out=q_out, k_out=k_out, v_out=v_out)
        p.kv_out_heads = H if expand else Hkv
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
        hk_out = H if ctx.expand else ctx.hkv
        dq_out = torch.zeros(T, H, D, dtype=dt, device=dev) if dq_out is None else dq_out.contiguous()
        dk_out = torch.zeros(T, hk_out, D, dtype=dt, device=dev) if dk_out is None else dk_out.contiguous()
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
        p.kv_out_heads = hk_out
        _ext.call("dsalt_rope_gqa_bwd", p)
        return dq, dk, dv, None, None, None


def rope_gqa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
             expand: bool = True):
    """RoPE on q and k and (``expand``) the expansion of k and v to q's heads, fused
    (see the module docstring)."""
    return RopeGqaFunction.apply(q, k, v, cos, sin, expand)


class QkvRopeFunction(torch.autograd.Function):
    """The q/k/v projections (bias-free) plus the prologue, with one GEMM each way.

    ``(x [T, d], w_q [H·D, d], w_k [Hkv·D, d], w_v [Hkv·D, d], cos, sin, H, Hkv, D,
    dtype) -> (q_rot, k_rot, v)`` ([T, H, D] each, k and v expanded to the query
    heads), plus under GQA the unexpanded value projection ``[T, Hkv·D]`` as a
    fourth output.  The three weights are stacked into one ``[(H + 2·Hkv)·D, d]``
    operand, so the forward is one GEMM whose ``[T, (H + 2·Hkv)·D]`` output the
    prologue kernel reads in column blocks (``ld``); the backward writes dq, dk and
    dv into one such buffer and runs one GEMM for dx and one for the three weight
    gradients (fp32 out).  The rotation and expansion round as in ``rope_gqa``;
    dx is one GEMM over all three blocks instead of the sum of three rounded ones.
    """

    @staticmethod
    def forward(ctx, x, w_q, w_k, w_v, cos, sin, H: int, Hkv: int, D: int, dtype: torch.dtype,
                expand_kv: bool = True):
        _ext.require_cuda(x, "x")
        T, d = x.shape
        nq, nk = H * D, Hkv * D
        W = nq + 2 * nk
        dev = x.device
        x2 = x.to(dtype).contiguous()
        w = torch.empty(W, d, dtype=dtype, device=dev)
        w[:nq].copy_(w_q.detach())
        w[nq:nq + nk].copy_(w_k.detach())
        w[nq + nk:].copy_(w_v.detach())
        qkv = torch.mm(x2, w.t())
        cos, sin = cos.to(dtype).contiguous(), sin.to(dtype).contiguous()
        expand = expand_kv and H != Hkv
        hk = H if expand else Hkv  # heads of k_out and v_out
        q_out = torch.empty(T, H, D, dtype=dtype, device=dev)
        k_out = torch.empty(T, hk, D, dtype=dtype, device=dev)
        v_out = torch.empty(T, hk, D, dtype=dtype, device=dev)
        p = _ext.RopeParams(q=_ext.ptr(qkv), k=_ext.ptr(qkv[:, nq:]), v=_ext.ptr(qkv[:, nq + nk:]), cos=_ext.ptr(cos),
                            sin=_ext.ptr(sin), q_out=_ext.ptr(q_out), k_out=_ext.ptr(k_out), v_out=_ext.ptr(v_out),
                            T=T, ld=W, H=H, Hkv=Hkv, D=D, dtype=_ext.dtype_code(dtype), kv_out_heads=hk)
        if T > 0:
            _ext.call("dsalt_rope_gqa_fwd", p)
        ctx.save_for_backward(x2, w, cos, sin)
        ctx.dims = (H, Hkv, D, hk)
        ctx.dtypes = (x.dtype, w_q.dtype, w_k.dtype, w_v.dtype)
        if not expand:
            return q_out, k_out, v_out
        return q_out, k_out, v_out, qkv[:, nq + nk:].contiguous()

    @staticmethod
    def backward(ctx, dq_out, dk_out, dv_out, *d_xwv):
        x2, w, cos, sin = ctx.saved_tensors
        H, Hkv, D, hk = ctx.dims
        T, d = x2.shape
        nq, nk = H * D, Hkv * D
        W = nq + 2 * nk
        dt, dev = x2.dtype, x2.device

        def dense(g, heads):
            return torch.zeros(T, heads, D, dtype=dt, device=dev) if g is None else g.contiguous().to(dt)
        dq_out, dk_out, dv_out = dense(dq_out, H), dense(dk_out, hk), dense(dv_out, hk)
        dqkv = torch.empty(T, W, dtype=dt, device=dev)
        p = _ext.RopeParams(cos=_ext.ptr(cos), sin=_ext.ptr(sin), dq_out=_ext.ptr(dq_out), dk_out=_ext.ptr(dk_out),
                            dv_out=_ext.ptr(dv_out), dq=_ext.ptr(dqkv), dk=_ext.ptr(dqkv[:, nq:]),
                            dv=_ext.ptr(dqkv[:, nq + nk:]), T=T, ld=W, H=H, Hkv=Hkv, D=D,
                            dtype=_ext.dtype_code(dt), kv_out_heads=hk)
        if T > 0:
            _ext.call("dsalt_rope_gqa_bwd", p)
        if d_xwv and d_xwv[0] is not None:
            dqkv[:, nq + nk:] += d_xwv[0].to(dt)
        x_dt, wq_dt, wk_dt, wv_dt = ctx.dtypes
        dx = torch.mm(dqkv, w).to(x_dt) if ctx.needs_input_grad[0] else None
        dw_q = dw_k = dw_v = None
        if any(ctx.needs_input_grad[1:4]):
            dw = torch.mm(dqkv.t(), x2, out_dtype=torch.float32)
            dw_q, dw_k, dw_v = dw[:nq].to(wq_dt), dw[nq:nq + nk].to(wk_dt), dw[nq + nk:].to(wv_dt)
        return dx, dw_q, dw_k, dw_v, None, None, None, None, None, None, None


def qkv_rope(x, w_q, w_k, w_v, cos, sin, H: int, Hkv: int, D: int, dtype: torch.dtype, expand: bool = True):
    """``(q_rot, k_rot, v, xwv)``: the bias-free q/k/v projections of ``x`` [T, d] in
    ``dtype`` with RoPE and (``expand``) the GQA expansion fused (see
    ``QkvRopeFunction``); ``xwv`` [T, Hkv·D] is the unexpanded value projection (a
    view of ``v`` when v is not expanded)."""
    out = QkvRopeFunction.apply(x, w_q, w_k, w_v, cos, sin, H, Hkv, D, dtype, expand)
    if H == Hkv or not expand:
        q, k, v = out
        return q, k, v, v.view(x.shape[0], Hkv * D)
    return out
