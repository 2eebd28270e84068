"""DSALT inference attention op on B200 (module name kept from the reference).

Drop-in for ``dsalt/kernels/dsalt_triton_attn.py``: ``DSALTAttentionFunction``
and ``dsalt_triton_attention(q, k, v, lmk_indices, lmk_bias, w_sizes,
cu_seqlens)`` with the reference semantics (``_dsalt_fwd_kernel``,
dsalt_triton_attn.py:27-169): integer window ``[i − w + 1, i]`` with
``w = max(int(w_sizes), 1)``, landmarks ``p ≤ i`` and ``p < i − w + 1``, additive
``lmk_bias``.  The backward returns ``(dq, dk, dv, None, d_bias, None, None)``
(dsalt_triton_attn.py:325-328), computed without atomics.

The selector helpers are re-exported here as in the reference (:18-24).
"""

from __future__ import annotations

import torch

from . import _ext
from . import dsalt_cuda as _cuda
from .selectors import (  # noqa: F401  (re-exported like the reference)
    _seq_meta,
    _build_seq_block_map,
    _score_block,
    _compute_landmark_indices,
    _build_landmark_kv,
)
from .dsalt_triton_train import _host_cu, _validate_cu


class DSALTAttentionFunction(torch.autograd.Function):
    """Autograd Function with the reference signature (dsalt_triton_attn.py:257-328)."""

    @staticmethod
    def forward(ctx, q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens):
        _cuda.check_inputs(q, k, v, cu_seqlens)
        cu_host = _host_cu(cu_seqlens, None)
        _validate_cu(cu_host, q.shape[0])
        dt = _cuda.compute_dtype(q)
        q_c = q.contiguous().to(dt)
        k_c = k.contiguous().to(dt)
        v_c = v.contiguous().to(dt)
        impl = _ext.default_impl()
        with torch.no_grad():
            prep = _cuda.prepare(k_c, v_c, lmk_indices, lmk_bias, w_sizes, cu_seqlens, _ext.INFER,
                                 cu_host=cu_host, for_backward=any(ctx.needs_input_grad))
            o, o_f32, lse = _cuda.forward(q_c, k_c, v_c, prep, 1.0, 0.0, impl)
        ctx.save_for_backward(q_c, k_c, v_c, o, lse)
        ctx.prep = prep
        ctx.impl = impl
        ctx.out_dtype = q.dtype
        return o_f32

    @staticmethod
    def backward(ctx, grad_out):
        q_c, k_c, v_c, o, lse = ctx.saved_tensors
        dq, dk, dv, d_bias, _ = _cuda.backward(grad_out, q_c, k_c, v_c, o, lse, ctx.prep, 1.0, 0.0,
                                               ctx.impl, want_dw=False)
        od = ctx.out_dtype
        # d_bias: fp32 holding the values of the reference's d_bias.to(out_dtype)
        return dq.to(od), dk.to(od), dv.to(od), None, d_bias, None, None


def _dynamo_opaque(fn):
    disable = getattr(getattr(torch, "_dynamo", None), "disable", None)
    return disable(fn) if disable is not None else fn


@_dynamo_opaque
def dsalt_triton_attention(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens):
    """Hard-selector sparse attention (reference dsalt_triton_attn.py:337-349).

    Returns ``O`` ``[T, H, D]`` float32.
    """
    return DSALTAttentionFunction.apply(q, k, v, lmk_indices, lmk_bias, w_sizes, cu_seqlens)
