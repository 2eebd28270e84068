"""DSALT training attention op on B200 (module name kept from the reference).

Drop-in for ``dsalt/kernels/dsalt_triton_train.py`` of the reference: the same
``DSALTTrainFunction`` signature (11 positional arguments, 11 gradients) and the
same public wrapper ``dsalt_triton_train_attention``.  The kernels are
hand-written sm_100a CUDA behind the C ABI of ``libdsalt_b200.so``; there is no
Triton and no CPU fallback.

Semantics (reference ``_train_fwd_kernel``, dsalt_triton_train.py:116-214):
query ``i`` attends the band ``0 ≤ i − j ≤ w̃(i)`` with the soft-edge log-bias
``log σ((w̃ − d)/τ_win)`` outside the core ``d ≤ w̃ − win_edge``, plus the
landmarks ``p`` of its (head, sequence) with ``p ≤ i`` and ``p < i − w̃(i)``,
biased by ``lmk_logw``.  The backward returns ``d_w̃`` (summed over heads) and
``d_logw``, which autograd carries to ``win_gate`` and ``α``.

Differences from the reference, all deliberate:
  * fp32 inputs are computed in exact fp32 (SIMT kernels) instead of being cast
    to fp16 (reference :601-604), so fp32 results match the fp32 dense path;
  * the key-parallel dK/dV scan covers each sequence's actual largest window,
    so gradients stay exact even when ``w̃ > n_max`` (the reference bounds the
    scan with ``n_max``, :439-444); ``n_max`` is accepted and unused;
  * landmark dK/dV/d_logw and d_w̃ are accumulated without atomics, so the
    backward is bitwise deterministic (reference :327-333, :382-383);
  * no autotune: tile shapes are fixed for B200 (see ``autotune``).
"""

from __future__ import annotations

import torch

from . import _ext
from . import dsalt_cuda as _cuda


def _host_cu(cu_seqlens: torch.Tensor, cu_list):
    if cu_list is not None:
        return [int(c) for c in cu_list]
    return [int(c) for c in cu_seqlens.detach().to("cpu").tolist()]


def _validate_cu(cu, T: int) -> None:
    if len(cu) < 1 or cu[0] != 0 or cu[-1] != T:
        raise ValueError(f"cu_seqlens must start at 0 and end at T={T}, got {cu[:1]}..{cu[-1:]}")
    for a, b in zip(cu[:-1], cu[1:]):
        if b < a:
            raise ValueError("cu_seqlens must be non-decreasing")


def _train_forward(ctx, q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge, cu_list, f32_out):
    _cuda.check_inputs(q, k, v, cu_seqlens)
    total_len = q.shape[0]
    cu_host = _host_cu(cu_seqlens, cu_list)
    _validate_cu(cu_host, total_len)
    dt = _cuda.compute_dtype(q)
    q_c = q.contiguous().to(dt)
    k_c = k.contiguous().to(dt)
    v_c = v.contiguous().to(dt)
    impl = _ext.default_impl()
    with torch.no_grad():
        prep = _cuda.prepare(k_c, v_c, lmk_pos, lmk_logw, w_cont, cu_seqlens, _ext.TRAIN, cu_host=cu_host,
                             for_backward=any(ctx.needs_input_grad))
        o, o_out, lse = _cuda.forward(q_c, k_c, v_c, prep, float(tau_win), float(win_edge), impl, f32_out=f32_out)
    ctx.save_for_backward(q_c, k_c, v_c, o, lse)
    ctx.prep = prep
    ctx.tau_win = float(tau_win)
    ctx.win_edge = float(win_edge)
    ctx.impl = impl
    ctx.out_dtype = q.dtype
    return o_out


def _train_backward(ctx, grad_out):
    q_c, k_c, v_c, o, lse = ctx.saved_tensors
    dq, dk, dv, d_lw, dw = _cuda.backward(grad_out, q_c, k_c, v_c, o, lse, ctx.prep, ctx.tau_win,
                                          ctx.win_edge, ctx.impl, want_dw=True)
    od = ctx.out_dtype
    # d_lw, dw: fp32 holding the values of the reference's .to(out_dtype) casts
    # (:750-757), so autograd hands them to the fp32 parameters without a cast
    return dq.to(od), dk.to(od), dv.to(od), d_lw, dw


class DSALTTrainFunction(torch.autograd.Function):
    """Autograd Function with the reference signature (dsalt_triton_train.py:585-760)."""

    @staticmethod
    def forward(ctx, q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens,
                tau_win, win_edge, n_max, cu_list=None):
        # fp32 view of the input-dtype output, written by the kernel itself
        # (the reference returns out.float(), :663)
        return _train_forward(ctx, q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge, cu_list,
                              f32_out=True)

    @staticmethod
    def backward(ctx, grad_out):
        dq, dk, dv, d_lw, dw = _train_backward(ctx, grad_out)
        return (dq, dk, dv,
                None,                 # lmk_pos
                d_lw,                 # -> alpha through log σ(s/τ)
                dw,                   # -> win_gate through w̃
                None, None, None,     # cu_seqlens, tau_win, win_edge
                None,                 # n_max
                None)                 # cu_list


class _DSALTTrainFunctionInputDtype(torch.autograd.Function):
    """The same op returning O in the (16-bit) input dtype: the values of the
    reference's fp32 output exactly (it holds input-dtype-rounded values), for
    callers that would cast it back at once (DSALTAttention under autocast)."""

    @staticmethod
    def forward(ctx, q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge, n_max, cu_list=None):
        return _train_forward(ctx, q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens, tau_win, win_edge, cu_list,
                              f32_out=False)

    @staticmethod
    def backward(ctx, grad_out):
        dq, dk, dv, d_lw, dw = _train_backward(ctx, grad_out)
        return dq, dk, dv, None, d_lw, dw, None, None, None, None, None


def _dynamo_opaque(fn):
    disable = getattr(getattr(torch, "_dynamo", None), "disable", None)
    return disable(fn) if disable is not None else fn


@_dynamo_opaque
def dsalt_triton_train_attention(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens,
                                 tau_win=1.0, win_edge=4.0, n_max=256, cu_list=None, out_dtype=None):
    """Differentiable sparse DSALT attention for training (reference :770-782).

    ``q, k, v`` ``[T, H, D]``; ``lmk_pos`` ``[H, S, k]`` positions inside each
    sequence (-1 = empty); ``lmk_logw`` ``[H, S, k]``; ``w_cont`` ``[T]``;
    ``cu_seqlens`` ``[S+1]``.  Returns ``O`` ``[T, H, D]`` float32 (the reference's
    output), or in q's 16-bit dtype when ``out_dtype`` is that dtype (the same
    values, without the fp32 copy; an extension, not in the reference).
    """
    if out_dtype is not None and out_dtype == q.dtype and q.dtype != torch.float32:
        return _DSALTTrainFunctionInputDtype.apply(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens,
                                                   tau_win, win_edge, n_max, cu_list)
    return DSALTTrainFunction.apply(q, k, v, lmk_pos, lmk_logw, w_cont, cu_seqlens,
                                    tau_win, win_edge, n_max, cu_list)
