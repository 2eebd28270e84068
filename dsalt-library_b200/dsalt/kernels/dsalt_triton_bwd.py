"""Backward of the DSALT inference op on B200 (module name kept from the reference).

Reference: ``dsalt/kernels/dsalt_triton_bwd.py:219-324``.  Same signature and
return value ``(dq, dk, dv, d_bias)`` as float32 tensors.  The reference
accumulates dK/dV with ``atomic_add`` (:206-207); here dK/dV are key-parallel
and atomic-free, so the result is deterministic.

* ``scale`` multiplies q·kᵀ in the recomputed logits, as in the reference kernel;
  ``lse`` is the natural-log LSE of those scaled logits (the reference forward's
  ``m + log l``, dsalt_triton_attn.py:164, which is also what this build's forward
  writes).
* ``lmk_K`` / ``lmk_V`` are ``k`` / ``v`` gathered at ``lmk_pos`` (the reference's
  only caller builds them that way, ``_build_landmark_kv``); this build gathers
  them itself from ``k`` / ``v`` in position order and checks only their shape.
* The block-size and launch arguments select Triton tiles in the reference and
  have no meaning for the fixed B200 kernels; they are accepted and ignored.
"""

from __future__ import annotations

import math

import torch

from . import _ext
from . import dsalt_cuda as _cuda


def dsalt_triton_backward(grad_out, q, k, v, out, lse, lmk_K, lmk_V, lmk_pos, lmk_bias,
                          w_sizes, cu_seqlens, scale, seq_block_map=None, total_blk=None,
                          BLOCK_M=None, BLOCK_N=None, HEAD_DIM_C=None,
                          num_warps=None, num_stages=None):
    _cuda.check_inputs(q, k, v, cu_seqlens)
    H, S, k_lmk = lmk_pos.shape
    for name, t in (("lmk_K", lmk_K), ("lmk_V", lmk_V)):
        if t is not None and (t.dim() != 4 or tuple(t.shape[:3]) != (H, S, k_lmk) or t.shape[3] != q.shape[2]):
            raise ValueError(f"{name} must be [H, S, k_lmk, D] = {(H, S, k_lmk, q.shape[2])}, "
                             f"got {tuple(t.shape)}")
    if not (isinstance(scale, (int, float)) and math.isfinite(scale)):
        raise ValueError(f"scale must be a finite number, got {scale!r}")
    dt = _cuda.compute_dtype(q)
    q_c = q.contiguous().to(dt)
    k_c = k.contiguous().to(dt)
    v_c = v.contiguous().to(dt)
    o_c = out.contiguous().to(dt)
    lse_c = lse.contiguous().to(torch.float32)
    prep = _cuda.prepare(k_c, v_c, lmk_pos, lmk_bias, w_sizes, cu_seqlens, _ext.INFER, for_backward=True)
    dq, dk, dv, d_bias, _ = _cuda.backward(grad_out, q_c, k_c, v_c, o_c, lse_c, prep, 1.0, 0.0,
                                           _ext.default_impl(), want_dw=False, scale=float(scale),
                                           grad_round=False)
    return dq.float(), dk.float(), dv.float(), d_bias
