"""Backward of the DSALT inference op on B200 (module name kept from the reference).

Reference: ``dsalt/kernels/dsalt_triton_bwd.py:219-324``.  Same signature and
return value ``(dq, dk, dv, d_bias)`` as float32 tensors.  The reference
accumulates dK/dV with ``atomic_add`` (:206-207); here dK/dV are key-parallel
and atomic-free, so the result is deterministic.  The block-size arguments are
accepted for compatibility and ignored (tiles are fixed for B200), and the
landmark keys/values are re-gathered from ``k``/``v`` at ``lmk_pos``.
"""

from __future__ import annotations

import torch

from . import _ext
from . import dsalt_cuda as _cuda


def dsalt_triton_backward(grad_out, q, k, v, out, lse, lmk_K, lmk_V, lmk_pos, lmk_bias,
                          w_sizes, cu_seqlens, scale, seq_block_map=None, total_blk=None,
                          BLOCK_M=None, BLOCK_N=None, HEAD_DIM_C=None,
                          num_warps=None, num_stages=None):
    _cuda.check_inputs(q, k, v, cu_seqlens)
    dt = _cuda.compute_dtype(q)
    q_c = q.contiguous().to(dt)
    k_c = k.contiguous().to(dt)
    v_c = v.contiguous().to(dt)
    o_c = out.contiguous().to(dt)
    lse_c = lse.contiguous().to(torch.float32)
    prep = _cuda.prepare(k_c, v_c, lmk_pos, lmk_bias, w_sizes, cu_seqlens, _ext.INFER)
    dq, dk, dv, d_bias, _ = _cuda.backward(grad_out, q_c, k_c, v_c, o_c, lse_c, prep, 1.0, 0.0,
                                           _ext.default_impl(), want_dw=False)
    return dq.float(), dk.float(), dv.float(), d_bias
