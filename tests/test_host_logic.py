"""CPU checks of host-side logic of the model path: the compute-dtype choice that
routes layers to the CUDA kernels, the cached host copy of ``cu_seqlens`` and the
argument checks of the model-step entry points (no kernel is launched)."""

from __future__ import annotations

import ctypes

import pytest
import torch


def test_half_compute_dtype_rules():
    from dsalt.kernels import _ext
    x32, w32 = torch.zeros(4, 8), torch.zeros(16, 8)
    assert _ext.half_compute_dtype(x32, w32) is None  # CPU tensors never take the CUDA path
    assert _ext.half_compute_dtype(x32.bfloat16(), w32.bfloat16()) is None


def test_host_cu_copy_is_reused_until_the_tensor_changes():
    from dsalt.model.dsalt_lm import DSALTLMHeadModel
    m = DSALTLMHeadModel(vocab_size=64, d_model=256, n_layers=1, n_heads=4, n_min=8, n_max=32, k_lmk=4,
                         max_seq_len=256)
    cu = torch.tensor([0, 100, 256], dtype=torch.int32)
    first = m._host_cu(cu)
    assert first == [0, 100, 256]
    assert m._host_cu(cu) is first                      # same tensor, unmodified: no new copy
    cu[1] = 120                                         # in-place write bumps the version counter
    assert m._host_cu(cu) == [0, 120, 256]
    other = torch.tensor([0, 120, 256], dtype=torch.int32)
    assert m._host_cu(other) == [0, 120, 256]            # another tensor object: copied again
    assert m._cu_host[0] is other


def test_fused_ce_falls_back_on_cpu():
    from dsalt.model.dsalt_lm import _fused_ce_dtype
    assert _fused_ce_dtype(torch.zeros(2, 8), torch.zeros(10, 8)) is None


def _rc(name, p):
    from dsalt.kernels import _ext
    lib = _ext.load()
    return getattr(lib, name)(ctypes.byref(p), ctypes.c_void_p(0))


def test_model_step_entry_points_reject_bad_arguments():
    """Argument checks run before any launch: bad sizes, strides and dtypes come back
    as status codes (null device pointers are never dereferenced)."""
    from dsalt.kernels import _ext
    ARG, DT, HD = 1, 2, 3  # DSALT_ERR_ARG, DSALT_ERR_DTYPE, DSALT_ERR_HEAD_DIM of include/dsalt_b200.h
    # SwiGLU: F must split into 16-byte pieces, the row strides must cover F
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=4, F=12, ld_in=24, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=4, F=16, ld_in=8, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_swiglu_bwd", _ext.SwigluParams(T=4, F=16, ld_in=32, ld_out=8, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=4, F=16, ld_in=32, dtype=_ext.F32)) == DT
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=0, F=16, ld_in=32, dtype=_ext.BF16)) == _ext.OK
    # RMSNorm: supported widths only
    assert _rc("dsalt_rmsnorm_fwd", _ext.RmsNormParams(T=4, d=300, eps=1e-6, dtype=_ext.BF16)) == HD
    # window-gate backward: d_model a multiple of 8, 16-bit only
    assert _rc("dsalt_win_gate_bwd", _ext.WinGateBwdParams(T=4, d_model=12, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_win_gate_bwd", _ext.WinGateBwdParams(T=4, d_model=16, dtype=_ext.F32)) == DT
    # the prologue's row stride: a multiple of 8 elements and at least H·D
    assert _rc("dsalt_rope_gqa_fwd", _ext.RopeParams(T=4, ld=100, H=2, Hkv=2, D=64, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_rope_gqa_fwd", _ext.RopeParams(T=4, ld=130, H=2, Hkv=2, D=64, dtype=_ext.BF16)) == ARG
    # cross-entropy: 16-bit logits only
    assert _rc("dsalt_xent_fwd_grad", _ext.XentParams(rows=4, vocab=10, dtype=_ext.F32)) == DT
