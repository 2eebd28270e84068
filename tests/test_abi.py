"""CPU-side checks of the C-ABI library: it loads, exports every declared symbol,
and the ctypes mirrors of the parameter structs match the C layout."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "dsalt_b200.h"


def _declared():
    txt = HEADER.read_text()
    return sorted(set(re.findall(r"DSALT_API\s+(?:const\s+char\s*\*|int)\s+(dsalt_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    names = _declared()
    for must in ("dsalt_attn_fwd", "dsalt_attn_bwd_dkdv", "dsalt_attn_bwd_dq", "dsalt_attn_bwd_preprocess",
                 "dsalt_build_schedule", "dsalt_gather_landmarks", "dsalt_select_topk",
                 "dsalt_hybrid_scores", "dsalt_win_gate"):
        assert must in names


def test_library_loads_and_exports_all_symbols():
    from dsalt.kernels import _ext
    lib = _ext.load()
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_ext.lib_path())], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r" T (dsalt_\w+)", out))
    assert set(_declared()) <= exported


def test_struct_layouts_match():
    from dsalt.kernels import _ext
    import ctypes
    lib = _ext.load()
    for i, st in enumerate(_ext._STRUCTS):
        assert lib.dsalt_b200_params_sizeof(i) == ctypes.sizeof(st), st.__name__


def test_header_constants_match_mirror():
    """ABI version and the landmark-split constant that sizes the dK/dV scratch."""
    from dsalt.kernels import _ext
    txt = HEADER.read_text()
    assert int(re.search(r"#define DSALT_B200_ABI_VERSION (\d+)", txt).group(1)) == _ext.ABI_VERSION
    assert int(re.search(r"#define DSALT_LMK_SPLIT (\d+)", txt).group(1)) == _ext.LMK_SPLIT
    assert int(re.search(r"#define DSALT_QREC_FLOATS (\d+)", txt).group(1)) == _ext.QREC_FLOATS
    assert _ext.load().dsalt_b200_abi_version() == _ext.ABI_VERSION


def test_status_strings():
    from dsalt.kernels import _ext
    assert _ext.status_string(0) == "ok"
    assert "argument" in _ext.status_string(1)


def test_argument_errors_without_launch():
    """Invalid arguments are rejected on the host before any launch (no GPU needed)."""
    from dsalt.kernels import _ext
    import ctypes
    lib = _ext.load()
    p = _ext.AttnParams(T=16, H=1, D=12, S=1, k_lmk=0, kp=0, tau_win=1.0, dtype=_ext.BF16)
    assert lib.dsalt_attn_fwd(ctypes.byref(p), None) == 3  # head_dim
    p.D = 64
    p.dtype = 7
    assert lib.dsalt_attn_fwd(ctypes.byref(p), None) == 2  # dtype
    p.dtype = _ext.BF16
    assert lib.dsalt_attn_fwd(ctypes.byref(p), None) == 1  # null pointers
    tp = _ext.TopkParams(T=10, H=1, S=1, k=2000, max_len=10)
    assert lib.dsalt_select_topk(ctypes.byref(tp), None) == 7  # too large


def test_no_cpu_fallback():
    """The ops refuse CPU tensors instead of silently computing elsewhere."""
    import torch
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    q = torch.randn(8, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        dsalt_triton_train_attention(q, q, q, torch.zeros(1, 1, 1, dtype=torch.long), torch.zeros(1, 1, 1),
                                     torch.ones(8), torch.tensor([0, 8], dtype=torch.int32))
