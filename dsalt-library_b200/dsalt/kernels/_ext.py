"""ctypes binding of ``libdsalt_b200.so`` (the C ABI in ``include/dsalt_b200.h``).

The library is built in-tree by ``dsalt-library_b200/build.py`` into
``dsalt/_lib/libdsalt_b200.so``.  There is no fallback: if the library is
missing or no CUDA device is present, every op raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parents[1] / "_lib" / "libdsalt_b200.so"

# status / enum values of include/dsalt_b200.h
OK = 0
F16, BF16, F32 = 0, 1, 2
TRAIN, INFER = 0, 1
IMPL_AUTO, IMPL_SIMT, IMPL_TCGEN05 = 0, 1, 2
DEV_WAIT_TIMEOUT, DEV_BAD_INDEX = 1, 2
ABI_VERSION = 8
QREC_FLOATS = 16  # DSALT_QREC_FLOATS
LMK_SPLIT = 4  # DSALT_LMK_SPLIT
DS_TILE_BYTES = 16384  # DSALT_DS_TILE_BYTES


def ds_tiles(H: int, max_blocks: int, S: int, kp: int, band_tiles: int, lmk_tiles: int) -> int:
    """DSALT_DS_TILES: dSᵀ tiles of the tensor-core backward's scratch."""
    return H * max_blocks * band_tiles + H * S * ((kp + 127) // 128) * lmk_tiles + 1

_c_void_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class ScheduleParams(ctypes.Structure):
    _fields_ = [("cu_seqlens", _c_void_p), ("w", _c_void_p), ("block_map", _c_void_p),
                ("num_blocks", _c_void_p), ("seq_wmax", _c_void_p), ("seq_id", _c_void_p),
                ("T", _i64), ("S", _i32), ("block", _i32), ("max_blocks", _i32),
                ("semantics", _i32), ("seq_wmax_batch", _c_void_p)]


class GatherParams(ctypes.Structure):
    _fields_ = [("k", _c_void_p), ("v", _c_void_p), ("lmk_pos", _c_void_p), ("lmk_w", _c_void_p),
                ("cu_seqlens", _c_void_p), ("lmk_k", _c_void_p), ("lmk_v", _c_void_p),
                ("pos_sorted", _c_void_p), ("w_sorted", _c_void_p), ("perm", _c_void_p),
                ("lmk_slot", _c_void_p), ("status", _c_void_p),
                ("T", _i64), ("H", _i32), ("D", _i32), ("S", _i32), ("k_lmk", _i32), ("kp", _i32),
                ("dtype", _i32), ("H_kv", _i32)]


class AttnParams(ctypes.Structure):
    _fields_ = [("q", _c_void_p), ("k", _c_void_p), ("v", _c_void_p), ("w", _c_void_p),
                ("cu_seqlens", _c_void_p), ("block_map", _c_void_p), ("num_blocks", _c_void_p),
                ("seq_wmax", _c_void_p), ("lmk_k", _c_void_p), ("lmk_v", _c_void_p),
                ("pos_sorted", _c_void_p), ("w_sorted", _c_void_p), ("perm", _c_void_p),
                ("lmk_slot", _c_void_p),
                ("o", _c_void_p), ("o_f32", _c_void_p), ("lse", _c_void_p),
                ("dout", _c_void_p), ("dout_f32", _c_void_p), ("delta", _c_void_p), ("dq", _c_void_p), ("dk", _c_void_p),
                ("dv", _c_void_p), ("dw_head", _c_void_p), ("dw", _c_void_p), ("d_lw", _c_void_p),
                ("lmk_grad", _c_void_p), ("qrec", _c_void_p), ("ds_tiles", _c_void_p), ("status", _c_void_p),
                ("T", _i64), ("H", _i32), ("D", _i32), ("S", _i32), ("k_lmk", _i32), ("kp", _i32),
                ("max_blocks", _i32), ("ds_band_tiles", _i32), ("ds_lmk_tiles", _i32),
                ("scale", _f32), ("tau_win", _f32), ("win_edge", _f32),
                ("semantics", _i32), ("dtype", _i32), ("impl", _i32), ("H_kv", _i32),
                ("grad_round", _i32)]


class ScoreParams(ctypes.Structure):
    _fields_ = [("x", _c_void_p), ("xwv", _c_void_p), ("alpha", _c_void_p), ("scores", _c_void_p),
                ("z_x", _c_void_p), ("z_v", _c_void_p), ("stats", _c_void_p), ("norms", _c_void_p),
                ("T", _i64), ("d_model", _i32), ("H", _i32), ("n_kv", _i32), ("dh", _i32),
                ("dtype", _i32)]


class TopkParams(ctypes.Structure):
    _fields_ = [("scores", _c_void_p), ("w_sizes", _c_void_p), ("cu_seqlens", _c_void_p),
                ("idx", _c_void_p), ("T", _i64), ("H", _i32), ("S", _i32), ("k", _i32),
                ("max_len", _i32)]


class WinGateParams(ctypes.Structure):
    _fields_ = [("x", _c_void_p), ("weight", _c_void_p), ("bias", _c_void_p), ("w_cont", _c_void_p),
                ("w_f32", _c_void_p), ("w_disc", _c_void_p), ("logits", _c_void_p),
                ("T", _i64), ("d_model", _i32), ("n_min", _f32), ("n_max", _f32), ("dtype", _i32)]


class RopeParams(ctypes.Structure):
    _fields_ = [("q", _c_void_p), ("k", _c_void_p), ("v", _c_void_p), ("cos", _c_void_p), ("sin", _c_void_p),
                ("q_out", _c_void_p), ("k_out", _c_void_p), ("v_out", _c_void_p),
                ("dq_out", _c_void_p), ("dk_out", _c_void_p), ("dv_out", _c_void_p),
                ("dq", _c_void_p), ("dk", _c_void_p), ("dv", _c_void_p),
                ("T", _i64), ("ld", _i64), ("H", _i32), ("Hkv", _i32), ("D", _i32), ("dtype", _i32),
                ("kv_out_heads", _i32)]


class RmsNormParams(ctypes.Structure):
    _fields_ = [("x", _c_void_p), ("res", _c_void_p), ("x_sum", _c_void_p), ("w", _c_void_p), ("y", _c_void_p),
                ("rstd", _c_void_p), ("dy", _c_void_p), ("dres", _c_void_p), ("dx", _c_void_p),
                ("dw_part", _c_void_p), ("dw", _c_void_p), ("T", _i64), ("d", _i32), ("eps", _f32), ("dtype", _i32)]


class ScaleRowsParams(ctypes.Structure):
    _fields_ = [("x", _c_void_p), ("coef", _c_void_p), ("out", _c_void_p), ("T", _i64), ("groups", _i32),
                ("width", _i32), ("dtype", _i32)]


class XentParams(ctypes.Structure):
    _fields_ = [("logits", _c_void_p), ("labels", _c_void_p), ("row_loss", _c_void_p), ("scale", _c_void_p),
                ("rows", _i64), ("vocab", _i32), ("ignore_index", _i32), ("dtype", _i32)]


class SwigluParams(ctypes.Structure):
    _fields_ = [("g", _c_void_p), ("u", _c_void_p), ("h", _c_void_p), ("dh", _c_void_p), ("dg", _c_void_p),
                ("du", _c_void_p), ("T", _i64), ("F", _i64), ("ld_in", _i64), ("ld_out", _i64), ("dtype", _i32)]


class ScoreBwdParams(ctypes.Structure):
    _fields_ = [("g_s", _c_void_p), ("alpha", _c_void_p), ("z_x", _c_void_p), ("z_v", _c_void_p),
                ("norms", _c_void_p), ("stats", _c_void_p), ("sums", _c_void_p), ("partials", _c_void_p),
                ("d_alpha", _c_void_p), ("coef_x", _c_void_p), ("coef_v", _c_void_p), ("T", _i64), ("H", _i32),
                ("n_kv", _i32)]


class WinGateBwdParams(ctypes.Structure):
    _fields_ = [("x", _c_void_p), ("weight", _c_void_p), ("dl", _c_void_p), ("dx", _c_void_p),
                ("dw_part", _c_void_p), ("T", _i64), ("d_model", _i32), ("dtype", _i32)]


RMSNORM_ROWS_PER_PART = 64  # DSALT_RMSNORM_ROWS_PER_PART
WIN_GATE_ROWS_PER_PART = 32  # DSALT_WIN_GATE_ROWS_PER_PART
SCORE_BWD_TOKENS = 128  # DSALT_SCORE_BWD_TOKENS

class GqaReduceParams(ctypes.Structure):
    _fields_ = [("x", _c_void_p), ("y", _c_void_p), ("T", _i64), ("H", _i32), ("H_kv", _i32), ("D", _i32),
                ("dtype", _i32)]


_STRUCTS = [ScheduleParams, GatherParams, AttnParams, ScoreParams, TopkParams, WinGateParams, RopeParams,
            RmsNormParams, ScaleRowsParams, XentParams, SwigluParams, WinGateBwdParams, ScoreBwdParams,
            GqaReduceParams]
_ENTRY = {
    "dsalt_build_schedule": ScheduleParams,
    "dsalt_gather_landmarks": GatherParams,
    "dsalt_attn_fwd": AttnParams,
    "dsalt_attn_bwd_preprocess": AttnParams,
    "dsalt_attn_bwd_dkdv": AttnParams,
    "dsalt_attn_bwd_dq": AttnParams,
    "dsalt_hybrid_scores": ScoreParams,
    "dsalt_hybrid_scores_noalloc": ScoreParams,
    "dsalt_select_topk": TopkParams,
    "dsalt_win_gate": WinGateParams,
    "dsalt_rope_gqa_fwd": RopeParams,
    "dsalt_rope_gqa_bwd": RopeParams,
    "dsalt_rmsnorm_fwd": RmsNormParams,
    "dsalt_rmsnorm_bwd": RmsNormParams,
    "dsalt_scale_rows": ScaleRowsParams,
    "dsalt_xent_fwd_grad": XentParams,
    "dsalt_win_gate_bwd": WinGateBwdParams,
    "dsalt_hybrid_scores_bwd": ScoreBwdParams,
    "dsalt_swiglu_fwd": SwigluParams,
    "dsalt_swiglu_bwd": SwigluParams,
    "dsalt_gqa_reduce": GqaReduceParams,
}

_lib = None


def lib_path() -> Path:
    return Path(os.environ.get("DSALT_B200_LIB", str(_LIB_PATH)))


def load() -> ctypes.CDLL:
    """Load (once) and check the shared library; raise if it is missing or stale."""
    global _lib
    if _lib is not None:
        return _lib
    path = lib_path()
    if not path.exists():
        raise RuntimeError(
            f"DSALT CUDA library not found at {path}; build it with "
            "`python dsalt-library_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    lib.dsalt_b200_abi_version.restype = ctypes.c_int
    lib.dsalt_b200_status_string.restype = ctypes.c_char_p
    lib.dsalt_b200_status_string.argtypes = [ctypes.c_int]
    lib.dsalt_b200_params_sizeof.restype = ctypes.c_int
    lib.dsalt_b200_params_sizeof.argtypes = [ctypes.c_int]
    if lib.dsalt_b200_abi_version() != ABI_VERSION:
        raise RuntimeError("libdsalt_b200.so ABI version mismatch; rebuild the library")
    for i, st in enumerate(_STRUCTS):
        n = lib.dsalt_b200_params_sizeof(i)
        if n != ctypes.sizeof(st):
            raise RuntimeError(f"{st.__name__}: ctypes size {ctypes.sizeof(st)} != C size {n}")
    for name, st in _ENTRY.items():
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.POINTER(st), ctypes.c_void_p]
    _lib = lib
    return lib


def status_string(code: int) -> str:
    return load().dsalt_b200_status_string(int(code)).decode()


# Optional launch recorder: when a list, every call appends (name, start, end)
# CUDA events recorded on the launching stream (used by the benchmark to time
# individual kernels live).
RECORD: list | None = None


def current_stream_handle() -> int:
    """Raw handle of the current CUDA stream of the current device (no Stream object)."""
    return torch._C._cuda_getCurrentRawStream(torch._C._cuda_getDevice())


def call(name: str, params) -> None:
    """Launch ``name`` on the current CUDA stream; raise RuntimeError on a bad status."""
    lib = _lib if _lib is not None else load()
    rec = RECORD
    if rec is not None:
        cs = torch.cuda.current_stream()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(cs)
    rc = getattr(lib, name)(ctypes.byref(params), current_stream_handle())
    if rc != OK:
        raise RuntimeError(f"{name} failed: {status_string(rc)} (status {rc})")
    if rec is not None:
        e1.record(cs)
        rec.append((name, e0, e1))


def ptr(t) -> int:
    """Device address of a tensor (0 for None)."""
    return 0 if t is None else int(t.data_ptr())


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float16:
        return F16
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {dt}")


def require_cuda(t: torch.Tensor, what: str = "input") -> None:
    if not t.is_cuda:
        raise RuntimeError(
            f"dsalt (B200 build) runs on CUDA devices only; {what} is on {t.device} "
            "(there is no CPU fallback)")


def half_compute_dtype(x: torch.Tensor, *weights: torch.Tensor):
    """The 16-bit dtype a CUDA layer computes in: autocast's when it is on and
    16-bit, else x's when x and every weight share one 16-bit dtype; None when the
    layer computes in fp32 (the callers then keep the reference's torch ops)."""
    if not x.is_cuda:
        return None
    half = (torch.float16, torch.bfloat16)
    if torch.is_autocast_enabled("cuda"):
        dt = torch.get_autocast_dtype("cuda")
        return dt if dt in half else None
    return x.dtype if x.dtype in half and all(w.dtype == x.dtype for w in weights) else None


def default_impl() -> int:
    """Kernel family: DSALT_IMPL env var ('auto' | 'simt' | 'tcgen05')."""
    v = os.environ.get("DSALT_IMPL", "auto").lower()
    return {"auto": IMPL_AUTO, "simt": IMPL_SIMT, "tcgen05": IMPL_TCGEN05}.get(v, IMPL_AUTO)
