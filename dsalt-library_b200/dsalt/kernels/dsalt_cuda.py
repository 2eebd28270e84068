"""Host side of the DSALT attention op on B200: buffer allocation and launches.

Every launch goes through the C ABI of ``libdsalt_b200.so`` (``_ext``).  This
module owns the order of the stages and the scratch buffers; the autograd
Functions with the reference's signatures live in ``dsalt_triton_train`` and
``dsalt_triton_attn`` (module names kept so the package drops in for the
reference's Triton path).

Stages (reference counterparts in dsalt/kernels/dsalt_triton_train.py):
  schedule  (seq, block) table + per-sequence max window   (_build_seq_block_map, :618)
  gather    landmarks sorted by position, K/V rows gathered (_build_landmark_kv, :617)
  fwd       O (input dtype), O as fp32, LSE                 (_train_fwd_kernel, :629-645)
  bwd       Delta, key-parallel dK/dV/d_logw, query-parallel dQ/d_w̃
                                                            (:693-745)
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _ext

BLOCK_M = 128  # query rows per tensor-core tile (tcgen05 M=128)

_STATUS: dict = {}


def device_status(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word the kernels OR their fault bits into."""
    key = (device.type, device.index if device.index is not None else torch.cuda.current_device())
    st = _STATUS.get(key)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS[key] = st
    return st


def check_device_status(device: torch.device, reset: bool = True) -> int:
    """Read (and optionally clear) the device status word; raise on a fault bit."""
    st = device_status(device)
    v = int(st.item())
    if reset:
        st.zero_()
    if v & _ext.DEV_WAIT_TIMEOUT:
        raise RuntimeError("dsalt kernel: an mbarrier wait timed out (device status %d)" % v)
    if v & _ext.DEV_BAD_INDEX:
        raise RuntimeError("dsalt kernel: an index was out of range (device status %d)" % v)
    return v


def padded_landmarks(k_lmk: int) -> int:
    """Landmark slots after padding: a multiple of 16, at least 16 (0 stays 0)."""
    return 0 if k_lmk <= 0 else max(16, (k_lmk + 15) // 16 * 16)


@dataclass
class Prepared:
    """Per-call metadata shared by the forward and the backward."""
    T: int
    H: int
    D: int
    S: int
    k_lmk: int
    kp: int
    semantics: int
    cu: torch.Tensor
    w: torch.Tensor
    block_map: torch.Tensor
    num_blocks: torch.Tensor
    seq_wmax: torch.Tensor
    lmk_k: torch.Tensor
    lmk_v: torch.Tensor
    pos_sorted: torch.Tensor
    w_sorted: torch.Tensor
    perm: torch.Tensor
    lmk_slot: torch.Tensor
    max_blocks: int
    lmax: int = 0                # longest sequence (host)
    H_kv: int = 0                # kv heads of k, v (grouped kv heads when < H)
    wmax_slot: int = -1          # slot of the widest band in the pinned ring (-1: none)
    wmax_gen: int = 0
    seq_wmax_batch: torch.Tensor | None = None   # [1] int32: max over s of seq_wmax


# The widest band of a batch (max over the sequences of seq_wmax) sizes the dSᵀ tile
# scratch of the backward.  The forward copies it into a small ring of pinned host
# slots right after the schedule kernel and records an event.  The backward uses it
# when that event has completed; otherwise (the host runs ahead of the device) it
# sizes the scratch for bands as long as the sequences, which needs no device
# value, and waits for the event only when that bound would exceed
# SCRATCH_BUDGET_BYTES.
_WMAX_RING = 64
_WMAX: dict = {}


def _wmax_ring(dev: torch.device):
    key = dev.index if dev.index is not None else torch.cuda.current_device()
    r = _WMAX.get(key)
    if r is None:
        r = {"host": torch.zeros(_WMAX_RING, dtype=torch.int32).pin_memory(),
             "events": [torch.cuda.Event() for _ in range(_WMAX_RING)], "gen": [0] * _WMAX_RING, "next": 0}
        _WMAX[key] = r
    return r


def _record_wmax(prep: "Prepared", dev: torch.device) -> None:
    if torch.cuda.is_current_stream_capturing():
        return  # a captured graph replays without the host: the backward uses the length bound
    r = _wmax_ring(dev)
    slot = r["next"]
    r["next"] = (slot + 1) % _WMAX_RING
    r["gen"][slot] += 1
    r["host"][slot:slot + 1].copy_(prep.seq_wmax_batch, non_blocking=True)
    r["events"][slot].record()
    prep.wmax_slot, prep.wmax_gen = slot, r["gen"][slot]


SCRATCH_BUDGET_BYTES = 8 << 30


def widest_band(prep: "Prepared", dev: torch.device, bytes_per_band_tile: int) -> int:
    """Upper bound of max_s seq_wmax[s] for sizing the backward's tile scratch
    (``bytes_per_band_tile``: scratch bytes per unit of band_tiles)."""
    r = _WMAX.get(dev.index if dev.index is not None else torch.cuda.current_device())
    recorded = prep.wmax_slot >= 0 and r is not None and r["gen"][prep.wmax_slot] == prep.wmax_gen
    length_bound = max(prep.lmax - 1, 0)   # a band never reaches past its sequence start
    if recorded:
        ev = r["events"][prep.wmax_slot]
        fits = (BLOCK_M + length_bound + 63) // 64 * bytes_per_band_tile <= SCRATCH_BUDGET_BYTES
        if ev.query() or (not fits and not torch.cuda.is_current_stream_capturing()):
            ev.synchronize()
            return max(int(r["host"][prep.wmax_slot]), 0)
    return length_bound


def prepare(k_c: torch.Tensor, v_c: torch.Tensor, lmk_pos: torch.Tensor, lmk_w: torch.Tensor,
            w: torch.Tensor, cu_seqlens: torch.Tensor, semantics: int, cu_host=None,
            for_backward: bool = False) -> Prepared:
    """Build the schedule and the sorted landmark buffers on the device.

    ``cu_host``: the host copy of ``cu_seqlens`` when the caller has one;
    ``for_backward``: record the widest band for the backward's scratch.
    ``k_c``, ``v_c`` are ``[T, H_kv, D]``; the query heads ``H`` are those of
    ``lmk_pos`` (``[H, S, k]``, a multiple of ``H_kv``)."""
    T, H_kv, D = k_c.shape
    dev = k_c.device
    cu = cu_seqlens.to(device=dev, dtype=torch.int32).contiguous()
    S = cu.shape[0] - 1
    H = int(lmk_pos.shape[0]) if lmk_pos.dim() == 3 else H_kv
    if lmk_pos.dim() != 3 or lmk_pos.shape[1] != S or H % H_kv != 0:
        raise ValueError(f"lmk_pos must be [H, S={S}, k] with H a multiple of H_kv={H_kv}, "
                         f"got {tuple(lmk_pos.shape)}")
    k_lmk = int(lmk_pos.shape[2])
    kp = padded_landmarks(k_lmk)
    w32 = w.detach().to(device=dev, dtype=torch.float32).contiguous()
    if w32.shape != (T,):
        raise ValueError(f"window must be [T={T}], got {tuple(w32.shape)}")
    max_blocks = (T + BLOCK_M - 1) // BLOCK_M + S
    block_map = torch.empty(max(max_blocks, 1), 2, dtype=torch.int32, device=dev)
    num_blocks = torch.empty(1, dtype=torch.int32, device=dev)
    # per-sequence band maxima, then the batch maximum (written by the schedule kernels)
    wmax_buf = torch.empty(max(S, 1) + 1, dtype=torch.int32, device=dev)
    seq_wmax, seq_wmax_batch = wmax_buf[:max(S, 1)], wmax_buf[max(S, 1):]
    sp = _ext.ScheduleParams(
        cu_seqlens=_ext.ptr(cu), w=_ext.ptr(w32), block_map=_ext.ptr(block_map),
        num_blocks=_ext.ptr(num_blocks), seq_wmax=_ext.ptr(seq_wmax), seq_id=0,
        T=T, S=S, block=BLOCK_M, max_blocks=max_blocks, semantics=semantics,
        seq_wmax_batch=_ext.ptr(seq_wmax_batch))
    _ext.call("dsalt_build_schedule", sp)

    dt = k_c.dtype
    lmk_k = torch.empty(H, S, kp, D, dtype=dt, device=dev)
    lmk_v = torch.empty(H, S, kp, D, dtype=dt, device=dev)
    pos_sorted = torch.empty(H, S, kp, dtype=torch.int32, device=dev)
    w_sorted = torch.empty(H, S, kp, dtype=torch.float32, device=dev)
    perm = torch.empty(H, S, kp, dtype=torch.int32, device=dev)
    lmk_slot = torch.empty(T, H, dtype=torch.int32, device=dev)
    if kp > 0 and S > 0:
        lp = lmk_pos.detach().to(device=dev, dtype=torch.int64).contiguous()
        lw = lmk_w.detach().to(device=dev, dtype=torch.float32).contiguous()
        gp = _ext.GatherParams(
            k=_ext.ptr(k_c), v=_ext.ptr(v_c), lmk_pos=_ext.ptr(lp), lmk_w=_ext.ptr(lw),
            cu_seqlens=_ext.ptr(cu), lmk_k=_ext.ptr(lmk_k), lmk_v=_ext.ptr(lmk_v),
            pos_sorted=_ext.ptr(pos_sorted), w_sorted=_ext.ptr(w_sorted), perm=_ext.ptr(perm),
            lmk_slot=_ext.ptr(lmk_slot), status=_ext.ptr(device_status(dev)),
            T=T, H=H, D=D, S=S, k_lmk=k_lmk, kp=kp, dtype=_ext.dtype_code(dt), H_kv=H_kv)
        _ext.call("dsalt_gather_landmarks", gp)
    else:
        lmk_slot.fill_(-1)
    if cu_host is None:
        cu_host = [int(c) for c in cu.to("cpu").tolist()]
    lmax = max((b - a for a, b in zip(cu_host[:-1], cu_host[1:])), default=0)
    prep = Prepared(T, H, D, S, k_lmk, kp, semantics, cu, w32, block_map, num_blocks, seq_wmax,
                    lmk_k, lmk_v, pos_sorted, w_sorted, perm, lmk_slot, max_blocks, lmax, H_kv,
                    seq_wmax_batch=seq_wmax_batch)
    if for_backward and T > 0:
        _record_wmax(prep, dev)
    return prep


def _params(prep: Prepared, q_c, k_c, v_c, tau_win: float, win_edge: float, impl: int,
            scale: float | None = None, **bufs) -> _ext.AttnParams:
    p = _ext.AttnParams(
        q=_ext.ptr(q_c), k=_ext.ptr(k_c), v=_ext.ptr(v_c), w=_ext.ptr(prep.w),
        cu_seqlens=_ext.ptr(prep.cu), block_map=_ext.ptr(prep.block_map),
        num_blocks=_ext.ptr(prep.num_blocks), seq_wmax=_ext.ptr(prep.seq_wmax),
        lmk_k=_ext.ptr(prep.lmk_k), lmk_v=_ext.ptr(prep.lmk_v), pos_sorted=_ext.ptr(prep.pos_sorted),
        w_sorted=_ext.ptr(prep.w_sorted), perm=_ext.ptr(prep.perm), lmk_slot=_ext.ptr(prep.lmk_slot),
        status=_ext.ptr(device_status(q_c.device)),
        T=prep.T, H=prep.H, D=prep.D, S=prep.S, k_lmk=prep.k_lmk, kp=prep.kp,
        max_blocks=prep.max_blocks, scale=1.0 / math.sqrt(prep.D) if scale is None else float(scale),
        tau_win=float(tau_win),
        win_edge=float(win_edge) if prep.semantics == _ext.TRAIN else 0.0,
        semantics=prep.semantics, dtype=_ext.dtype_code(q_c.dtype), impl=impl, H_kv=prep.H_kv)
    for name, t in bufs.items():
        setattr(p, name, _ext.ptr(t))
    return p


def forward(q_c, k_c, v_c, prep: Prepared, tau_win: float, win_edge: float, impl: int, f32_out: bool = True):
    """Run the forward; returns ``(o, o_out, lse [T,H] fp32)``: the O the backward
    reads and the op's output.

    16-bit inputs with ``f32_out`` write only the fp32 O (the input-dtype-rounded
    values, the reference's ``out.float()``), which is both items; with
    ``f32_out=False`` only the input-dtype O.  fp32 inputs write their fp32 O.
    """
    lse = torch.empty(prep.T, prep.H, dtype=torch.float32, device=q_c.device)
    if q_c.dtype != torch.float32 and f32_out:
        o_f32 = torch.empty(q_c.shape, dtype=torch.float32, device=q_c.device)
        p = _params(prep, q_c, k_c, v_c, tau_win, win_edge, impl, o=None, o_f32=o_f32, lse=lse)
        _ext.call("dsalt_attn_fwd", p)
        return o_f32, o_f32, lse
    o = torch.empty_like(q_c)
    p = _params(prep, q_c, k_c, v_c, tau_win, win_edge, impl, o=o, o_f32=None, lse=lse)
    _ext.call("dsalt_attn_fwd", p)
    return o, o, lse


def backward(grad_out, q_c, k_c, v_c, o, lse, prep: Prepared, tau_win: float, win_edge: float,
             impl: int, want_dw: bool, scale: float | None = None, grad_round: bool = True):
    """Run the backward stages; returns ``(dq, dk, dv, d_lw [H,S,k] fp32, dw [T] fp32 or None)``.

    ``grad_round``: ``d_lw`` and ``dw`` hold their sums rounded to the input dtype,
    in fp32 (the values the reference's autograd functions return after their
    ``.to(out_dtype)``, which autograd widens back for the fp32 parameters).

    ``grad_out`` may be fp32 (the op's output dtype) or the input dtype; an fp32
    gradient is rounded to the input dtype by the preprocess kernel itself.
    ``scale`` multiplies q·kᵀ (default ``1/√D``, what every forward of the op uses);
    ``lse`` is the natural-log LSE of the scaled logits, as the forward writes it.
    """
    dev = q_c.device
    grad_out = grad_out.contiguous()
    if grad_out.dtype == torch.float32 and q_c.dtype != torch.float32:
        do_f32, do_c = grad_out, torch.empty_like(q_c)
    else:
        do_f32, do_c = None, grad_out.to(q_c.dtype)
    T, H = prep.T, prep.H
    delta = torch.empty(T, H, dtype=torch.float32, device=dev)
    dq = torch.empty_like(q_c)
    # grouped kv heads: the stages write dk, dv per query head (the gradients of
    # the expanded K/V), summed per group at the end
    grouped = prep.H_kv != H
    dk = torch.empty_like(q_c) if grouped else torch.empty_like(k_c)
    dv = torch.empty_like(q_c) if grouped else torch.empty_like(v_c)
    d_lw = torch.empty(H, prep.S, prep.k_lmk, dtype=torch.float32, device=dev)  # every slot written
    dw_head = torch.empty(T, H, dtype=torch.float32, device=dev) if want_dw else None
    dw = torch.empty(T, dtype=torch.float32, device=dev) if want_dw else None
    # partial landmark-slot dK, dV, d_lw of the tensor-core dK/dV stage
    lmk_grad = torch.empty(((2 * prep.D + 1) * _ext.LMK_SPLIT + 2 * prep.D) * H * prep.S * prep.kp,
                           dtype=torch.float32, device=dev) if prep.kp > 0 else None
    # per-query records (LSE, Delta, window, soft-edge factors) of the tensor-core stages
    qrec = torch.empty(H, T, _ext.QREC_FLOATS, dtype=torch.float32, device=dev)
    # O as the forward wrote it: the input dtype, or only the fp32 copy of 16-bit inputs
    o_in, o32 = (None, o) if (o.dtype == torch.float32 and q_c.dtype != torch.float32) else (o, None)
    p = _params(prep, q_c, k_c, v_c, tau_win, win_edge, impl, scale, o=o_in, o_f32=o32, lse=lse, dout=do_c,
                dout_f32=do_f32,
                delta=delta, dq=dq, dk=dk, dv=dv, dw_head=dw_head, dw=dw, d_lw=d_lw, lmk_grad=lmk_grad,
                qrec=qrec)
    p.grad_round = 1 if grad_round else 0
    # the dSᵀ tiles the dK/dV stage stores for the dQ stage (tensor-core family)
    band_tiles = (BLOCK_M + widest_band(prep, dev, H * prep.max_blocks * _ext.DS_TILE_BYTES) + 63) // 64
    lmk_tiles = (prep.lmax + 63) // 64 + 1
    n_tiles = _ext.ds_tiles(H, prep.max_blocks, prep.S, prep.kp, band_tiles, lmk_tiles)
    p.ds_tiles = _tile_scratch(dev, n_tiles * _ext.DS_TILE_BYTES)
    p.ds_band_tiles, p.ds_lmk_tiles = band_tiles, lmk_tiles
    _ext.call("dsalt_attn_bwd_preprocess", p)
    # dQ multiplies the dSᵀ tiles that dK/dV stores: one after the other
    _ext.call("dsalt_attn_bwd_dkdv", p)
    _ext.call("dsalt_attn_bwd_dq", p)
    if grouped:
        dk, dv = gqa_reduce(dk, prep.H_kv), gqa_reduce(dv, prep.H_kv)
    return dq, dk, dv, d_lw, dw


def gqa_reduce(x: torch.Tensor, h_kv: int) -> torch.Tensor:
    """``[T, H, D]`` per-query-head gradient -> ``[T, H_kv, D]``: each group of
    ``H / H_kv`` heads summed in fp32 and rounded once (``dsalt_gqa_reduce``)."""
    T, H, D = x.shape
    y = torch.empty(T, h_kv, D, dtype=x.dtype, device=x.device)
    p = _ext.GqaReduceParams(x=_ext.ptr(x), y=_ext.ptr(y), T=T, H=H, H_kv=h_kv, D=D,
                             dtype=_ext.dtype_code(x.dtype))
    _ext.call("dsalt_gqa_reduce", p)
    return y


# The dSᵀ tile scratch, kept per (device, stream) and only ever grown: its size
# changes with the band bound of each call, and a fresh multi-GB allocation per
# backward would churn the caching allocator.  Backward calls on one stream run
# in stream order, so they can share it.  A buffer that is outgrown stays
# allocated, since a captured CUDA graph may still hold its address.
_TILE_SCRATCH: dict = {}
_RETIRED: list = []


def _tile_scratch(dev: torch.device, nbytes: int) -> int:
    """1024-byte-aligned device address of at least ``nbytes`` of tile scratch."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (idx, _ext.current_stream_handle())
    buf = _TILE_SCRATCH.get(key)
    if buf is None or buf.numel() < nbytes + 1024:
        if buf is not None:
            _RETIRED.append(buf)
        buf = torch.empty(nbytes + 1024, dtype=torch.uint8, device=dev)
        _TILE_SCRATCH[key] = buf
    return buf.data_ptr() + (-buf.data_ptr()) % 1024


def compute_dtype(q: torch.Tensor) -> torch.dtype:
    """Arithmetic dtype of the op: the input dtype (fp16, bf16 or exact fp32)."""
    if q.dtype in (torch.float16, torch.bfloat16, torch.float32):
        return q.dtype
    raise TypeError(f"unsupported dtype {q.dtype}")


def check_inputs(q, k, v, cu_seqlens):
    for name, t in (("q", q), ("k", k), ("v", v)):
        _ext.require_cuda(t, name)
        if t.dim() != 3:
            raise ValueError(f"{name} must be [T, H, D], got {tuple(t.shape)}")
    # k, v may carry fewer (grouped) heads: H a multiple of H_kv, read in place
    if (k.shape != v.shape or k.shape[0] != q.shape[0] or k.shape[2] != q.shape[2]
            or k.shape[1] <= 0 or q.shape[1] % k.shape[1] != 0):
        raise ValueError(f"q/k/v shapes differ: {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)} "
                         "(k and v: [T, H_kv, D] with H a multiple of H_kv)")
    if q.shape[2] % 8 != 0 or not 8 <= q.shape[2] <= 256:
        raise ValueError(f"head_dim {q.shape[2]} not supported (multiples of 8 up to 256)")
    if cu_seqlens.dim() != 1 or cu_seqlens.shape[0] < 1:
        raise ValueError("cu_seqlens must be a 1-D tensor [S+1]")
