"""Selector helpers on B200 (module name kept from the reference).

Reference: ``dsalt/kernels/selectors.py``.  The landmark top-k runs in the
``dsalt_select_topk`` CUDA kernel (shared-memory radix select, one CTA per
(head, sequence)); the score in ``dsalt_hybrid_scores``.  The packed-metadata
helpers are recomputed from the actual ``cu_seqlens`` on every call: the
reference caches them by ``(total_len, num_seqs)`` (:17-22, :51-54), which
returns stale tables for batches with equal totals but different lengths.
"""

from __future__ import annotations

import torch

from . import _ext
from .landmark_tokens_ker import hybrid_scores_per_head

_TOPK_MAX_LEN = 49152
_TOPK_MAX_K = 1024


def _host_cu(cu_seqlens: torch.Tensor, cu_list):
    if cu_list is not None:
        return [int(c) for c in cu_list]
    return [int(c) for c in cu_seqlens.detach().to("cpu").tolist()]


def _seq_meta(cu_seqlens: torch.Tensor, total: int, device: torch.device, cu_list: list | None = None):
    """``(num_seqs, lens, starts, seq_ids, seq_off, max_len)`` (reference :15-34), uncached."""
    num_seqs = cu_seqlens.shape[0] - 1
    cu = cu_seqlens.to(device)
    lens = (cu[1:] - cu[:-1])
    starts = cu[:-1]
    seq_ids = torch.repeat_interleave(torch.arange(num_seqs, device=device), lens)
    seq_off = torch.arange(total, device=device) - starts[seq_ids]
    hc = _host_cu(cu_seqlens, cu_list)
    max_len = max((hc[b + 1] - hc[b] for b in range(len(hc) - 1)), default=0)
    return num_seqs, lens, starts, seq_ids, seq_off, max_len


def _build_seq_block_map(cu_seqlens: torch.Tensor, block_m: int, device: torch.device,
                         cu_list: list | None = None) -> tuple[torch.Tensor, int]:
    """``(seq_block_map [total_blocks, 2] int32, total_blocks)`` (reference :37-67), uncached.

    The op itself builds this table on the device (``dsalt_build_schedule``);
    this helper keeps the reference's host-returning signature.
    """
    hc = _host_cu(cu_seqlens, cu_list)
    rows = []
    for b in range(len(hc) - 1):
        n = (hc[b + 1] - hc[b] + block_m - 1) // block_m
        rows.extend((b, j) for j in range(n))
    t = torch.tensor(rows, dtype=torch.int32).reshape(-1, 2).to(device)
    return t, len(rows)


def _score_block(x, W_V, alpha, n_heads, dh):
    return hybrid_scores_per_head(x, W_V, alpha, n_heads, dh)


def select_topk(scores: torch.Tensor, w_sizes: torch.Tensor, cu_seqlens: torch.Tensor, k_lmk: int,
                max_len: int) -> torch.Tensor:
    """``[H, S, k_lmk]`` int64 top-k positions (CUDA), -1 where fewer candidates exist.

    Tokens whose in-sequence offset is below their own ``w_sizes`` are excluded
    (reference :105-107).  Ties go to the lower position; entries are ordered by
    descending score (the reference's order is unspecified, ``sorted=False``).
    """
    _ext.require_cuda(scores, "scores")
    T, H = scores.shape
    S = cu_seqlens.shape[0] - 1
    out = torch.empty(H, S, k_lmk, dtype=torch.int64, device=scores.device)
    if k_lmk == 0 or S == 0:
        return out
    if k_lmk > _TOPK_MAX_K:
        raise ValueError(f"k_lmk={k_lmk} exceeds the top-k kernel limit {_TOPK_MAX_K}")
    if max_len > _TOPK_MAX_LEN:
        raise ValueError(f"sequence length {max_len} exceeds the top-k kernel limit {_TOPK_MAX_LEN}")
    sc = scores.detach().to(torch.float32).contiguous()
    ws = w_sizes.detach().to(device=scores.device, dtype=torch.float32).contiguous()
    cu = cu_seqlens.to(device=scores.device, dtype=torch.int32).contiguous()
    p = _ext.TopkParams(scores=_ext.ptr(sc), w_sizes=_ext.ptr(ws), cu_seqlens=_ext.ptr(cu),
                        idx=_ext.ptr(out), T=T, H=H, S=S, k=k_lmk, max_len=max(max_len, 1))
    _ext.call("dsalt_select_topk", p)
    return out


def _compute_landmark_indices(
    x:          torch.Tensor,
    W_V:        torch.Tensor,
    alpha:      torch.Tensor,
    w_sizes:    torch.Tensor,
    cu_seqlens: torch.Tensor,
    k_lmk:      int,
    n_min:      int,
    total_len:  int,
    cu_list:    list | None = None,
    head_dim:   int | None = None,
    xwv:        torch.Tensor | None = None,
):
    """Hard top-k landmark indices per (head, sequence) (reference :75-134).

    Returns ``(idx [H, S, k_lmk] int64, z_x, z_v)``; the selection is detached.
    ``xwv`` optionally passes ``x·W_Vᵀ`` (see ``hybrid_scores_per_head``).
    """
    n_heads = alpha.shape[0]
    dh = head_dim if head_dim is not None else W_V.shape[0] // n_heads
    with torch.no_grad():
        scores, z_x, z_v = hybrid_scores_per_head(x, W_V, alpha, n_heads, dh, xwv=xwv)
        hc = _host_cu(cu_seqlens, cu_list)
        max_len = max((hc[b + 1] - hc[b] for b in range(len(hc) - 1)), default=0)
        idx = select_topk(scores, w_sizes, cu_seqlens, k_lmk, max_len)
    return idx, z_x, z_v


def _build_landmark_kv(K: torch.Tensor, V: torch.Tensor, lmk_indices: torch.Tensor,
                       cu_seqlens: torch.Tensor, k_lmk: int, n_heads: int, head_dim: int):
    """Landmark keys/values ``[H, S, k, D]`` in slot order, zeros for -1 (reference :137-159).

    The op itself uses the position-sorted gather of ``dsalt_gather_landmarks``.
    """
    starts = cu_seqlens[:-1].to(K.device).long()
    safe = lmk_indices.clamp(min=0)
    abs_idx = starts[None, :, None] + safe
    h_idx = torch.arange(n_heads, device=K.device)[:, None, None]
    lk = K[abs_idx, h_idx, :]
    lv = V[abs_idx, h_idx, :]
    invalid = (lmk_indices < 0).unsqueeze(-1)
    return lk.masked_fill(invalid, 0.0).contiguous(), lv.masked_fill(invalid, 0.0).contiguous()
