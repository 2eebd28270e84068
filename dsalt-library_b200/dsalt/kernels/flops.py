"""Algorithmic work of the DSALT attention: attended (query, key) pairs.

``P = Σ_(seq, head, i) |W(i)| + |L(i)|`` with (training semantics)
``|W(i)| = min(⌊w̃_i⌋, i) + 1`` and ``|L(i)| = #{valid landmark p : p ≤ i ∧ p < i − w̃_i}``;
inference uses ``|W(i)| = min(w_i, i + 1)`` and ``p < i − w_i + 1``.
FLOPs: forward ``4·D·P``, backward ``10·D·P``.  Padded, masked or recomputed
work is not counted.  Computed on the device with torch (benchmark bookkeeping,
not part of the op).
"""

from __future__ import annotations

import torch


@torch.no_grad()
def attended_pairs(w: torch.Tensor, lmk_pos: torch.Tensor, cu_seqlens: torch.Tensor,
                   semantics: str = "train") -> int:
    dev = w.device
    cu = cu_seqlens.to(dev).long()
    S = cu.shape[0] - 1
    T = w.shape[0]
    lens = cu[1:] - cu[:-1]
    seq = torch.repeat_interleave(torch.arange(S, device=dev), lens)
    i = torch.arange(T, device=dev) - cu[:-1][seq]
    w32 = w.float()
    if semantics == "train":
        nw = torch.where(w32 >= 0, torch.minimum(torch.floor(w32), i.float()) + 1, torch.zeros_like(w32))
        win_lo = i.float() - w32
    else:
        wi = torch.clamp(w32.trunc(), min=1)
        nw = torch.minimum(wi, i.float() + 1)
        win_lo = i.float() - wi + 1
    H = lmk_pos.shape[0]
    total = int(nw.double().sum().item()) * H
    if lmk_pos.numel() == 0:
        return total
    for b in range(S):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        if s1 == s0:
            continue
        pos = lmk_pos[:, b, :].to(dev).long()                       # [H, k]
        valid = (pos >= 0) & (pos < s1 - s0)
        pf = pos.float()[:, :, None]                                # [H, k, 1]
        ii = i[s0:s1].float()[None, None, :]
        ok = valid[:, :, None] & (pf <= ii) & (pf < win_lo[s0:s1][None, None, :])
        total += int(ok.sum().item())
    return total


@torch.no_grad()
def scanned_pairs_fwd(w: torch.Tensor, lmk_pos: torch.Tensor, cu_seqlens: torch.Tensor,
                      semantics: str = "train", block_m: int = 128, block_n: int = 128) -> int:
    """(query, key) pairs the forward's Q·Kᵀ MMAs compute: per 128-row query block and
    head, the band tiles ``[min_i(i − W_i), max_i i]`` in 128-key tiles (the last one
    rounded up to 16 keys) plus the landmark tiles (valid slots rounded up to 16),
    times the block's 128 MMA rows (tcgen05 M = 128, also past the sequence end).
    Mirrors the tile walk of ``tc_fwd_kernel``; ``attended / scanned`` is the
    structural density of the band tiling."""
    dev = w.device
    cu = cu_seqlens.to(dev).long()
    S = cu.shape[0] - 1
    T = w.shape[0]
    lens = cu[1:] - cu[:-1]
    seq = torch.repeat_interleave(torch.arange(S, device=dev), lens)
    i = torch.arange(T, device=dev) - cu[:-1][seq]
    w32 = w.float()
    if semantics == "train":
        wt = w32
    else:
        wt = torch.clamp(w32.trunc(), min=1.0) - 1.0
    has_band = wt >= 0
    W = torch.floor(torch.clamp(wt, max=2.0 ** 30)).long()
    lo = torch.where(has_band, i - torch.minimum(W, i), torch.full_like(i, 1 << 40))
    H = lmk_pos.shape[0]
    total = 0
    for b in range(S):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        L = s1 - s0
        if L == 0:
            continue
        nb = (L + block_m - 1) // block_m
        pad = nb * block_m - L
        lo_b = torch.nn.functional.pad(lo[s0:s1], (0, pad), value=1 << 40).view(nb, block_m).min(1).values
        hi_b = torch.clamp(torch.arange(nb, device=dev) * block_m + block_m - 1, max=L - 1)
        span = torch.where(lo_b <= hi_b, hi_b - lo_b + 1, torch.zeros_like(hi_b))
        full, rem = span // block_n, span % block_n
        band_keys = full * block_n + (rem + 15) // 16 * 16
        if lmk_pos.numel():
            pos = lmk_pos[:, b, :].to(dev).long()
            n_valid = ((pos >= 0) & (pos < L)).sum(1)                      # [H]
            lfull, lrem = n_valid // block_n, n_valid % block_n
            lmk_keys = lfull * block_n + (lrem + 15) // 16 * 16           # [H]
        else:
            lmk_keys = torch.zeros(H, dtype=torch.long, device=dev)
        total += block_m * (int(band_keys.sum().item()) * H + int(lmk_keys.sum().item()) * nb)
    return total
