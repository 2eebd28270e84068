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
