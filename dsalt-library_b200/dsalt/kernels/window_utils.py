"""Window and RoPE utilities (reference ``dsalt/kernels/window_utils.py``).

Plain torch helpers kept for API compatibility; the adaptive window of the op
comes from ``DSALTAttention`` (``dsalt_win_gate`` kernel), not from these.
"""

from __future__ import annotations

import torch


def compute_window_sizes(x_prev: torch.Tensor, n_min: int, n_max: int) -> torch.Tensor:
    """Constant window ``(n_min + n_max)//2`` for every token (reference :4-16)."""
    w = (n_min + n_max) // 2
    return torch.full((x_prev.shape[0],), float(w), device=x_prev.device, dtype=torch.float32)


def build_local_window_mask(seq_len: int, window_sizes: torch.Tensor, device: torch.device) -> torch.Tensor:
    """Boolean causal window mask ``[T, T]``: row i attends ``[i − w(i) + 1, i]`` (reference :19-37)."""
    rows = torch.arange(seq_len, device=device)
    w = window_sizes.clamp(min=1, max=seq_len).long()
    lo = (rows - w + 1).clamp(min=0)
    cols = torch.arange(seq_len, device=device)
    return (cols[None, :] >= lo[:, None]) & (cols[None, :] <= rows[:, None])


def build_local_window_mask_packed(cu_seqlens: torch.Tensor, window_sizes: torch.Tensor,
                                   total_len: int, device: torch.device) -> torch.Tensor:
    """Packed ``[T, T]`` window mask restricted to each sequence (reference :40-70)."""
    num_seqs = cu_seqlens.shape[0] - 1
    cu = cu_seqlens.to(device)
    lens = cu[1:] - cu[:-1]
    starts = cu[:-1]
    seq_ids = torch.repeat_interleave(torch.arange(num_seqs, device=device), lens)
    seq_off = torch.arange(total_len, device=device) - starts[seq_ids]
    w = window_sizes.clamp(min=1).long()
    lo = starts[seq_ids] + (seq_off - w + 1).clamp(min=0)
    hi = starts[seq_ids] + seq_off
    c = torch.arange(total_len, device=device)[None, :]
    same = seq_ids[:, None] == seq_ids[None, :]
    return same & (c >= lo[:, None]) & (c <= hi[:, None])


def apply_rotary_emb(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """Half-split RoPE on ``q`` and ``k`` (reference :73-88)."""
    half = q.shape[-1] // 2

    def _rot(x):
        return torch.cat([-x[..., half:], x[..., :half]], dim=-1)

    return q * cos + _rot(q) * sin, k * cos + _rot(k) * sin


def build_rope_cache(seq_len: int, head_dim: int, device: torch.device, dtype: torch.dtype = torch.float32,
                     base: float = 10000.0, scale: float = 1.0):
    """RoPE ``(cos, sin)`` cache ``[seq_len, head_dim]`` (reference :91-106)."""
    theta = 1.0 / (base ** (torch.arange(0, head_dim, 2, device=device, dtype=dtype) / head_dim))
    positions = torch.arange(seq_len, device=device, dtype=dtype) / scale
    emb = torch.cat([torch.outer(positions, theta)] * 2, dim=-1)
    return emb.cos(), emb.sin()
