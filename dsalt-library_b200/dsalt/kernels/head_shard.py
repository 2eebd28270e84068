"""Head sharding of the DSALT attention op over the GPUs of one node.

Every (sequence, head) unit of the op is independent: the window, the landmark
set and the softmax are per head, and the landmark z-statistics span tokens, not
heads (``landmark_tokens_ker.py:47-55``: ``z_x`` depends on x only, ``z_v`` is per
head).  So the op splits over heads with no exchange inside it: rank ``r`` of
``world`` runs heads ``[h0, h1)`` of every sequence, one launch over the whole
packed batch.  An optional all-gather along heads reassembles ``O`` (or any
``[T, H_shard, ...]`` result) on every rank.

The reference has no sharded op (its only parallel code is DDP,
``dsalt/training/trainer.py:366-373``); this module is the B200 build's.
"""

from __future__ import annotations

import torch


def head_range(n_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Heads ``[h0, h1)`` of ``rank``: contiguous blocks, as even as ``n_heads`` allows
    (the first ``n_heads % world`` ranks take one head more)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_heads < world:
        raise ValueError(f"{n_heads} heads cannot be split over {world} ranks")
    base, extra = divmod(n_heads, world)
    h0 = rank * base + min(rank, extra)
    return h0, h0 + base + (1 if rank < extra else 0)


def shard_heads(t: torch.Tensor, h0: int, h1: int, dim: int) -> torch.Tensor:
    """Contiguous copy of heads ``[h0, h1)`` of ``t`` along ``dim``."""
    return t.narrow(dim, h0, h1 - h0).contiguous()


def shard_op_inputs(q, k, v, lmk_pos, lmk_logw, rank: int, world: int, extra: dict | None = None) -> dict:
    """This rank's slice of the training op's inputs: ``q [T, H, D]`` and any other
    ``[T, H, ...]`` tensors in ``extra`` along dim 1, ``lmk_pos, lmk_logw [H, S, k]``
    along dim 0, and ``k, v [T, H_kv, D]``.  With grouped kv heads (``H_kv < H``)
    whole groups stay together: the kv heads are split over the ranks and each rank
    takes the query heads of its kv heads.  Per-token inputs (``w̃``, ``cu_seqlens``)
    are shared by all heads and stay whole."""
    n_rep = q.shape[1] // k.shape[1]
    g0, g1 = head_range(k.shape[1], world, rank)
    h0, h1 = g0 * n_rep, g1 * n_rep
    out = {"q": shard_heads(q, h0, h1, 1), "k": shard_heads(k, g0, g1, 1), "v": shard_heads(v, g0, g1, 1),
           "lmk_pos": shard_heads(lmk_pos, h0, h1, 0), "lmk_logw": shard_heads(lmk_logw, h0, h1, 0),
           "heads": (h0, h1)}
    for name, t in (extra or {}).items():
        out[name] = shard_heads(t, h0, h1, 1)
    return out


def gather_heads(shard: torch.Tensor, n_heads: int, group=None, n_rep: int = 1) -> torch.Tensor:
    """All-gather ``[T, H_r, ...]`` shards along dim 1 into ``[T, n_heads, ...]`` on every rank
    (``n_rep`` query heads per kv head: the split of ``shard_op_inputs``).

    One collective: each rank's shard is padded to the largest shard's head count,
    gathered rank-major with ``all_gather_into_tensor`` and reordered to head order."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world == 1:
        return shard
    sizes = [(g0 * n_rep, g1 * n_rep) for g0, g1 in (head_range(n_heads // n_rep, world, r) for r in range(world))]
    hmax = max(h1 - h0 for h0, h1 in sizes)
    T, rest = shard.shape[0], tuple(shard.shape[2:])
    h0, h1 = sizes[rank]
    if shard.shape[1] != h1 - h0:
        raise ValueError(f"rank {rank} holds {shard.shape[1]} heads, expected {h1 - h0}")
    send = shard
    if shard.shape[1] != hmax:
        send = shard.new_zeros((T, hmax) + rest)
        send[:, :shard.shape[1]] = shard
    recv = shard.new_empty((world * T, hmax) + rest)   # rank-major blocks of [T, hmax, ...]
    dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
    recv = recv.view((world, T, hmax) + rest)
    parts = [recv[r, :, :h1 - h0] for r, (h0, h1) in enumerate(sizes)]
    return torch.cat(parts, dim=1)


def reduce_window_grad(partial: torch.Tensor, out_dtype: torch.dtype | None = None, group=None) -> torch.Tensor:
    """∂loss/∂w̃ of the whole op from the head shards.

    ``w̃ [T]`` is shared by every head, so its gradient is a sum over heads
    (``dsalt_triton_train.py:748``): with the heads split over the ranks, each rank
    holds the sum over its own heads.  One ``all_reduce`` (SUM, fp32) adds the
    shards; with ``out_dtype`` the total is then rounded once to that dtype and kept
    in fp32, as the reference's ``d_w_tok.to(out_dtype)`` (``:756``) reaches an fp32
    ``w̃``.  The training op rounds each rank's own sum already (``grad_round``),
    so the total differs from the unsharded op's by at most those per-rank
    roundings.  Outside the timed op: a ``[T]`` fp32 exchange."""
    import torch.distributed as dist
    total = partial.detach().to(torch.float32).clone()
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    if out_dtype is not None and out_dtype != torch.float32:
        total = total.to(out_dtype).to(torch.float32)
    return total
