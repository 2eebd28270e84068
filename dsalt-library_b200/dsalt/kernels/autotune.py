"""Fixed B200 tile configuration (replaces the reference's one-shot autotuner).

Reference: ``dsalt/kernels/autotune.py:55-278`` benchmarks Triton block configs
once per ``(head_dim, compute capability)`` on the first batch, and
``_maybe_autotune_train`` (``dsalt_triton_train.py:512-582``) does the same for the
training kernel.  The B200 kernels have one fixed shape per head_dim, set by the
tcgen05 MMA (M = 128 rows in 128 TMEM lanes) and the 227 KB shared-memory and
512-column TMEM budgets, and chosen from ncu measurements on B200 (the
per-kernel captures record tensor-pipe activity, issue rate and stalls).  The
table below states those shapes; nothing is benchmarked at run time.

The reference-named keys map onto them: ``BLOCK_M`` is the forward's query rows
per work item, ``BLOCK_N`` its keys per tile, ``BLOCK_N_BWD`` the keys per dK/dV
work item, ``num_warps`` the forward's warps.  The per-kernel entries give the
rest (warp roles, pipeline stages).  head_dim other than 64 and 128 runs on the
exact SIMT kernels (one warp per query row, no tiles).
"""

from __future__ import annotations

import torch

_TUNED_CONFIG: dict = {}


def _tiles(head_dim: int) -> dict:
    return {
        "BLOCK_M": 128, "BLOCK_N": 128, "BLOCK_N_BWD": 128, "num_warps": 12, "num_stages": 2,
        # attn_tc.cu: persistent, one CTA per SM over (head, 128-query block) items
        "fwd": {"query_rows": 128, "key_tile": 128, "kv_stages": 2, "threads": 384,
                "warps": {"softmax (two 64-column halves)": 8, "tma": 1, "mma_s": 1, "mma_pv": 1,
                          "scheduler": 1},
                "tmem_columns": {"S (double buffer)": 256, "O (one per half)": 2 * head_dim}},
        # attn_tc_bwd.cu: persistent, one CTA per SM over (head, 128-key block) items
        "bwd_dkdv": {"key_rows": 128, "query_tile": 64, "q_do_stages": 3, "record_stages": 4, "threads": 640,
                     "warps": {"rows (16-column quarters)": 16, "tma + tile store": 1, "mma_s_dv": 1,
                               "records": 1, "mma_dp_dk": 1},
                     "tmem_columns": {"S^T, dP^T (double buffer; P^T, dS^T written over them)": 256,
                                      "dK": head_dim, "dV": head_dim}},
        # attn_tc_dq.cu: persistent, dQ = dS·K over the stored dS^T tiles
        "bwd_dq": {"query_rows": 128, "key_block": 128, "stages": 3, "threads": 192,
                   "warps": {"loads": 1, "mma": 1, "epilogue": 4},
                   "tmem_columns": {"dQ (double buffer)": 2 * head_dim}},
    }


_B200_TILES = {64: _tiles(64), 128: _tiles(128)}


def _heuristic_config(head_dim: int, device: torch.device | None = None) -> dict:
    """The fixed configuration for ``head_dim`` (the SIMT kernels for other sizes)."""
    cfg = _B200_TILES.get(int(head_dim))
    if cfg is None:
        return {"BLOCK_M": 1, "BLOCK_N": 1, "BLOCK_N_BWD": 1, "num_warps": 8, "num_stages": 1,
                "simt": "one warp per query row over its attended keys"}
    return {k: (dict(v) if isinstance(v, dict) else v) for k, v in cfg.items()}


def get_tuned_config(head_dim: int, device: torch.device | None = None) -> dict:
    return _heuristic_config(head_dim, device)


def autotune_blocks(head_dim: int, device: torch.device, make_runner=None, verbose: bool = False) -> dict:
    """Return the fixed configuration; ``make_runner`` is not benchmarked."""
    cfg = _heuristic_config(head_dim, device)
    _TUNED_CONFIG[(int(head_dim),) + tuple(torch.cuda.get_device_capability(device))] = cfg
    return cfg
