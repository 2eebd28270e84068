"""DSALT kernels for B200 (sm_100a).

Public names follow the reference's ``dsalt.kernels``.  The attention ops
(``dsalt_triton_attention``, ``dsalt_triton_backward``, and the training op in
``dsalt_triton_train``) run hand-written CUDA through ``libdsalt_b200.so``;
importing this package does not load the library, the first op call does (and
raises if it is missing).  ``LigerFusedLinearCrossEntropyFunction`` (a Triton
loss kernel, outside the attention path) is not provided and is ``None``.
"""

from .RMSENorm import RMSENorm
from .window_utils import (
    compute_window_sizes,
    build_local_window_mask,
    build_local_window_mask_packed,
    apply_rotary_emb,
    build_rope_cache,
)
from .landmark_tokens_ker import (
    hybrid_scores_per_head,
    compute_hybrid_scores,
    select_landmarks,
    soft_landmark_weights,
    HybridEnergyLandmarkSelector,
)
from .dsalt_triton_bwd import dsalt_triton_backward
from .dsalt_triton_attn import dsalt_triton_attention
from .dsalt_triton_train import dsalt_triton_train_attention
from .autotune import autotune_blocks, get_tuned_config

LigerFusedLinearCrossEntropyFunction = None
_TRITON_OK = True  # the CUDA ops play the role the Triton ops had

__all__ = [
    "dsalt_triton_backward",
    "LigerFusedLinearCrossEntropyFunction",
    "dsalt_triton_attention",
    "dsalt_triton_train_attention",
    "autotune_blocks",
    "get_tuned_config",
    "RMSENorm",
    "compute_window_sizes",
    "build_local_window_mask",
    "build_local_window_mask_packed",
    "apply_rotary_emb",
    "build_rope_cache",
    "hybrid_scores_per_head",
    "compute_hybrid_scores",
    "select_landmarks",
    "soft_landmark_weights",
    "HybridEnergyLandmarkSelector",
]
