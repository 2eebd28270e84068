"""DSALT sparse attention, B200-native build.

Drop-in for the reference package ``dsalt`` (LeonardoCofone/dsalt-library):
the same module paths and public names for the attention path, with the
kernels rewritten as hand-written sm_100a CUDA (``libdsalt_b200.so``).
"""

from dsalt.kernels import (  # noqa: F401
    dsalt_triton_attention,
    dsalt_triton_train_attention,
    RMSENorm,
    compute_window_sizes,
    build_local_window_mask,
    build_local_window_mask_packed,
    apply_rotary_emb,
    build_rope_cache,
    hybrid_scores_per_head,
    compute_hybrid_scores,
    select_landmarks,
    soft_landmark_weights,
    HybridEnergyLandmarkSelector,
    LigerFusedLinearCrossEntropyFunction,
)

__version__ = "1.0.0+b200"
