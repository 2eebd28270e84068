"""Serializable configuration of the DSALT model (reference dsalt/model/config.py)."""

from __future__ import annotations

import json
from dataclasses import dataclass, asdict, fields
from pathlib import Path


@dataclass
class DSALTConfig:
    """Hyperparameters of :class:`~dsalt.model.dsalt_lm.DSALTLMHeadModel` (same fields as the reference)."""

    vocab_size: int
    d_model: int
    n_layers: int
    n_heads: int
    n_min: int
    n_max: int
    k_lmk: int
    max_seq_len: int
    d_ff: int | None = None
    dropout: float = 0.0
    yarn_scale: float = 1.0
    tie_weights: bool = True
    n_kv_heads: int | None = None
    qkv_bias: bool = False
    rope_base: float = 10000.0
    padding_idx: int | None = None
    lm_head_chunk_size: int = 2048
    loss_fn: str = "chunked"
    aux_loss_weight: float = 0.0

    def __post_init__(self) -> None:
        if self.d_model % self.n_heads != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by n_heads ({self.n_heads})")
        if not (0 <= self.n_min <= self.n_max):
            raise ValueError(f"required 0 <= n_min <= n_max, got n_min={self.n_min} n_max={self.n_max}")
        if self.k_lmk < 0:
            raise ValueError(f"k_lmk must be >= 0, got {self.k_lmk}")
        if self.n_kv_heads is not None and (self.n_kv_heads <= 0 or self.n_heads % self.n_kv_heads != 0):
            raise ValueError(f"n_heads ({self.n_heads}) must be a positive multiple of n_kv_heads "
                             f"({self.n_kv_heads}) for grouped-query attention")
        if self.loss_fn not in ("auto", "chunked", "liger"):
            raise ValueError(f"loss_fn must be 'auto', 'chunked' or 'liger', got {self.loss_fn!r}")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict) -> "DSALTConfig":
        known = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in known})

    def save(self, path: str | Path) -> None:
        Path(path).write_text(json.dumps(self.to_dict(), indent=2), encoding="utf-8")

    @classmethod
    def load(cls, path: str | Path) -> "DSALTConfig":
        return cls.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))
