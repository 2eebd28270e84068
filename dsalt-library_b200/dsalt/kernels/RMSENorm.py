"""RMSNorm (reference ``dsalt/kernels/RMSENorm.py``), used by the model blocks."""

import torch
import torch.nn as nn
import torch.nn.functional as F


class RMSENorm(nn.Module):
    """RMSNorm over the last dimension with a learnable scale; output in the input dtype."""

    def __init__(self, d_model: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model))
        self.normalized_shape = (d_model,)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.rms_norm(x, self.normalized_shape, self.weight, self.eps).to(x.dtype)
