"""RMSNorm (reference ``dsalt/kernels/RMSENorm.py``), used by the model blocks.

On CUDA tensors of a supported width it runs the library's fused kernels
(``rmsnorm_cuda``); elsewhere ``F.rms_norm``, the reference's own computation.
"""

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import rmsnorm_cuda


class RMSENorm(nn.Module):
    """RMSNorm over the last dimension with a learnable scale; output in the input dtype."""

    def __init__(self, d_model: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model))
        self.normalized_shape = (d_model,)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if rmsnorm_cuda.supported(x):
            return rmsnorm_cuda.rms_norm(x, self.weight, self.eps)
        return F.rms_norm(x, self.normalized_shape, self.weight, self.eps).to(x.dtype)

    def add_forward(self, x: torch.Tensor, res: torch.Tensor):
        """``(x + res, self(x + res))``: the residual add in front of the norm, fused
        into the CUDA kernel when x and res share a dtype and shape."""
        if rmsnorm_cuda.supported(x) and res.dtype == x.dtype and res.shape == x.shape and res.is_cuda:
            return rmsnorm_cuda.add_rms_norm(x, res, self.weight, self.eps)
        s = x + res
        return s, self(s)
