"""RMSNorm (reference tops/modules/layernorm.py:6): x * rsqrt(mean(x^2) + eps) * weight in
fp32, output in the input dtype."""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["RMSNorm"]


class RMSNorm(nn.Module):
    """RMSNorm over the last dim, fp32 arithmetic, output in the input dtype."""

    def __init__(self, hidden_size: int, elementwise_affine: bool = True, eps: float = 1e-5, dtype=None, device=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size, dtype=dtype, device=device)) if elementwise_affine else None

    def forward(self, x):
        w = None if self.weight is None else self.weight.float()
        return F.rms_norm(x.float(), (x.shape[-1],), w, self.eps).to(x.dtype)
