"""Causal depthwise short convolution (reference tops/modules/convolution.py:6)."""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

__all__ = ["ShortConvolution"]


class ShortConvolution(nn.Module):
    """Causal depthwise conv1d over time with an optional activation (reference
    tops/modules/convolution.py; torch gold tests/src/modules/convolution.py).  Fixed-length
    batches only; the decode cache holds the last ``kernel_size - 1`` inputs."""

    def __init__(self, hidden_size: int, kernel_size: int = 4, bias: bool = False, activation: str | None = "silu"):
        super().__init__()
        self.hidden_size, self.kernel_size = hidden_size, kernel_size
        self.weight = nn.Parameter(torch.empty(hidden_size, 1, kernel_size))
        self.bias = nn.Parameter(torch.zeros(hidden_size)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        self.activation = activation

    def forward(self, x, cache=None, output_final_state=False, cu_seqlens=None):
        if cu_seqlens is not None:
            raise NotImplementedError("ShortConvolution: packed (cu_seqlens) inputs are not supported")
        B, T, D = x.shape
        xt = x.transpose(1, 2)  # [B, D, T]
        prev = cache if cache is not None else x.new_zeros(B, D, self.kernel_size - 1)
        xin = torch.cat([prev.to(x.dtype), xt], -1)
        y = F.conv1d(xin, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype),
                     groups=D)
        if self.activation in ("silu", "swish"):
            y = F.silu(y)
        new_cache = xin[..., -(self.kernel_size - 1):].detach() if output_final_state else None
        return y.transpose(1, 2), new_cache
