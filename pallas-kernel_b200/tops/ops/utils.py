"""Small helpers of the reference's ``tops/ops/utils.py`` (``exp`` :6, ``is_tpu_runtime`` :9)."""
from __future__ import annotations

import torch


def exp(x: torch.Tensor) -> torch.Tensor:
    return torch.exp(x.float())


def is_tpu_runtime() -> bool:
    """Always False: this build targets NVIDIA B200 (sm_100a)."""
    return False
