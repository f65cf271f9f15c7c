"""Host-side helpers with the names of the reference's ``tops/utils.py``.

``pad_to_multiple`` (:38), ``prepare_lens`` (:61), ``prepare_chunk_indices`` (:70),
``assert_shape`` / ``assert_shape_or_none`` (:91/:110), ``cdiv``, ``align_up``,
``next_power_of_2``.  The GLA kernels do not need padding (ragged chunks are
handled in-kernel); these exist for callers of the reference API.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def next_power_of_2(n: int) -> int:
    return 1 if n <= 1 else 1 << (int(n) - 1).bit_length()


def cdiv(x, y: int):
    return (x + y - 1) // y


def align_up(x, align: int):
    return cdiv(x, align) * align


def pad_to_multiple(x: torch.Tensor, multiple, axis, val):
    multiple = [multiple] if isinstance(multiple, int) else list(multiple)
    axis = [axis] if isinstance(axis, int) else list(axis)
    assert len(multiple) == len(axis), f"Length of multiple {len(multiple)} must match length of axis {len(axis)}"
    pad = [0] * (2 * x.dim())
    for mu, ax in zip(multiple, axis):
        ax = ax % x.dim()
        r = x.shape[ax] % mu
        if r:
            pad[2 * (x.dim() - 1 - ax) + 1] = mu - r
    return F.pad(x, pad, value=val) if any(pad) else x


def prepare_lens(cu_seqlens: torch.Tensor) -> torch.Tensor:
    return cu_seqlens[1:] - cu_seqlens[:-1]


def prepare_chunk_indices(cu_seqlens: torch.Tensor, chunk_size: int) -> torch.Tensor:
    """[NT_total, 2] int32 rows (sequence id, chunk id within the sequence)."""
    lens = prepare_lens(cu_seqlens.long())
    n = cdiv(lens, chunk_size)
    seq_ids = torch.repeat_interleave(torch.arange(len(lens), device=cu_seqlens.device), n)
    starts = torch.cumsum(n, 0) - n
    block = torch.arange(int(n.sum()), device=cu_seqlens.device) - torch.repeat_interleave(starts, n)
    return torch.stack([seq_ids, block], 1).to(torch.int32)


def assert_shape_or_none(x, expected_shape, name="tensor"):
    if x is None:
        return
    assert_shape(x, expected_shape, name, allow_none=True)


def assert_shape(x, expected_shape, name="tensor", allow_none=False):
    if isinstance(x, (list, tuple)):
        names = name if isinstance(name, (list, tuple)) and len(name) == len(x) else None
        for i, t in enumerate(x):
            if t is None and allow_none:
                continue
            nm = names[i] if names else f"{name}_{i}"
            assert tuple(t.shape) == tuple(expected_shape), f"[{nm}] Expected shape {expected_shape}, got {t.shape}"
    else:
        assert tuple(x.shape) == tuple(expected_shape), f"[{name}] Expected shape {expected_shape}, got {x.shape}"
