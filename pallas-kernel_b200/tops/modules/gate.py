"""Gate activation of the GLA layer: gk = logsigmoid(x) / normalizer (optionally clamped
from below), returned in fp32 for the chunked op (reference tops/layers/gla.py:285-287).
Forward and backward run in ``layer.cu`` (``tops_gla_gate_logsigmoid_fwd`` / ``_bwd``)."""
from __future__ import annotations

import torch

from .. import _C


class _Gate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, normalizer, clamp_min):
        if not x.is_cuda:
            raise RuntimeError("gate_logsigmoid needs CUDA tensors (the kernels are the only implementation)")
        xc = x.contiguous()
        out = torch.empty(xc.shape, dtype=torch.float32, device=x.device)
        has = clamp_min is not None
        _C.call("tops_gla_gate_logsigmoid_fwd", xc.numel(), _C.dtype_code(xc.dtype), float(normalizer),
                float(clamp_min) if has else 0.0, int(has), _C.ptr(xc), _C.ptr(out), _C.stream_of(xc))
        ctx.save_for_backward(xc)
        ctx.normalizer, ctx.clamp_min = normalizer, clamp_min
        return out

    @staticmethod
    def backward(ctx, dy):
        (xc,) = ctx.saved_tensors
        dyc = dy.float().contiguous()
        dx = torch.empty_like(xc)
        has = ctx.clamp_min is not None
        _C.call("tops_gla_gate_logsigmoid_bwd", xc.numel(), _C.dtype_code(xc.dtype), float(ctx.normalizer),
                float(ctx.clamp_min) if has else 0.0, int(has), _C.ptr(xc), _C.ptr(dyc), _C.ptr(dx),
                _C.stream_of(xc))
        return dx, None, None


def gate_logsigmoid(x: torch.Tensor, normalizer: float = 16.0, clamp_min: float | None = None) -> torch.Tensor:
    """logsigmoid(x) / normalizer (clamped from below when clamp_min is given), fp32."""
    return _Gate.apply(x, normalizer, clamp_min)
