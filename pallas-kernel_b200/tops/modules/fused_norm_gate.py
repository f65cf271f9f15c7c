"""Fused RMSNorm x swish output gate: y = rmsnorm(x) * weight * silu(g) over the last dim.

Reference: ``FusedRMSNormGated`` (tops/modules/fused_norm_gate.py:28; its torch gold
tests/src/modules/fused_norm_gate.py:30-44), applied per head by the GLA layer
(tops/layers/gla.py:323-329).  Forward and backward run in ``layer.cu``
(``tops_gla_norm_gate_fwd`` / ``_bwd``), fp32 arithmetic on fp32 or bf16 tensors.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import _C


def _check(x):
    if not x.is_cuda:
        raise RuntimeError("fused_rms_norm_gated needs CUDA tensors (the kernels are the only implementation)")
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"fused_rms_norm_gated: unsupported dtype {x.dtype} (float32 or bfloat16)")


class _NormGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, g, weight, eps):
        _check(x)
        shape = x.shape
        V = shape[-1]
        xc = x.contiguous()
        gc = g.to(x.dtype).contiguous()
        w = None if weight is None else weight.to(x.dtype).contiguous()
        rows = xc.numel() // V
        y = torch.empty_like(xc)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        _C.call("tops_gla_norm_gate_fwd", rows, V, _C.dtype_code(x.dtype), float(eps), _C.ptr(xc), _C.ptr(gc),
                _C.ptr(w), _C.ptr(y), _C.ptr(rstd), _C.stream_of(xc))
        ctx.save_for_backward(xc, gc, w, rstd)
        ctx.has_w = weight is not None
        ctx.w_dtype = None if weight is None else weight.dtype
        ctx.g_dtype = g.dtype
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        xc, gc, w, rstd = ctx.saved_tensors
        V = xc.shape[-1]
        rows = xc.numel() // V
        dyc = dy.to(xc.dtype).contiguous()
        dx = torch.empty_like(xc)
        dg = torch.empty_like(gc)
        dw = torch.empty(V, dtype=xc.dtype, device=xc.device) if ctx.has_w else None
        nws = int(_C.lib().tops_gla_norm_gate_bwd_workspace_size(rows, V)) if ctx.has_w else 0
        ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=xc.device) if nws else None
        _C.call("tops_gla_norm_gate_bwd", rows, V, _C.dtype_code(xc.dtype), _C.ptr(dyc), _C.ptr(xc), _C.ptr(gc),
                _C.ptr(w), _C.ptr(rstd), _C.ptr(dx), _C.ptr(dg), _C.ptr(dw), _C.ptr(ws), nws, _C.stream_of(xc))
        return dx, dg.to(ctx.g_dtype), (None if dw is None else dw.to(ctx.w_dtype)), None


def fused_rms_norm_gated(x: torch.Tensor, g: torch.Tensor, weight: torch.Tensor | None = None,
                         eps: float = 1e-5) -> torch.Tensor:
    """rmsnorm(x) * weight * silu(g) over the last dim (x, g same shape; weight [V] or None)."""
    return _NormGate.apply(x, g, weight, eps)


class FusedRMSNormGated(nn.Module):
    """``FusedRMSNormGated(hidden_size, elementwise_affine=True, eps=1e-5)``; ``forward(x, g)``."""

    def __init__(self, hidden_size: int, elementwise_affine: bool = True, eps: float = 1e-5, device=None,
                 dtype=None):
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.elementwise_affine = elementwise_affine
        if elementwise_affine:
            self.weight = nn.Parameter(torch.ones(hidden_size, device=device, dtype=dtype))
        else:
            self.register_parameter("weight", None)

    def forward(self, x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        return fused_rms_norm_gated(x, g, self.weight, self.eps)
