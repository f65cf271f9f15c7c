"""Inter-chunk state scans -- the API of the reference's ``tops.ops.common.chunk_h``
(primatrix/pallas-kernel ``tops/ops/common/chunk_h.py``) for the key-wise gate path.

``chunk_fwd_h_kernel`` (:137) and ``chunk_bwd_dh_kernel`` (:605) return states
flattened over (batch, chunk) as ``[NS, H, K, V]`` (one per ``split_size`` tokens);
``chunk_fwd_h_ref`` (:277) / ``chunk_bwd_dh_ref`` (:399) return ``[B, NT, H, K, V]``.
The scalar-gate variants (``g`` [B,T,H], ``g_gamma`` [H]) belong to simple-GLA and
are not provided by this library.
"""
from __future__ import annotations

import torch

from ..gla import _core
from ..gla._core import _cuda, _f32, make_plan

__all__ = ["chunk_fwd_h_kernel", "chunk_fwd_h_ref", "chunk_bwd_dh_kernel", "chunk_bwd_dh_ref"]


def _no_scalar_gates(g, g_gamma, gv=None):
    if g is not None or g_gamma is not None or gv is not None:
        raise NotImplementedError("scalar / value-wise gates (simple-GLA) are not supported; pass gk")


def chunk_fwd_h_ref(k, v, g=None, g_gamma=None, gk=None, gv=None, h0=None, output_final_state=False,
                    states_in_fp32=False, cu_seqlens=None, cu_seqlens_cpu=None, chunk_size=64):
    """h [B, NT, H, K, V] (k.dtype, or fp32 with states_in_fp32) and ht [N, H, K, V] fp32."""
    _no_scalar_gates(g, g_gamma, gv)
    cu = cu_seqlens if cu_seqlens is not None else cu_seqlens_cpu
    p = make_plan(k, v.shape[-1], chunk_size, cu, 1.0)
    k, v = _cuda("k", k), _cuda("v", v)
    gc = _f32("gk", gk) if gk is not None else torch.zeros(k.shape, dtype=torch.float32, device=k.device)
    h, ht = _core.fwd_h(p, k, v, gc, _f32("h0", h0), True, True)
    if not output_final_state:
        ht = torch.zeros_like(ht)
    h = h.view(1 if p.cu_host is not None else p.B, -1, p.H, p.K, p.V)
    return (h if states_in_fp32 else h.to(k.dtype)), ht


def chunk_fwd_h_kernel(k, v, *, g=None, g_gamma=None, gk=None, gv=None, h0=None, output_final_state=False,
                       cu_seqlens=None, chunk_size=64, split_size=None, states_in_fp32=False, interpret=False):
    """Returns h [NS, H, K, V] (NS = B*T // split_size) and ht [N, H, K, V] (or None)."""
    _no_scalar_gates(g, g_gamma, gv)
    B, T, H, K = k.shape
    assert T % chunk_size == 0, "T mod chunk_size must equal to 0."
    BS = chunk_size if split_size is None else split_size
    assert BS % chunk_size == 0, f"The `split_size` (got {BS}) must be a multiple of `chunk_size` {chunk_size}"
    p = make_plan(k, v.shape[-1], chunk_size, cu_seqlens, 1.0)
    kk, vv = _cuda("k", k), _cuda("v", v)
    gc = _f32("gk", gk) if gk is not None else torch.zeros(kk.shape, dtype=torch.float32, device=kk.device)
    h, ht = _core.fwd_h(p, kk, vv, gc, _f32("h0", h0), True, bool(output_final_state))
    h = h[:: BS // chunk_size]
    h = h if states_in_fp32 else h.to(k.dtype)
    return h, (ht if output_final_state else None)


def chunk_bwd_dh_ref(q, k, v, gk, do, h0=None, dht=None, scale=1.0, cu_seqlens_cpu=None, chunk_size=64):
    """dh [B, NT, H, K, V] fp32 (gradient at each chunk's END state) and dh0 (when h0 or dht is given)."""
    p = make_plan(q, do.shape[-1], chunk_size, cu_seqlens_cpu, scale)
    q = _cuda("q", q)
    gc = _f32("gk", gk) if gk is not None else torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    dh, dh0 = _core.bwd_dh(p, q, gc, _cuda("do", do).to(q.dtype), _f32("dht", dht),
                           want_dh0=(h0 is not None or dht is not None))
    return dh.view(1 if p.cu_host is not None else p.B, -1, p.H, p.K, p.V), dh0


def chunk_bwd_dh_kernel(q, k, v, g=None, g_gamma=None, gk=None, do=None, dht=None, scale=1.0, output_dh0=False,
                        cu_seqlens=None, chunk_size=128, split_size=None, states_in_fp32=False, interpret=False):
    """dh [NS, H, K, V] (q.dtype unless states_in_fp32) and dh0 [N, H, K, V] when output_dh0."""
    _no_scalar_gates(g, g_gamma)
    B, T, H, K = q.shape
    assert T % chunk_size == 0, "T mod chunk_size must equal to 0."
    BS = chunk_size if split_size is None else split_size
    assert BS % chunk_size == 0, f"The `split_size` (got {BS}) must be a multiple of `chunk_size` {chunk_size}"
    p = make_plan(q, do.shape[-1], chunk_size, cu_seqlens, scale)
    qq = _cuda("q", q)
    gc = _f32("gk", gk) if gk is not None else torch.zeros(qq.shape, dtype=torch.float32, device=qq.device)
    dh, dh0 = _core.bwd_dh(p, qq, gc, _cuda("do", do).to(qq.dtype), _f32("dht", dht), want_dh0=bool(output_dh0))
    dh = dh[:: BS // chunk_size]
    dt = torch.float32 if states_in_fp32 else q.dtype
    return dh.to(dt), (None if dh0 is None else dh0.to(dt))
