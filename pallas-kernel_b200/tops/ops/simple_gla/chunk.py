"""Simple GLA (one scalar log-gate per token and head) on B200 -- the API of the
reference's ``tops.ops.simple_gla`` (tops/ops/simple_gla/__init__.py:1-3).

A scalar gate is the GLA gate with all K entries equal; the reference's own tests check
that simple GLA equals GLA on the gate broadcast over K
(tests/ops/simple_gla/test_pallas_chunk_simple_gla.py:98-133, :236-268).  These operators
therefore run this library's GLA chunk kernels on the effective per-step gate
``g[b, t, h] + g_gamma[h]`` broadcast to [B, T, H, K] (the reference's Torch code builds
the same effective gate before its chunk-local cumsum, tests/src/ops/simple_gla/
chunk.py:72-137); the scalar gate's gradient is the K-sum of the GLA gate gradient.

Lengths need not be multiples of the chunk size and K, V need not be multiples of 128
(the reference's Pallas operator asserts both, tops/ops/simple_gla/chunk.py:493-496).
"""
from __future__ import annotations

import torch

from ..gla import _core
from ..gla._core import _cuda, _f32, make_plan
from ..gla.chunk import _check_qkv, chunk_gla

__all__ = ["chunk_simple_gla", "chunk_simple_gla_fwd", "chunk_simple_gla_bwd"]


def _gate(q, g, g_gamma):
    """Effective log-gate broadcast to q's shape (a view; differentiable), or None."""
    B, T, H, K = q.shape
    x = None
    if g is not None:
        assert tuple(g.shape) == (B, T, H), f"Expected g shape {(B, T, H)}, got {tuple(g.shape)}"
        x = _cuda("g", g).float().unsqueeze(-1)
    if g_gamma is not None:
        assert tuple(g_gamma.shape) == (H,), f"Expected g_gamma shape {(H,)}, got {tuple(g_gamma.shape)}"
        gg = _cuda("g_gamma", g_gamma).float().view(1, 1, H, 1)
        x = gg if x is None else x + gg
    return None if x is None else x.expand(B, T, H, K)


def _check_state(name, t, N, H, K, V):
    if t is not None:
        assert tuple(t.shape) == (N, H, K, V), f"Expected {name} shape {(N, H, K, V)}, got {tuple(t.shape)}"


def chunk_simple_gla_fwd(q, k, v, *, g=None, g_gamma=None, scale=None, h0=None, use_ht: bool = False,
                         cu_seqlens=None, chunk_size: int = 64):
    """Forward -> ``(o, ht)``.  Mirrors tops/ops/simple_gla/chunk.py:471.

    q, k [B, T, H, K]; v [B, T, H, V]; g [B, T, H] raw per-step log gates or None;
    g_gamma [H] constant per-head log decay or None; h0 [N, H, K, V]; ``use_ht``: return
    the final state (fp32), else None.  ``cu_seqlens`` [N+1] packs N sequences (B = 1).
    """
    _check_qkv(q, k, v)
    p = make_plan(q, v.shape[-1], chunk_size, cu_seqlens, scale)
    _check_state("h0", h0, p.N, p.H, p.K, p.V)
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    gk = _gate(q, g, g_gamma)
    o, ht, _ = _core.chunk_fwd(p, q, k, v, _f32("g", gk), _f32("h0", h0), bool(use_ht), False)
    return o, (ht if use_ht else None)


def chunk_simple_gla_bwd(q, k, v, g_gamma, scale, initial_state, do, dht, chunk_size: int = 64):
    """Backward -> ``(dq, dk, dv, dh0)`` (dh0 only when ``initial_state`` is given).
    Mirrors tops/ops/simple_gla/chunk.py:538-615 (g_gamma only; its gradient is not
    returned, as in the reference)."""
    _check_qkv(q, k, v)
    assert do.shape == v.shape, f"Expected do shape {tuple(v.shape)}, got {tuple(do.shape)}"
    p = make_plan(q, v.shape[-1], chunk_size, None, scale)
    _check_state("initial_state", initial_state, p.N, p.H, p.K, p.V)
    _check_state("dht", dht, p.N, p.H, p.K, p.V)
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    gk = _gate(q, None, g_gamma)
    do = _cuda("do", do).to(q.dtype)
    want = initial_state is not None
    dq, dk, dv, _, dh0 = _core.chunk_bwd(p, q, k, v, _f32("g", gk), _f32("initial_state", initial_state), do,
                                         _f32("dht", dht), want_dh0=want)
    return dq, dk, dv, (dh0 if want else None)


def chunk_simple_gla(q, k, v, g=None, g_gamma=None, scale=None, initial_state=None, output_final_state=False,
                     cu_seqlens=None, chunk_size: int = 64):
    """Differentiable simple GLA -> ``(o, final_state or None)``.

    Gradients flow to q, k, v, ``g`` ([B, T, H]: the K-sum of the GLA gate gradient),
    ``g_gamma`` ([H]: summed over batch, time and K) and ``initial_state``.
    """
    _check_qkv(q, k, v)
    return chunk_gla(q, k, v, g=_gate(q, g, g_gamma), scale=scale, initial_state=initial_state,
                     output_final_state=output_final_state, cu_seqlens=cu_seqlens, chunk_size=chunk_size)
