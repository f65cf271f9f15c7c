"""CPU oracle for the simple-GLA operators (one scalar log-gate per token and head) --
TEST INFRASTRUCTURE.

Only ``tests/`` may import this module; the CUDA library never calls into it.

The reference's Torch CPU restatement (``tests/src/ops/simple_gla/chunk.py``) builds
the chunk-local cumsum of the effective gate g[b, t, h] + g_gamma[h] (``build_gc``,
:72-137) and runs the GLA chunk steps with that scalar broadcast over K
(:140-430 forward, :430-894 backward).  A scalar gate is the GLA gate with every K
entry equal, and the reference's own tests check exactly that equivalence
(``tests/ops/simple_gla/test_pallas_chunk_simple_gla.py:98-133,236-268``), so this
oracle restates simple GLA as the GLA oracle on the broadcast gate; the scalar
gate's gradient is the K-sum of the GLA gate gradient.  Pinned against fixtures
from the reference's Torch code by ``tests/test_simple_gla_oracle.py``.
"""
from __future__ import annotations

import numpy as np

from . import gla_oracle as O

__all__ = ["effective_gate", "chunk_simple_gla_fwd", "chunk_simple_gla_bwd", "simple_gla_naive"]


def effective_gate(shape, g=None, g_gamma=None, dtype=np.float64):
    """[B, T, H, K] per-step log-gate: g[b, t, h] (+ g_gamma[h]) broadcast over K, or None."""
    B, T, H, K = shape
    x = None
    if g is not None:
        x = np.asarray(g, dtype)[..., None]
    if g_gamma is not None:
        gg = np.asarray(g_gamma, dtype).reshape(1, 1, H, 1)
        x = gg if x is None else x + gg
    return None if x is None else np.broadcast_to(x, (B, T, H, K)).copy()


def chunk_simple_gla_fwd(q, k, v, g=None, g_gamma=None, scale=None, initial_state=None, output_final_state=False,
                         cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """-> (o, ht).  Follows tests/src/ops/simple_gla/chunk.py:329-427."""
    gk = effective_gate(np.shape(q), g, g_gamma, dtype)
    if gk is None:
        gk = np.zeros(np.shape(q), dtype)
    _, _, _, ht, o = O.chunk_gla_fwd(q, k, v, gk, None, scale, initial_state, output_final_state, cu_seqlens,
                                     chunk_size, dtype=dtype)
    return o, ht


def chunk_simple_gla_bwd(q, k, v, g=None, g_gamma=None, scale=None, initial_state=None, do=None, dht=None,
                         cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """-> (dq, dk, dv, dg [B, T, H] or None, dh0).  Follows tests/src/ops/simple_gla/chunk.py:784-894."""
    gk = effective_gate(np.shape(q), g, g_gamma, dtype)
    if gk is None:
        gk = np.zeros(np.shape(q), dtype)
    dq, dk, dv, dgk, dh0 = O.chunk_gla_bwd(q, k, v, gk, None, scale, initial_state, None, None, do, dht,
                                           cu_seqlens, chunk_size, dtype=dtype)
    dg = None if g is None else dgk.sum(-1)
    return dq, dk, dv, dg, dh0


def simple_gla_naive(q, k, v, g=None, g_gamma=None, scale=None, initial_state=None, output_final_state=False,
                     cu_seqlens=None, dtype=np.float64):
    """Per-step recurrence of tops/ops/simple_gla/naive.py:5-94 (g, g_gamma broadcastable to
    [B, T, H, K]) -> (o, S)."""
    shape = np.shape(q)
    gk = None
    if g is not None:
        gk = np.broadcast_to(np.asarray(g, dtype), shape)
    if g_gamma is not None:
        gg = np.broadcast_to(np.asarray(g_gamma, dtype), shape)
        gk = gg if gk is None else gk + gg
    if gk is None:
        gk = np.zeros(shape, dtype)
    return O.naive_recurrent_gla(q, k, v, np.ascontiguousarray(gk), scale, initial_state, output_final_state,
                                 cu_seqlens, dtype=dtype)
