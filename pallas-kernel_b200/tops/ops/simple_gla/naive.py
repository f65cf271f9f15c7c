"""``simple_gla_naive`` -- the step-loop definition of simple GLA
(reference tops/ops/simple_gla/naive.py:5-94).

On B200 the definition runs as this library's recurrence kernel (the decode path) on the
effective gate g (+ g_gamma), both broadcastable to [B, T, H, K].
"""
from __future__ import annotations

import torch

from ..gla.fused_recurrent import fused_recurrent_gla

__all__ = ["simple_gla_naive"]


def simple_gla_naive(q, k, v, *, g=None, g_gamma=None, scale=None, initial_state=None, output_final_state=False,
                     chunk_size: int = 64, cu_seqlens_cpu=None):
    """h_t = h_{t-1} e^{g_t} + k_t^T v_t;  o_t = (scale q_t)^T h_t.

    Returns o [B, T, H, V] (fp32, as the reference) and the final state [N, H, K, V] (fp32)
    or None.  ``chunk_size`` is accepted for signature parity and unused.
    """
    B, T, H, K = q.shape
    V = v.shape[-1]
    gk = None
    if g is not None:
        gk = torch.broadcast_to(g.float(), (B, T, H, K))
    if g_gamma is not None:
        gg = torch.broadcast_to(g_gamma.float().to(q.device), (B, T, H, K))
        gk = gg if gk is None else gk + gg
    if gk is not None:
        gk = gk.contiguous()
    if cu_seqlens_cpu is not None:
        q, k, v = q.reshape(1, -1, H, K), k.reshape(1, -1, H, K), v.reshape(1, -1, H, V)
        gk = None if gk is None else gk.reshape(1, -1, H, K)
    o, ht = fused_recurrent_gla(q, k, v, gk=gk, scale=scale, initial_state=initial_state,
                                output_final_state=output_final_state, cu_seqlens=cu_seqlens_cpu)
    return o.float().reshape(B, T, H, V), ht
