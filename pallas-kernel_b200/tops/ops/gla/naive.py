"""``naive_recurrent_gla`` -- the step-loop definition of GLA (reference tops/ops/gla/naive.py:5).

On B200 the definition runs as the same recurrence kernel as the decode path;
the output is cast back to the input dtype as the reference's naive form does.
"""
from __future__ import annotations

from .fused_recurrent import fused_recurrent_gla


def naive_recurrent_gla(q, k, v, gk, scale=None, initial_state=None, output_final_state=False, cu_seqlens=None):
    """h_t = h_{t-1} e^{gk_t} + k_t^T v_t;  o_t = (scale q_t)^T h_t.

    Returns o [B, T, H, V] in q's dtype and the final state [N, H, K, V] (fp32) or None.
    """
    o, ht = fused_recurrent_gla(q, k, v, gk=gk, scale=scale, initial_state=initial_state,
                                output_final_state=output_final_state, cu_seqlens=cu_seqlens)
    return o.to(q.dtype), ht
