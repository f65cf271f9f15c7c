"""``fused_chunk_gla`` -- alias of ``chunk_gla`` (reference tops/ops/gla/fused_chunk.py:4-30).

In the reference (and in FLA) the fused-chunk entry point delegates to
``chunk_gla`` with the same arguments; the default chunk size is 16.
"""
from __future__ import annotations

from .chunk import chunk_gla


def fused_chunk_gla(q, k, v, g, scale=None, initial_state=None, output_final_state=False, cu_seqlens=None,
                    chunk_size=16):
    """Fused chunk GLA: delegates to :func:`chunk_gla` (same shapes and outputs)."""
    return chunk_gla(q=q, k=k, v=v, g=g, scale=scale, initial_state=initial_state,
                     output_final_state=output_final_state, cu_seqlens=cu_seqlens, chunk_size=chunk_size)
