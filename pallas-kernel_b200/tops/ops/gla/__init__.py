"""B200-native GLA operators with the export list of the reference's ``tops.ops.gla``
(primatrix/pallas-kernel ``tops/ops/gla/__init__.py:1-34``)."""
from .naive import naive_recurrent_gla
from .chunk import (
    chunk_gla,
    chunk_local_cumsum_vector as chunk_local_cumsum,
    chunk_fwd_h_ref as chunk_fwd_h,
    chunk_gla_fwd_intra_gk,
    chunk_gla_fwd_o_gk,
    chunk_gla_fwd,
    chunk_gla_bwd_dA_ref,
    chunk_gla_bwd_dv_ref,
    chunk_gla_bwd_dqk_intra_ref,
    chunk_gla_bwd_dqkg_ref,
    chunk_gla_bwd,
)
from .fused_chunk import fused_chunk_gla
from .fused_recurrent import fused_recurrent_gla, fused_recurrent_gla_bwd
from .host import PinnedGLAPipeline, chunk_gla_fwd_bwd_pinned

__all__ = [
    "chunk_gla_fwd_bwd_pinned",
    "PinnedGLAPipeline",
    "naive_recurrent_gla",
    "chunk_gla",
    "chunk_local_cumsum",
    "chunk_fwd_h",
    "chunk_gla_fwd_intra_gk",
    "chunk_gla_fwd_o_gk",
    "chunk_gla_fwd",
    "chunk_gla_bwd_dA_ref",
    "chunk_gla_bwd_dv_ref",
    "chunk_gla_bwd_dqk_intra_ref",
    "chunk_gla_bwd_dqkg_ref",
    "chunk_gla_bwd",
    "fused_chunk_gla",
    "fused_recurrent_gla",
    "fused_recurrent_gla_bwd",
]
