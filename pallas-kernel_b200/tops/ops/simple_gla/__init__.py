"""B200-native simple-GLA operators with the export list of the reference's
``tops.ops.simple_gla`` (tops/ops/simple_gla/__init__.py:1-3), plus the differentiable
``chunk_simple_gla``."""
from .chunk import chunk_simple_gla, chunk_simple_gla_bwd, chunk_simple_gla_fwd
from .naive import simple_gla_naive

__all__ = ["chunk_simple_gla", "chunk_simple_gla_bwd", "chunk_simple_gla_fwd", "simple_gla_naive"]
