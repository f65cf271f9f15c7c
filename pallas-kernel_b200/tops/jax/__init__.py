"""JAX frontend of the B200 GLA ops (requires jax; import fails cleanly without it).

Same signatures as the reference's ``tops.ops.gla`` (JAX arrays in and out):
``chunk_gla`` / ``fused_chunk_gla`` (differentiable through ``jax.custom_vjp``) and
``fused_recurrent_gla``.  The kernels are reached through XLA custom calls
(``tops_gla_xla_*`` in libtops_gla.so, status-returning legacy API).
"""
from .gla import chunk_gla, fused_chunk_gla, fused_recurrent_gla  # noqa: F401
