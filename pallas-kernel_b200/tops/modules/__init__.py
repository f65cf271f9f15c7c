"""Modules of the GLA layer around the chunked op (reference tops/modules)."""
from .fused_norm_gate import FusedRMSNormGated, fused_rms_norm_gated
from .gate import gate_logsigmoid

__all__ = ["FusedRMSNormGated", "fused_rms_norm_gated", "gate_logsigmoid"]
