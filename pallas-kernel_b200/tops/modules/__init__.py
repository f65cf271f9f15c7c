"""Modules of the GLA layer around the chunked op (reference tops/modules)."""
from .fused_norm_gate import FusedRMSNormGated, fused_rms_norm_gated
from .convolution import ShortConvolution
from .gate import gate_logsigmoid
from .layernorm import RMSNorm

__all__ = ["FusedRMSNormGated", "fused_rms_norm_gated", "gate_logsigmoid", "RMSNorm", "ShortConvolution"]
