"""GLA layer (reference tops/layers) and the config-5 language model around it."""
from .gla import GatedLinearAttention, GLACache, RMSNorm, ShortConvolution
from .lm import GLABlock, GLAConfig, GLAForCausalLM, MasterAdamW, train_step

__all__ = ["GatedLinearAttention", "GLACache", "RMSNorm", "ShortConvolution", "GLABlock", "GLAConfig",
           "GLAForCausalLM", "MasterAdamW", "train_step"]
