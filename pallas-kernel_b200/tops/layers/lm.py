"""GLA language model for BASELINE config 5 (the reference has the layer only,
tops/layers/gla.py:71; the stack is new): token embedding, ``num_layers`` blocks of
[RMSNorm -> GatedLinearAttention -> residual, RMSNorm -> SwiGLU MLP -> residual], final
RMSNorm, LM head, next-token cross-entropy.  Data-parallel training with bf16 parameters
and fp32 master weights is in ``train_step`` / ``MasterAdamW``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .gla import GatedLinearAttention, RMSNorm

__all__ = ["GLAConfig", "GLABlock", "GLAForCausalLM", "MasterAdamW", "train_step"]


@dataclass
class GLAConfig:
    vocab_size: int = 32000
    hidden_size: int = 2048
    num_layers: int = 24
    num_heads: int = 4
    expand_k: float = 0.5
    expand_v: float = 1.0
    intermediate_size: int = 5632
    gate_low_rank_dim: int = 16
    gate_logit_normalizer: int = 16
    norm_eps: float = 1e-5
    init_std: float = 0.02
    attn_mode: str = "chunk"


class SwiGLU(nn.Module):
    def __init__(self, hidden: int, inter: int):
        super().__init__()
        self.gate_up = nn.Linear(hidden, 2 * inter, bias=False)
        self.down = nn.Linear(inter, hidden, bias=False)

    def forward(self, x):
        a, b = self.gate_up(x).chunk(2, dim=-1)
        return self.down(F.silu(a) * b)


class GLABlock(nn.Module):
    def __init__(self, cfg: GLAConfig, idx: int):
        super().__init__()
        self.attn_norm = RMSNorm(cfg.hidden_size, eps=cfg.norm_eps)
        self.attn = GatedLinearAttention(mode=cfg.attn_mode, hidden_size=cfg.hidden_size, expand_k=cfg.expand_k,
                                         expand_v=cfg.expand_v, num_heads=cfg.num_heads,
                                         gate_low_rank_dim=cfg.gate_low_rank_dim,
                                         gate_logit_normalizer=cfg.gate_logit_normalizer, norm_eps=cfg.norm_eps,
                                         layer_idx=idx)
        self.mlp_norm = RMSNorm(cfg.hidden_size, eps=cfg.norm_eps)
        self.mlp = SwiGLU(cfg.hidden_size, cfg.intermediate_size)

    def forward(self, x, attention_mask=None, past_key_values=None, use_cache=False):
        h, _, past_key_values = self.attn(self.attn_norm(x), attention_mask, past_key_values, use_cache)
        x = x + h
        return x + self.mlp(self.mlp_norm(x)), past_key_values


class GLAForCausalLM(nn.Module):
    def __init__(self, cfg: GLAConfig):
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList([GLABlock(cfg, i) for i in range(cfg.num_layers)])
        self.norm = RMSNorm(cfg.hidden_size, eps=cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, generator: torch.Generator | None = None):
        """N(0, init_std) weights, zero biases, unit norm weights (seeded by ``generator``)."""
        for name, p in self.named_parameters():
            if p.dim() >= 2:
                p.copy_(torch.randn(p.shape, generator=generator, device=p.device, dtype=torch.float32)
                        .mul_(self.cfg.init_std).to(p.dtype))
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.fill_(1.0)

    def forward(self, input_ids, labels=None, attention_mask=None, past_key_values=None, use_cache=False):
        x = self.embed(input_ids)
        for blk in self.layers:
            x, past_key_values = blk(x, attention_mask, past_key_values, use_cache)
        logits = self.lm_head(self.norm(x))
        if labels is None:
            return logits, past_key_values
        loss = F.cross_entropy(logits[:, :-1].flatten(0, 1).float(), labels[:, 1:].flatten())
        return loss, past_key_values


class MasterAdamW:
    """AdamW on fp32 master copies of (bf16) model parameters: gradients are upcast into
    the master copies, the fused AdamW step runs in fp32, results are cast back."""

    def __init__(self, params, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1):
        self.params = [p for p in params if p.requires_grad]
        self.master = [p.detach().float().clone().requires_grad_(True) for p in self.params]
        self.opt = torch.optim.AdamW(self.master, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                     fused=self.master[0].is_cuda if self.master else False)

    @torch.no_grad()
    def step(self):
        for p, m in zip(self.params, self.master):
            m.grad = None if p.grad is None else p.grad.float()
        self.opt.step()
        for p, m in zip(self.params, self.master):
            p.copy_(m)

    def zero_grad(self):
        for p in self.params:
            p.grad = None


def train_step(model, opt: MasterAdamW, input_ids: torch.Tensor) -> torch.Tensor:
    """One data-parallel training step (``model`` may be wrapped in DistributedDataParallel,
    which all-reduces the gradients over NCCL during the backward).  Returns the loss."""
    opt.zero_grad()
    loss, _ = model(input_ids, labels=input_ids)
    loss.backward()
    opt.step()
    return loss.detach()
