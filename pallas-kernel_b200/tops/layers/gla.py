"""GatedLinearAttention layer (reference tops/layers/gla.py:71-345; torch gold
tests/src/layers/gla.py:53-395).

Same constructor arguments and forward contract as the reference:
``forward(hidden_states, attention_mask=None, past_key_values=None, use_cache=False,
output_attentions=False, **kwargs) -> (o, None, past_key_values)``.  The projections are
plain GEMMs (torch / cuBLAS); the recurrence runs on this library's GLA kernels
(``chunk_gla`` / ``fused_chunk_gla`` / ``fused_recurrent_gla``), the gate activation and
the RMSNorm x swish output gate on its fused kernels (``tops.modules``).
Sequences of at most 64 tokens use ``fused_recurrent`` (reference :224).  A 0/1
``attention_mask`` [B, T] packs the valid tokens into one varlen sequence
(``cu_seqlens``) and scatters the output back, as the torch gold does.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..modules import FusedRMSNormGated, RMSNorm, ShortConvolution, gate_logsigmoid
from ..ops.gla import chunk_gla, fused_chunk_gla, fused_recurrent_gla

__all__ = ["GatedLinearAttention", "ShortConvolution", "RMSNorm", "GLACache"]

ACT2FN = {
    "relu": F.relu,
    "sigmoid": torch.sigmoid,
    "silu": F.silu,
    "swish": F.silu,
    "gelu": F.gelu,
    "tanh": torch.tanh,
}


class GLACache:
    """Per-layer decode state (recurrent_state, conv_state) with the cache protocol the
    layer uses: ``len(cache)``, ``cache[layer_idx]`` and ``cache.update(...)``."""

    def __init__(self):
        self.states: list[dict] = []
        self.seen_tokens = 0

    def __len__(self):
        return len(self.states)

    def __getitem__(self, i):
        return self.states[i]

    def update(self, recurrent_state=None, conv_state=None, layer_idx: int = 0, offset: int = 0):
        while len(self.states) <= layer_idx:
            self.states.append({"recurrent_state": None, "conv_state": None})
        self.states[layer_idx] = {"recurrent_state": recurrent_state, "conv_state": conv_state}
        if layer_idx == 0:
            self.seen_tokens += offset


def _unpad(mask: torch.Tensor):
    """0/1 mask [B, T] -> (indices of valid tokens in B*T, cu_seqlens int32 [B+1])."""
    lens = mask.sum(-1, dtype=torch.int32)
    indices = torch.nonzero(mask.flatten(), as_tuple=False).flatten()
    cu = F.pad(torch.cumsum(lens, 0, dtype=torch.int32), (1, 0))
    return indices, cu


class GatedLinearAttention(nn.Module):
    def __init__(
        self,
        mode: str = "chunk",
        hidden_size: int = 1024,
        expand_k: float = 0.5,
        expand_v: float = 1.0,
        num_heads: int = 4,
        num_kv_heads: int | None = None,
        feature_map: str | None = None,
        use_short_conv: bool = False,
        conv_size: int = 4,
        conv_bias: bool = False,
        use_output_gate: bool = True,
        gate_fn: str = "swish",
        elementwise_affine: bool | None = True,
        norm_eps: float = 1e-5,
        gate_logit_normalizer: int = 16,
        gate_low_rank_dim: int = 16,
        clamp_min: float | None = None,
        fuse_norm: bool = True,
        layer_idx: int | None = None,
    ) -> None:
        super().__init__()
        self.mode = mode
        self.hidden_size = hidden_size
        self.expand_k = expand_k
        self.expand_v = expand_v
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads if num_kv_heads is not None else num_heads
        self.num_kv_groups = self.num_heads // self.num_kv_heads
        self.feature_map_fn = ACT2FN[feature_map] if feature_map is not None else None
        self.use_short_conv = use_short_conv
        self.conv_size = conv_size
        self.conv_bias = conv_bias
        self.use_output_gate = use_output_gate
        self.key_dim = int(hidden_size * expand_k)
        self.value_dim = int(hidden_size * expand_v)
        self.key_dim_per_group = self.key_dim // self.num_kv_groups
        self.value_dim_per_group = self.value_dim // self.num_kv_groups
        self.clamp_min = clamp_min
        self.layer_idx = layer_idx
        assert mode in ["chunk", "fused_recurrent", "fused_chunk"], f"Not supported mode `{mode}`."
        assert self.key_dim % num_heads == 0, f"key dim must be divisible by num_heads of {num_heads}"
        assert self.value_dim % num_heads == 0, f"value dim must be divisible by num_heads of {num_heads}"
        self.head_k_dim = self.key_dim // num_heads
        self.head_v_dim = self.value_dim // num_heads

        self.q_proj = nn.Linear(hidden_size, self.key_dim, bias=False)
        self.k_proj = nn.Linear(hidden_size, self.key_dim_per_group, bias=False)
        self.v_proj = nn.Linear(hidden_size, self.value_dim_per_group, bias=False)
        if self.use_output_gate:
            self.g_proj = nn.Linear(hidden_size, self.value_dim, bias=False)
        if use_short_conv:
            self.q_conv1d = ShortConvolution(self.key_dim, conv_size, conv_bias, "silu")
            self.k_conv1d = ShortConvolution(self.key_dim_per_group, conv_size, conv_bias, "silu")
            self.v_conv1d = ShortConvolution(self.value_dim_per_group, conv_size, conv_bias, "silu")
        self.gk_proj = nn.Sequential(nn.Linear(hidden_size, gate_low_rank_dim, bias=False),
                                     nn.Linear(gate_low_rank_dim, self.key_dim_per_group, bias=True))
        self.o_proj = nn.Linear(self.value_dim, hidden_size, bias=False)
        if gate_fn == "swish" and fuse_norm and use_output_gate:
            self.g_norm_swish_gate = FusedRMSNormGated(self.head_v_dim, elementwise_affine=bool(elementwise_affine),
                                                       eps=norm_eps)
            self.fuse_norm_and_gate = True
        else:
            self.fuse_norm_and_gate = False
            self.g_norm = RMSNorm(self.head_v_dim, elementwise_affine=bool(elementwise_affine), eps=norm_eps)
            self.gate_fn = ACT2FN[gate_fn]
        self.gate_logit_normalizer = gate_logit_normalizer

    def _heads(self, x, d):
        return x.unflatten(-1, (-1, d))

    def _repeat(self, x, d):
        # "... (h d) -> ... (h g) d": every kv head repeated num_kv_groups times
        return self._heads(x, d).repeat_interleave(self.num_kv_groups, dim=-2)

    def forward(self, hidden_states: torch.Tensor, attention_mask: torch.Tensor | None = None,
                past_key_values: Any | None = None, use_cache: bool | None = False,
                output_attentions: bool | None = False, **kwargs):
        if attention_mask is not None:
            assert attention_mask.dim() == 2, (
                "Expected attention_mask as a 0-1 matrix with shape [batch_size, seq_len] (0 = padding).")
        batch_size, q_len, _ = hidden_states.shape
        mode = "fused_recurrent" if q_len <= 64 else self.mode
        last_state = None
        if past_key_values is not None and len(past_key_values) > self.layer_idx:
            last_state = past_key_values[self.layer_idx]
        cu_seqlens = kwargs.get("cu_seqlens")
        indices = None
        if attention_mask is not None:
            indices, cu_seqlens = _unpad(attention_mask[:, -q_len:])
            hidden_states = hidden_states.flatten(0, 1).index_select(0, indices).unsqueeze(0)

        conv_q = conv_k = conv_v = None
        if self.use_short_conv:
            if last_state is not None and last_state.get("conv_state") is not None:
                conv_q, conv_k, conv_v = last_state["conv_state"]
            q, conv_q = self.q_conv1d(self.q_proj(hidden_states), conv_q, use_cache, cu_seqlens)
            k, conv_k = self.k_conv1d(self.k_proj(hidden_states), conv_k, use_cache, cu_seqlens)
            v, conv_v = self.v_conv1d(self.v_proj(hidden_states), conv_v, use_cache, cu_seqlens)
        else:
            q = self.q_proj(hidden_states)
            k = self.k_proj(hidden_states)
            v = self.v_proj(hidden_states)
        gk = self.gk_proj(hidden_states)

        q = self._heads(q, self.head_k_dim)
        if self.num_kv_groups > 1:
            k, gk = self._repeat(k, self.head_k_dim), self._repeat(gk, self.head_k_dim)
            v = self._repeat(v, self.head_v_dim)
        else:
            k, gk = self._heads(k, self.head_k_dim), self._heads(gk, self.head_k_dim)
            v = self._heads(v, self.head_v_dim)
        gk = gate_logsigmoid(gk, self.gate_logit_normalizer, self.clamp_min)  # fp32 [B, T, H, K]
        if self.feature_map_fn is not None:
            q, k = map(self.feature_map_fn, (q, k))

        recurrent_state = last_state["recurrent_state"] if last_state is not None else None
        if mode == "fused_recurrent":
            o, recurrent_state = fused_recurrent_gla(q, k, v, gk=gk, initial_state=recurrent_state,
                                                     output_final_state=use_cache, cu_seqlens=cu_seqlens)
            o = o.to(q.dtype)  # the recurrent op returns fp32 (reference fused_recurrent.py:261-263)
        elif mode == "fused_chunk":
            o, recurrent_state = fused_chunk_gla(q, k, v, g=gk, initial_state=recurrent_state,
                                                 output_final_state=use_cache, cu_seqlens=cu_seqlens)
        else:
            o, recurrent_state = chunk_gla(q, k, v, g=gk, initial_state=recurrent_state,
                                           output_final_state=use_cache, cu_seqlens=cu_seqlens, chunk_size=16)

        if past_key_values is not None:
            past_key_values.update(recurrent_state=recurrent_state,
                                   conv_state=(conv_q, conv_k, conv_v) if self.use_short_conv else None,
                                   layer_idx=self.layer_idx, offset=q_len)

        if self.use_output_gate:
            g = self.g_proj(hidden_states)
            if self.fuse_norm_and_gate:
                o = self.g_norm_swish_gate(o, self._heads(g, self.head_v_dim)).flatten(-2)
            else:
                o = self.g_norm(o).flatten(-2) * self.gate_fn(g)
        else:
            o = self.g_norm(o).flatten(-2)
        o = self.o_proj(o)
        if indices is not None:
            out = o.new_zeros(batch_size * q_len, o.shape[-1])
            o = out.index_copy(0, indices, o.squeeze(0)).view(batch_size, q_len, -1)
        return o, None, past_key_values
