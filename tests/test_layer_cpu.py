"""Host-side pieces of the GLA layer that need no GPU: padding-mask packing, the decode
cache protocol, the short convolution, and the refusal of CPU tensors by the fused ops
(the kernels are the only implementation)."""
from __future__ import annotations

import pytest
import torch


def test_unpad_packs_valid_tokens_and_cu_seqlens():
    from tops.layers.gla import _unpad
    mask = torch.tensor([[1, 1, 1, 0], [1, 0, 0, 0], [1, 1, 1, 1]])
    idx, cu = _unpad(mask)
    assert idx.tolist() == [0, 1, 2, 4, 8, 9, 10, 11]
    assert cu.tolist() == [0, 3, 4, 8] and cu.dtype == torch.int32


def test_cache_protocol():
    from tops.layers import GLACache
    c = GLACache()
    assert len(c) == 0
    c.update(recurrent_state="s0", conv_state=None, layer_idx=0, offset=5)
    c.update(recurrent_state="s1", conv_state=("a", "b", "c"), layer_idx=1, offset=5)
    assert len(c) == 2 and c[0]["recurrent_state"] == "s0" and c[1]["conv_state"] == ("a", "b", "c")
    assert c.seen_tokens == 5


def test_short_convolution_is_causal_and_caches():
    from tops.layers import ShortConvolution
    torch.manual_seed(0)
    conv = ShortConvolution(8, kernel_size=4)
    x = torch.randn(2, 10, 8)
    y, _ = conv(x)
    x2 = x.clone()
    x2[:, 6:] += 1.0  # the future does not change the past
    y2, _ = conv(x2)
    assert torch.allclose(y[:, :6], y2[:, :6])
    # prefill + one step through the cache equals the full sequence
    y_pre, cache = conv(x[:, :9], output_final_state=True)
    y_last, _ = conv(x[:, 9:], cache=cache)
    assert torch.allclose(torch.cat([y_pre, y_last], 1), y, atol=1e-6)


def test_fused_ops_refuse_cpu_tensors():
    from tops.modules import fused_rms_norm_gated, gate_logsigmoid
    with pytest.raises(RuntimeError, match="CUDA"):
        gate_logsigmoid(torch.randn(4, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_rms_norm_gated(torch.randn(4, 8), torch.randn(4, 8))


def test_model_config_5_parameter_count():
    """The config-5 stack (24 layers, hidden 2048, MLP 5632, vocab 32000) has 1.37 B parameters."""
    from tops.layers import GLAConfig, GLAForCausalLM
    cfg = GLAConfig()
    with torch.device("meta"):
        m = GLAForCausalLM.__new__(GLAForCausalLM)
        torch.nn.Module.__init__(m)
        m.cfg = cfg
        m.embed = torch.nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        from tops.layers.lm import GLABlock
        m.layers = torch.nn.ModuleList([GLABlock(cfg, i) for i in range(cfg.num_layers)])
        m.lm_head = torch.nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
    n = sum(p.numel() for p in m.parameters())
    assert 1.3e9 < n < 1.4e9, n
