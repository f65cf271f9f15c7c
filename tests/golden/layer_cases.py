"""Cases of the GLA layer fixtures (``layer_*.npz``): constructor arguments, input shape,
and the seeded generators of weights, inputs and the output cotangent.  Shared by
``make_layer_golden.py`` (reference side) and the GPU tests (our layer)."""
from __future__ import annotations

import numpy as np

LAYER_CASES = {
    # fp32, chunk mode (T > 64), 2 heads of K=32 / V=64
    "layer_chunk": dict(args=dict(hidden_size=128, num_heads=2), B=2, T=100, seed=71),
    # fp32, T <= 64: the layer switches to fused_recurrent
    "layer_recurrent": dict(args=dict(hidden_size=128, num_heads=2), B=2, T=40, seed=72),
    # fp32, padding mask -> packed varlen sequence
    "layer_mask": dict(args=dict(hidden_size=128, num_heads=2), B=3, T=90, seed=73, mask=[90, 71, 30]),
    # fp32, grouped kv heads (MQA): 4 heads share 2 kv heads
    "layer_mqa": dict(args=dict(hidden_size=128, num_heads=4, num_kv_heads=2), B=2, T=80, seed=74),
    # shape of the tensor-core path (K=128, V=256); run in bf16 on our side
    "layer_tc": dict(args=dict(hidden_size=256, num_heads=1), B=2, T=200, seed=75, small_grads=True),
}


def weights(names_shapes, seed):
    """name -> float32 array: N(0, 0.05) matrices, N(0, 0.1) + 1 norm weights, N(0, 0.1) biases."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in names_shapes:
        if name.endswith("norm_swish_gate.weight") or name.endswith("g_norm.weight"):
            out[name] = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        elif name.endswith("bias"):
            out[name] = (0.1 * rng.standard_normal(shape)).astype(np.float32)
        else:
            out[name] = (0.05 * rng.standard_normal(shape)).astype(np.float32)
    return out


def inputs(case):
    rng = np.random.default_rng(case["seed"] + 1000)
    D = case["args"]["hidden_size"]
    x = rng.standard_normal((case["B"], case["T"], D)).astype(np.float32)
    do = rng.standard_normal((case["B"], case["T"], D)).astype(np.float32)
    mask = None
    if case.get("mask"):
        mask = np.zeros((case["B"], case["T"]), dtype=np.int64)
        for b, n in enumerate(case["mask"]):
            mask[b, :n] = 1
    return x, do, mask
