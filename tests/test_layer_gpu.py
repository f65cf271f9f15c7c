"""GLA layer (BASELINE config 5 building block) on the GPU against fixtures made by the
reference's torch layer (tests/golden/make_layer_golden.py), plus the fused norm-gate and
gate kernels against plain torch fp32."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "tests" / "golden")]
import layer_cases as LC  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    import tops.layers as layers
    from tops import _C
    _C.lib()
    return layers


def rel(a, b):
    a, b = torch.as_tensor(a).detach().double().cpu(), torch.as_tensor(b).detach().double().cpu()
    return float((a - b).norm() / (b.norm() + 1e-30))


def _build(L, case, dtype):
    layer = L.GatedLinearAttention(mode="chunk", **case["args"], layer_idx=0).cuda()
    W = LC.weights([(n, tuple(p.shape)) for n, p in layer.named_parameters()], case["seed"])
    with torch.no_grad():
        for n, p in layer.named_parameters():
            p.copy_(torch.from_numpy(W[n]))
    return layer.to(dtype)


@pytest.mark.parametrize("name", ["layer_chunk", "layer_recurrent", "layer_mask", "layer_mqa"])
def test_layer_fp32_matches_reference_layer(L, name):
    case = LC.LAYER_CASES[name]
    ref = np.load(ROOT / "tests" / "golden" / f"{name}.npz")
    layer = _build(L, case, torch.float32)
    x, do, mask = LC.inputs(case)
    xt = torch.from_numpy(x).cuda().requires_grad_()
    mt = None if mask is None else torch.from_numpy(mask).cuda()
    o, _, _ = layer(xt, attention_mask=mt)
    (o * torch.from_numpy(do).cuda()).sum().backward()
    assert rel(o.detach(), ref["o"]) < 1e-4
    assert rel(xt.grad, ref["dx"]) < 1e-4
    for n, p in layer.named_parameters():
        assert rel(p.grad, ref["grad." + n]) < 1e-4, n


def test_layer_bf16_tensor_core_shape_matches_reference_layer(L):
    """bf16 weights/activations (tensor-core GLA path) vs the fp32 reference layer."""
    from tops.ops.gla import _core
    case = LC.LAYER_CASES["layer_tc"]
    ref = np.load(ROOT / "tests" / "golden" / "layer_tc.npz")
    layer = _build(L, case, torch.bfloat16)
    x, do, _ = LC.inputs(case)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16).requires_grad_()
    q = torch.empty(case["B"], case["T"], 1, 128, device="cuda", dtype=torch.bfloat16)
    assert _core.saved_size(_core.make_plan(q, 256, 16, None, 1.0), q.float()) > 0, "shape should take the TC path"
    o, _, _ = layer(xt)
    (o.float() * torch.from_numpy(do).cuda()).sum().backward()
    assert rel(o.detach().float(), ref["o"]) < 3e-2
    assert rel(xt.grad.float(), ref["dx"]) < 3e-2
    for n, p in layer.named_parameters():
        if "grad." + n in ref:
            assert rel(p.grad.float(), ref["grad." + n]) < 5e-2, n


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("V,affine", [(64, True), (512, True), (256, False), (1024, True)])
def test_fused_norm_gate_matches_torch(L, dtype, V, affine):
    from tops.modules import fused_rms_norm_gated
    if dtype == torch.float32 and V > 512:
        pytest.skip("fp32 rows are limited to 512 columns")
    torch.manual_seed(V)
    x = torch.randn(3, 37, 2, V, device="cuda").to(dtype).requires_grad_()
    g = torch.randn(3, 37, 2, V, device="cuda").to(dtype).requires_grad_()
    w = (1 + 0.1 * torch.randn(V, device="cuda")).to(dtype).requires_grad_() if affine else None
    dy = torch.randn(3, 37, 2, V, device="cuda")
    y = fused_rms_norm_gated(x, g, w, 1e-5)
    (y.float() * dy).sum().backward()
    xr, gr = x.detach().float().requires_grad_(), g.detach().float().requires_grad_()
    wr = None if w is None else w.detach().float().requires_grad_()
    yr = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5)
    if wr is not None:
        yr = yr * wr
    yr = yr * torch.nn.functional.silu(gr)
    (yr * dy).sum().backward()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert rel(y.detach().float(), yr.detach()) < tol
    assert rel(x.grad.float(), xr.grad) < tol
    assert rel(g.grad.float(), gr.grad) < tol
    if w is not None:
        assert rel(w.grad.float(), wr.grad) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("clamp", [None, -0.05])
def test_gate_logsigmoid_matches_torch(L, dtype, clamp):
    from tops.modules import gate_logsigmoid
    torch.manual_seed(2)
    x = (3 * torch.randn(1000, 33, device="cuda")).to(dtype).requires_grad_()
    dy = torch.randn(1000, 33, device="cuda")
    y = gate_logsigmoid(x, 16.0, clamp)
    (y * dy).sum().backward()
    xr = x.detach().float().requires_grad_()
    yr = torch.nn.functional.logsigmoid(xr) / 16
    if clamp is not None:
        yr = torch.clamp_min(yr, clamp)
    (yr * dy).sum().backward()
    assert y.dtype == torch.float32
    assert rel(y.detach(), yr.detach()) < 1e-6
    assert rel(x.grad.float(), xr.grad) < (1e-6 if dtype == torch.float32 else 1e-2)


def test_layer_decode_cache_matches_full_sequence(L):
    """Prefill + token-by-token decode through the cache equals one pass over the sequence."""
    torch.manual_seed(4)
    layer = L.GatedLinearAttention(hidden_size=128, num_heads=2, layer_idx=0).cuda()
    x = torch.randn(2, 90, 128, device="cuda")
    full, _, _ = layer(x)
    cache = L.GLACache()
    parts = [layer(x[:, :70], past_key_values=cache, use_cache=True)[0]]
    for t in range(70, 90):
        parts.append(layer(x[:, t:t + 1], past_key_values=cache, use_cache=True)[0])
    assert rel(torch.cat(parts, 1), full) < 1e-4
