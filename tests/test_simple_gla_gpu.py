"""Parity of the simple-GLA operators (tops.ops.simple_gla, on the GLA kernels of the C ABI)
with the reference's simple-GLA Torch code (golden fixtures) and the numpy oracle.

Tolerances: fp32 max-abs/rel 1e-4 against the reference; bf16 rel-L2 2e-2 against the
fp64 oracle on the same bf16-valued inputs.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as GC
import simple_gla_cases as SC
from _util import assert_close, assert_rel_l2
from oracle import simple_gla_oracle as SO

pytestmark = pytest.mark.gpu

FP32 = dict(atol=1e-4, rtol=1e-4)


@pytest.fixture(scope="module")
def sg():
    import tops.ops.simple_gla as S
    from tops import _C
    _C.lib()
    return S


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


@pytest.mark.parametrize("case", SC.SIMPLE_CASES, ids=lambda c: c["name"])
def test_simple_fwd_matches_reference(sg, case):
    c, inp, fx = SC.load(case["name"])
    o, ht = sg.chunk_simple_gla_fwd(dev(inp["q"]), dev(inp["k"]), dev(inp["v"]), g=dev(inp["g"]),
                                    g_gamma=dev(inp["g_gamma"]), scale=inp["scale"], h0=dev(inp["h0"]), use_ht=True,
                                    cu_seqlens=inp["cu"], chunk_size=inp["C"])
    assert_close("o", o, fx["o"], **FP32)
    assert_close("ht", ht.cpu().double().numpy() * SC.pad_decay(inp), fx["ht"], **FP32)


@pytest.mark.parametrize("case", [c for c in SC.SIMPLE_CASES if c["gate"] == "gamma"], ids=lambda c: c["name"])
def test_simple_bwd_matches_reference(sg, case):
    """The reference's backward entry point (g_gamma only) -> (dq, dk, dv, dh0)."""
    c, inp, fx = SC.load(case["name"])
    dq, dk, dv, dh0 = sg.chunk_simple_gla_bwd(dev(inp["q"]), dev(inp["k"]), dev(inp["v"]), dev(inp["g_gamma"]),
                                              inp["scale"], dev(inp["h0"]), dev(inp["do"]), dev(inp["dht"]),
                                              chunk_size=inp["C"])
    for nm, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert_close(nm, got, fx[nm], **FP32)
    assert (dh0 is None) == (inp["h0"] is None)
    if dh0 is not None:
        assert_close("dh0", dh0, fx["dh0"], **FP32)


@pytest.mark.parametrize("case", [c for c in SC.SIMPLE_CASES if c["gate"] != "gamma"], ids=lambda c: c["name"])
def test_simple_autograd_matches_reference(sg, case):
    """chunk_simple_gla differentiated by torch.autograd: dq, dk, dv, dg [B, T, H], dh0."""
    c, inp, fx = SC.load(case["name"])
    q, k, v, g = (dev(inp[n]).requires_grad_() for n in ("q", "k", "v", "g"))
    h0 = dev(inp["h0"])
    if h0 is not None:
        h0.requires_grad_()
    o, ht = sg.chunk_simple_gla(q, k, v, g=g, g_gamma=dev(inp["g_gamma"]), scale=inp["scale"], initial_state=h0,
                                output_final_state=True, cu_seqlens=inp["cu"], chunk_size=inp["C"])
    assert_close("o", o, fx["o"], **FP32)
    loss = (o * dev(inp["do"])).sum()
    if inp["dht"] is not None:
        loss = loss + (ht * dev(inp["dht"])).sum()
    loss.backward()
    for nm, t in (("dq", q), ("dk", k), ("dv", v), ("dg", g)):
        assert_close(nm, t.grad, fx[nm], **FP32)
    if h0 is not None:
        assert_close("dh0", h0.grad, fx["dh0"], **FP32)


def test_simple_g_gamma_gradient(sg):
    """d g_gamma = the sum over batch, time and K of the GLA gate gradient."""
    c, inp, fx = SC.load("both_h0_dht")
    q, k, v = (dev(inp[n]) for n in "qkv")
    gg = dev(inp["g_gamma"]).requires_grad_()
    o, ht = sg.chunk_simple_gla(q, k, v, g=dev(inp["g"]), g_gamma=gg, scale=inp["scale"],
                                initial_state=dev(inp["h0"]), output_final_state=True, chunk_size=inp["C"])
    ((o * dev(inp["do"])).sum() + (ht * dev(inp["dht"])).sum()).backward()
    # the scalar-gate gradient per step is dg[b, t, h]; g_gamma adds to every step of head h
    assert_close("dg_gamma", gg.grad, fx["dg"].sum(axis=(0, 1)), atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("gate", ["g", "gamma", "both"])
def test_simple_bf16_tensor_core_vs_oracle(sg, gate):
    """bf16, K = V = 128: the tcgen05 path, forward + backward."""
    rng = np.random.default_rng(77)
    B, T, H, K, V = 2, 320, 2, 128, 128
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    do = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H))) / 16).astype(np.float32) if gate != "gamma" else None
    gam = (-np.abs(rng.random(H)) * 0.05).astype(np.float32) if gate != "g" else None
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32)
    scale = K ** -0.5
    o_r, ht_r = SO.chunk_simple_gla_fwd(q, k, v, g, gam, scale, h0, True)
    dq_r, dk_r, dv_r, dg_r, dh0_r = SO.chunk_simple_gla_bwd(q, k, v, g, gam, scale, h0, do, None)
    bf = torch.bfloat16
    qt, kt, vt = (dev(x, bf).requires_grad_() for x in (q, k, v))
    gt = None if g is None else dev(g).requires_grad_()
    h0t = dev(h0).requires_grad_()
    o, ht = sg.chunk_simple_gla(qt, kt, vt, g=gt, g_gamma=dev(gam), scale=scale, initial_state=h0t,
                                output_final_state=True)
    assert o.dtype == bf
    assert_rel_l2("o", o, o_r, 2e-2)
    assert_rel_l2("ht", ht, ht_r, 2e-2)
    (o.float() * dev(do)).sum().backward()
    for nm, got, want in (("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r), ("dv", vt.grad, dv_r),
                          ("dh0", h0t.grad, dh0_r)):
        assert_rel_l2(nm, got, want, 2e-2)
    if g is not None:
        assert_rel_l2("dg", gt.grad, dg_r, 2e-2)


@pytest.mark.parametrize("case", SC.SIMPLE_CASES[:8], ids=lambda c: c["name"])
def test_simple_naive_matches_reference(sg, case):
    """simple_gla_naive (the step loop, 4-D broadcastable gates) gives the chunked result."""
    c, inp, fx = SC.load(case["name"])
    H = inp["q"].shape[2]
    g4 = None if inp["g"] is None else dev(inp["g"][..., None])
    gg4 = None if inp["g_gamma"] is None else dev(inp["g_gamma"].reshape(1, 1, H, 1))
    o, S = sg.simple_gla_naive(dev(inp["q"]), dev(inp["k"]), dev(inp["v"]), g=g4, g_gamma=gg4, scale=inp["scale"],
                               initial_state=dev(inp["h0"]), output_final_state=True)
    assert o.dtype == torch.float32
    assert_close("o", o, fx["o"], **FP32)
    assert_close("S", S.cpu().double().numpy() * SC.pad_decay(inp), fx["ht"], **FP32)
