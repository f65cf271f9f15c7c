"""Parity of the CUDA GLA ops (called through the C ABI via tops.ops.gla) with the
reference's outputs (golden fixtures) and the numpy oracle.

Tolerances (from the task's north star):
  * fp32 inputs: max-abs/rel 1e-4 against the reference (|err| <= 1e-4 + 1e-4 |ref|);
  * bf16 inputs: relative L2 <= 2e-2 against an fp32/fp64 reference of the same inputs.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import cases as GC
from _util import assert_close, assert_rel_l2
from oracle import gla_oracle as O

pytestmark = pytest.mark.gpu

FP32 = dict(atol=1e-4, rtol=1e-4)
BF16_L2 = 2e-2


@pytest.fixture(scope="module")
def gla():
    import tops.ops.gla as G
    from tops import _C
    _C.lib()
    return G


def dev(x, dtype=torch.float32):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


# ---------------------------------------------------------------------------
# chunk_gla forward/backward against the reference's fixtures (fp32)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", GC.CHUNK_CASES, ids=lambda c: c["name"])
def test_chunk_fwd_bwd_matches_reference(gla, case):
    c, inp, fx = GC.load("chunk", case["name"])
    q, k, v, g = (dev(inp[n]) for n in "qkvg")
    h0 = dev(inp["h0"])
    gc, A, h, ht, o = gla.chunk_gla_fwd(q, k, v, g, None, None, inp["scale"], h0, True, cu_seqlens=inp["cu"],
                                        chunk_size=inp["C"])
    assert_close("o", o, fx["o"], **FP32)
    assert_close("ht", ht, fx["ht"], **FP32)
    if "h" in fx:
        assert_close("g_cumsum", gc, fx["g_cumsum"], **FP32)
        assert_close("A", A, fx["A"], **FP32)
        assert_close("h", h, fx["h"], **FP32)
    if "dq" not in fx:
        return
    dq, dk, dv, dg, dh0 = gla.chunk_gla_bwd(q, k, v, g, None, None, inp["scale"], h0, None, None, dev(inp["do"]),
                                            dev(inp["dht"]), cu_seqlens=inp["cu"], chunk_size=inp["C"])
    for nm, got in (("dq", dq), ("dk", dk), ("dv", dv), ("dg", dg)):
        assert_close(nm, got, fx[nm], **FP32)
    assert (dh0 is None) == ("dh0" not in fx)
    if dh0 is not None:
        assert_close("dh0", dh0, fx["dh0"], **FP32)


@pytest.mark.parametrize("case", [c for c in GC.CHUNK_CASES if not c.get("fwd_only")][:12],
                         ids=lambda c: c["name"])
def test_chunk_gla_autograd_matches_reference(gla, case):
    """The public op, differentiated by torch.autograd, gives the reference's gradients."""
    c, inp, fx = GC.load("chunk", case["name"])
    q, k, v, g = (dev(inp[n]).requires_grad_() for n in "qkvg")
    h0 = dev(inp["h0"])
    if h0 is not None:
        h0.requires_grad_()
    o, ht = gla.chunk_gla(q, k, v, g, scale=inp["scale"], initial_state=h0, output_final_state=True,
                          cu_seqlens=inp["cu"], chunk_size=inp["C"])
    assert_close("o", o, fx["o"], **FP32)
    loss = (o * dev(inp["do"])).sum()
    if inp["dht"] is not None:
        loss = loss + (ht * dev(inp["dht"])).sum()
    loss.backward()
    for nm, t in (("dq", q), ("dk", k), ("dv", v), ("dg", g)):
        assert_close(nm, t.grad, fx[nm], **FP32)
    if h0 is not None and "dh0" in fx:
        assert_close("dh0", h0.grad, fx["dh0"], **FP32)


def test_cfg1_forward(gla):
    """B2 T256 H4 K64 V64 C64 fp32, g = logsigmoid/16, h0 = 0, final state."""
    c, inp, fx = GC.load("chunk", "cfg1")
    o, ht = gla.chunk_gla(dev(inp["q"]), dev(inp["k"]), dev(inp["v"]), dev(inp["g"]), scale=inp["scale"],
                          initial_state=dev(inp["h0"]), output_final_state=True, chunk_size=64)
    assert_close("o", o, fx["o"], **FP32)
    assert_close("ht", ht, fx["ht"], **FP32)


# ---------------------------------------------------------------------------
# bf16 inputs: rel-L2 2e-2 against the fp64 oracle on the same (bf16-valued) inputs
# ---------------------------------------------------------------------------

BF16_CASES = [
    dict(B=2, T=256, H=4, K=64, V=64, C=64, seed=1),
    dict(B=1, T=300, H=2, K=128, V=256, C=64, seed=2, h0=True, dht=True),
    dict(B=1, T=200, H=2, K=256, V=128, C=64, seed=3, cu=[0, 50, 130, 200]),
    dict(B=2, T=128, H=2, K=32, V=48, C=16, seed=4),
]


@pytest.mark.parametrize("case", BF16_CASES, ids=lambda c: f"B{c['B']}T{c['T']}K{c['K']}V{c['V']}C{c['C']}")
def test_chunk_bf16_fwd_bwd_vs_oracle(gla, case):
    rng = np.random.default_rng(case["seed"])
    B, T, H, K, V = case["B"], case["T"], case["H"], case["K"], case["V"]
    N = len(case["cu"]) - 1 if case.get("cu") else B
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
    do = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    h0 = rng.standard_normal((N, H, K, V), dtype=np.float32) if case.get("h0") else None
    dht = rng.standard_normal((N, H, K, V), dtype=np.float32) if case.get("dht") else None
    scale = K ** -0.5
    o_r, ht_r = O.chunk_gla(q, k, v, g, scale=scale, initial_state=h0, output_final_state=True,
                            cu_seqlens=case.get("cu"), chunk_size=case["C"])
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(q, k, v, g, None, scale, h0, None, None, do, dht,
                                                    case.get("cu"), case["C"])
    bf = torch.bfloat16
    qt, kt, vt = (dev(x, bf).requires_grad_() for x in (q, k, v))
    gt = dev(g).requires_grad_()
    h0t = dev(h0)
    o, ht = gla.chunk_gla(qt, kt, vt, gt, scale=scale, initial_state=h0t, output_final_state=True,
                          cu_seqlens=case.get("cu"), chunk_size=case["C"])
    assert o.dtype == bf and ht.dtype == torch.float32
    assert_rel_l2("o", o, o_r, BF16_L2)
    assert_rel_l2("ht", ht, ht_r, BF16_L2)
    loss = (o.float() * dev(do)).sum() + (0 if dht is None else (ht * dev(dht)).sum())
    loss.backward()
    for nm, got, want in (("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r), ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r)):
        assert_rel_l2(nm, got, want, BF16_L2)


# ---------------------------------------------------------------------------
# sub-functions
# ---------------------------------------------------------------------------

def test_subfunctions_match_oracle(gla):
    rng = np.random.default_rng(11)
    B, T, H, K, V, C = 2, 100, 3, 40, 72, 32
    q, k = rng.standard_normal((2, B, T, H, K), dtype=np.float32)
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    g = GC.logsigmoid(rng.standard_normal((B, T, H, K))).astype(np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32)
    scale = 0.3
    gc_r = O.chunk_local_cumsum(g, C)
    gc = gla.chunk_local_cumsum(dev(g), C)
    assert_close("cumsum", gc, gc_r, **FP32)
    rev = gla.chunk_local_cumsum(dev(g), C, reverse=True, scale=2.0)
    rev_r = np.zeros_like(g, dtype=np.float64)
    for s in range(0, T, C):
        e = min(s + C, T)
        rev_r[:, s:e] = 2.0 * np.cumsum(g[:, s:e][:, ::-1], axis=1)[:, ::-1]
    assert_close("cumsum_rev", rev, rev_r, **FP32)
    h_r, ht_r = O.chunk_fwd_h(k, v, gc_r, h0, True, None, C)
    h, ht = gla.chunk_fwd_h(dev(k), dev(v), dev(gc_r), dev(h0), True, chunk_size=C)
    assert_close("h", h, h_r, **FP32)
    assert_close("ht", ht, ht_r, **FP32)
    A_full = gla.chunk_gla_fwd_intra_gk(dev(q), dev(k), dev(gc_r), scale, C)
    A_r = O.chunk_gla_fwd_intra_gk(q, k, gc_r, scale, None, C)  # causal
    tril = np.zeros_like(A_r)
    for s in range(0, T, C):
        L = min(C, T - s)
        tril[:, s:s + L, :, :L] = np.tril(np.ones((L, L)))[:, None, :]
    assert_close("A(lower)", A_full.cpu().numpy() * tril, A_r, **FP32)
    o = gla.chunk_gla_fwd_o_gk(dev(q), dev(v), dev(gc_r), dev(A_r), dev(h_r), scale, chunk_size=C)
    assert_close("o", o, O.chunk_gla_fwd_o_gk(q, v, gc_r, A_r, h_r, scale, None, C), **FP32)
    dh_r, dh0_r = O.chunk_bwd_dh(q, k, v, gc_r, do, h0, None, scale, None, C)
    from tops.ops.common.chunk_h import chunk_bwd_dh_ref
    dh, dh0 = chunk_bwd_dh_ref(dev(q), dev(k), dev(v), dev(gc_r), dev(do), h0=dev(h0), scale=scale, chunk_size=C)
    assert_close("dh", dh, dh_r, **FP32)
    assert_close("dh0", dh0, dh0_r, **FP32)
    dA_r = O.chunk_gla_bwd_dA(v, do, scale, None, C)
    assert_close("dA", gla.chunk_gla_bwd_dA_ref(dev(v), dev(do), scale, chunk_size=C), dA_r, **FP32)
    dv_r = O.chunk_gla_bwd_dv(k, gc_r, A_r, do, dh_r, None, C)
    assert_close("dv", gla.chunk_gla_bwd_dv_ref(dev(k), dev(gc_r), dev(A_r), dev(do), dev(dh_r), chunk_size=C),
                 dv_r, **FP32)
    dqi_r, dki_r = O.chunk_gla_bwd_dqk_intra(q, k, gc_r, dA_r, None, C)
    dqi, dki = gla.chunk_gla_bwd_dqk_intra_ref(dev(q), dev(k), dev(gc_r), dev(dA_r), chunk_size=C)
    assert_close("dq_intra", dqi, dqi_r, **FP32)
    assert_close("dk_intra", dki, dki_r, **FP32)
    r = O.chunk_gla_bwd_dqkg(q, k, v, h_r, gc_r, do, dh_r, dqi_r, dki_r, scale, None, C)
    got = gla.chunk_gla_bwd_dqkg_ref(dev(q), dev(k), dev(v), dev(h_r), dev(gc_r), dev(do), dev(dh_r), dev(dqi_r),
                                     dev(dki_r), scale, chunk_size=C)
    for nm, a, b in zip(("dq", "dk", "dg"), got, r):
        assert_close(nm, a, b, **FP32)


def test_common_chunk_h_entry_points(gla):
    """tops.ops.common.chunk_h: chunk_fwd_h_ref / chunk_fwd_h_kernel / chunk_bwd_dh_kernel against
    the oracle's state scans; with split_size = 2 chunks the kernel forms keep the state of the
    first chunk of every split (as the reference stores it when i_t % (split / chunk) == 0)."""
    from tops.ops.common import chunk_h as CH
    rng = np.random.default_rng(71)
    B, T, H, K, V, C = 2, 64, 2, 16, 24, 16
    q, k = (rng.standard_normal((B, T, H, K), dtype=np.float32) for _ in range(2))
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 4).astype(np.float32)
    gc = O.chunk_local_cumsum(g, C).astype(np.float32)
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    dht = rng.standard_normal((B, H, K, V), dtype=np.float32)
    scale = K ** -0.5
    h_r, ht_r = O.chunk_fwd_h(k, v, gc, h0, True, None, C)  # [B, NT, H, K, V]
    h, ht = CH.chunk_fwd_h_ref(dev(k), dev(v), gk=dev(gc), h0=dev(h0), output_final_state=True,
                               states_in_fp32=True, chunk_size=C)
    assert_close("h (ref form)", h, h_r, **FP32)
    assert_close("ht (ref form)", ht, ht_r, **FP32)
    hs, ht2 = CH.chunk_fwd_h_kernel(dev(k), dev(v), gk=dev(gc), h0=dev(h0), output_final_state=True, chunk_size=C,
                                    split_size=2 * C, states_in_fp32=True)
    assert_close("h (kernel form, split 2)", hs, h_r.reshape(-1, H, K, V)[::2], **FP32)
    assert_close("ht (kernel form)", ht2, ht_r, **FP32)
    dh_r, dh0_r = O.chunk_bwd_dh(q, k, v, gc, do, None, dht, scale, None, C)
    dhs, dh0 = CH.chunk_bwd_dh_kernel(dev(q), dev(k), dev(v), gk=dev(gc), do=dev(do), dht=dev(dht), scale=scale,
                                      output_dh0=True, chunk_size=C, split_size=2 * C, states_in_fp32=True)
    assert_close("dh (kernel form, split 2)", dhs, dh_r.reshape(-1, H, K, V)[::2], **FP32)
    assert_close("dh0 (kernel form)", dh0, dh0_r, **FP32)


# ---------------------------------------------------------------------------
# structural behaviour (reference test_pallas_chunk_gla.py:223-273)
# ---------------------------------------------------------------------------

def test_state_split(gla):
    rng = np.random.default_rng(77)
    B, T, H, K, V = 1, 40, 2, 16, 32
    q, k = (dev(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = dev(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = dev(GC.logsigmoid(rng.standard_normal((B, T, H, K))).astype(np.float32))
    o, s = gla.chunk_gla(q, k, v, g, output_final_state=True)
    o1, s1 = gla.chunk_gla(q[:, :20], k[:, :20], v[:, :20], g[:, :20], output_final_state=True)
    o2, s2 = gla.chunk_gla(q[:, 20:], k[:, 20:], v[:, 20:], g[:, 20:], initial_state=s1, output_final_state=True)
    assert_close("o split", torch.cat([o1, o2], 1), o, atol=1e-4, rtol=1e-4)
    assert_close("state split", s2, s, atol=1e-4, rtol=1e-4)


def test_no_final_state_returns_none(gla):
    x = torch.randn(2, 32, 4, 32, device="cuda")
    o, s = gla.chunk_gla(x, x, torch.randn(2, 32, 4, 64, device="cuda"), torch.zeros_like(x))
    assert s is None and o.shape == (2, 32, 4, 64)
    o, s = gla.fused_recurrent_gla(x, x, torch.randn(2, 32, 4, 64, device="cuda"))
    assert s is None and o.dtype == torch.float32


def test_fused_chunk_and_naive_agree(gla):
    rng = np.random.default_rng(9)
    B, T, H, K, V = 2, 70, 2, 32, 32
    q, k = (dev(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = dev(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = dev(GC.logsigmoid(rng.standard_normal((B, T, H, K))).astype(np.float32))
    o1, s1 = gla.fused_chunk_gla(q, k, v, g, output_final_state=True)
    o2, s2 = gla.naive_recurrent_gla(q, k, v, g, output_final_state=True)
    o3, s3 = gla.chunk_gla(q, k, v, g, output_final_state=True, chunk_size=64)
    assert_close("fused_chunk vs naive", o1, o2, atol=1e-4, rtol=1e-4)
    assert_close("chunk64 vs naive", o3, o2, atol=1e-4, rtol=1e-4)
    assert_close("states", s1, s2, atol=1e-4, rtol=1e-4)


def test_ungated_chunk_gla(gla):
    """Neither g nor g_gamma (the reference's defaults: plain linear attention with state):
    fwd + bwd match the oracle run with g=None (fp32 1e-4) and an explicit all-zero gate."""
    rng = np.random.default_rng(13)
    B, T, H, K, V = 2, 45, 2, 32, 24
    q, k = (rng.standard_normal((B, T, H, K), dtype=np.float32) for _ in range(2))
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    qt, kt, vt, h0t = (dev(x).requires_grad_() for x in (q, k, v, h0))
    o, ht = gla.chunk_gla(qt, kt, vt, initial_state=h0t, output_final_state=True)
    (o * dev(do)).sum().backward()
    o_r, ht_r = O.chunk_gla(q, k, v, None, initial_state=h0, output_final_state=True, chunk_size=16)
    dq_r, dk_r, dv_r, _, dh0_r = O.chunk_gla_bwd(q, k, v, None, None, K ** -0.5, h0, None, None, do, None, None, 16)
    for nm, got, want in (("o", o, o_r), ("ht", ht, ht_r), ("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r),
                          ("dv", vt.grad, dv_r), ("dh0", h0t.grad, dh0_r)):
        assert_close(nm, got, want, **FP32)
    o0, ht0 = gla.chunk_gla(dev(q), dev(k), dev(v), torch.zeros(B, T, H, K, device="cuda"), initial_state=dev(h0),
                            output_final_state=True)
    assert_close("o vs g = 0", o.detach(), o0, **FP32)
    assert_close("ht vs g = 0", ht.detach(), ht0, **FP32)


def test_g_gamma_matches_broadcast_g(gla):
    rng = np.random.default_rng(12)
    B, T, H, K, V = 2, 48, 4, 32, 32
    q, k = (dev(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = dev(rng.standard_normal((B, T, H, V), dtype=np.float32))
    gamma = dev(-np.abs(rng.standard_normal((H, 1)).astype(np.float32)) * 0.1)
    o1, _ = gla.chunk_gla(q, k, v, g_gamma=gamma)
    o2, _ = gla.chunk_gla(q, k, v, g=gamma.expand(B, T, H, K).contiguous())
    assert_close("g_gamma", o1, o2, atol=1e-5, rtol=1e-5)


def test_errors_are_raised_not_faulted(gla):
    x = torch.randn(2, 32, 4, 32, device="cuda")
    with pytest.raises(AssertionError):
        gla.chunk_gla(x, x[:, :16], x, x)
    with pytest.raises(AssertionError):
        gla.chunk_gla(x, x, x, x, chunk_size=12)
    with pytest.raises(ValueError):
        gla.chunk_gla(x.cpu(), x.cpu(), x.cpu(), x.cpu())


# ---------------------------------------------------------------------------
# fused_recurrent (decode path)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", GC.REC_CASES, ids=lambda c: c["name"])
def test_recurrent_matches_reference(gla, case):
    c, inp, fx = GC.load("rec", case["name"])
    dt = torch.bfloat16 if case.get("bf16") else torch.float32
    q, k, v = (dev(inp[n], dt) for n in "qkv")
    o, ht = gla.fused_recurrent_gla(q, k, v, gk=dev(inp["gk"]), gv=dev(inp["gv"]), scale=inp["scale"],
                                    initial_state=dev(inp["h0"]), output_final_state=True, reverse=inp["reverse"],
                                    cu_seqlens=inp["cu"])
    assert o.dtype == torch.float32 and ht.dtype == torch.float32
    assert_close("o", o, fx["o"], **FP32)
    assert_close("ht", ht, fx["ht"], **FP32)
    dq, dk, dv, dgk, dgv, dh0 = gla.fused_recurrent_gla_bwd(
        q, k, v, gk=dev(inp["gk"]), gv=dev(inp["gv"]), o=o, do=dev(inp["do"], dt), dht=dev(inp["dht"]),
        scale=inp["scale"], initial_state=dev(inp["h0"]), reverse=inp["reverse"], cu_seqlens=inp["cu"])
    for nm, got in (("dq", dq), ("dk", dk), ("dv", dv), ("dgk", dgk), ("dgv", dgv), ("dh0", dh0)):
        if nm in fx:
            assert_close(nm, got, fx[nm], atol=2e-4, rtol=2e-4)
        else:
            assert got is None, nm
    if "naive_o" in fx:
        on, hn = gla.naive_recurrent_gla(q, k, v, dev(inp["gk"]), scale=inp["scale"], initial_state=dev(inp["h0"]),
                                         output_final_state=True, cu_seqlens=inp["cu"])
        tol = FP32 if dt == torch.float32 else dict(atol=1e-2, rtol=1e-2)  # naive returns o in q's dtype
        assert_close("naive_o", on.float(), fx["naive_o"], **tol)


def test_decode_config2_shape_vs_oracle(gla):
    """BASELINE config 2 at full size: B256 T1 H16 K128 V128, bf16 q/k/v, fp32 gk/h0."""
    torch.manual_seed(0)
    B, H, K, V = 256, 16, 128, 128
    q, k, v = (torch.randn(B, 1, H, D, device="cuda").bfloat16() for D in (K, K, V))
    gk = torch.nn.functional.logsigmoid(torch.randn(B, 1, H, K, device="cuda")) / 16
    h0 = torch.randn(B, H, K, V, device="cuda") * 0.1
    o, ht = gla.fused_recurrent_gla(q, k, v, gk=gk, initial_state=h0, output_final_state=True)
    # exact fp64 recurrence for one step: h = h0 * e^gk + k v^T ; o = scale q^T h
    qd, kd, vd = (x.double() for x in (q, k, v))
    hd = h0.double() * gk.double().exp()[:, 0, :, :, None] + kd[:, 0, :, :, None] * vd[:, 0, :, None, :]
    od = torch.einsum("bhk,bhkv->bhv", qd[:, 0] * K ** -0.5, hd)[:, None]
    assert_close("ht", ht, hd, atol=1e-5, rtol=1e-5)
    assert_close("o", o, od, atol=1e-4, rtol=1e-4)


def test_recurrent_autograd(gla):
    rng = np.random.default_rng(21)
    B, T, H, K, V = 2, 9, 2, 16, 24
    q, k = (dev(rng.standard_normal((B, T, H, K), dtype=np.float32)).requires_grad_() for _ in range(2))
    v = dev(rng.standard_normal((B, T, H, V), dtype=np.float32)).requires_grad_()
    gk = dev(GC.logsigmoid(rng.standard_normal((B, T, H, K))).astype(np.float32)).requires_grad_()
    h0 = dev(rng.standard_normal((B, H, K, V), dtype=np.float32)).requires_grad_()
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    dht = rng.standard_normal((B, H, K, V), dtype=np.float32)
    o, ht = gla.fused_recurrent_gla(q, k, v, gk=gk, initial_state=h0, output_final_state=True)
    ((o * dev(do)).sum() + (ht * dev(dht)).sum()).backward()
    ref = O.fused_recurrent_gla_bwd(*(x.detach().cpu().numpy() for x in (q, k, v, gk)), None, do, dht, None,
                                    h0.detach().cpu().numpy())
    for nm, t, r in (("dq", q, ref[0]), ("dk", k, ref[1]), ("dv", v, ref[2]), ("dgk", gk, ref[3]),
                     ("dh0", h0, ref[5])):
        assert_close(nm, t.grad, r, atol=2e-4, rtol=2e-4)


def test_recurrent_bf16_inputs_multi_step(gla):
    """bf16 q, k, v over T > 1: o and ht come back in fp32 whatever the input dtype (as in the
    reference, fused_recurrent.py:261-263) and match the oracle on the same bf16 values (fp32
    1e-4); dq, dk, dv come back in bf16 (rel-L2 2e-2), dgk and dh0 in fp32."""
    rng = np.random.default_rng(27)
    B, T, H, K, V = 2, 37, 2, 64, 64
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    gk = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 4).astype(np.float32)
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    dht = rng.standard_normal((B, H, K, V), dtype=np.float32)
    bf = torch.bfloat16
    qt, kt, vt = (dev(x, bf).requires_grad_() for x in (q, k, v))
    gkt, h0t = dev(gk).requires_grad_(), dev(h0).requires_grad_()
    o, ht = gla.fused_recurrent_gla(qt, kt, vt, gk=gkt, initial_state=h0t, output_final_state=True)
    assert o.dtype == torch.float32 and ht.dtype == torch.float32
    o_r, ht_r = O.fused_recurrent_gla(q, k, v, gk, None, None, h0, True)
    assert_close("o", o, o_r, **FP32)
    assert_close("ht", ht, ht_r, **FP32)
    ((o * dev(do)).sum() + (ht * dev(dht)).sum()).backward()
    ref = O.fused_recurrent_gla_bwd(q, k, v, gk, None, do, dht, None, h0)
    assert qt.grad.dtype == bf and gkt.grad.dtype == torch.float32
    for nm, t, r in (("dq", qt, ref[0]), ("dk", kt, ref[1]), ("dv", vt, ref[2])):
        assert_rel_l2(nm, t.grad, r, BF16_L2)
    assert_close("dgk", gkt.grad, ref[3], atol=2e-4, rtol=2e-4)
    assert_close("dh0", h0t.grad, ref[5], atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("op", ["chunk", "recurrent"])
def test_fp16_inputs_fwd_bwd(gla, op):
    """fp16 q, k, v (CUDA-core path for chunk_gla; the recurrence for fused_recurrent_gla):
    chunk_gla returns o in fp16, fused_recurrent_gla in fp32, as in the reference; outputs and
    gradients match the fp64 oracle on the same fp16 values within relative L2 2e-3."""
    rng = np.random.default_rng(33 if op == "chunk" else 34)
    B, T, H, K, V = 2, 70, 2, 32, 48
    f16 = lambda x: x.astype(np.float16).astype(np.float32)
    q, k = (f16(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = f16(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 8).astype(np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    h16 = torch.float16
    qt, kt, vt = (dev(x, h16).requires_grad_() for x in (q, k, v))
    gt = dev(g).requires_grad_()
    if op == "chunk":
        do = f16(do)  # o is fp16, so its gradient is too
        o, ht = gla.chunk_gla(qt, kt, vt, gt, output_final_state=True, chunk_size=16)
        assert o.dtype == h16 and ht.dtype == torch.float32
        o_r, ht_r = O.chunk_gla(q, k, v, g, output_final_state=True, chunk_size=16)
        (o.float() * dev(do)).sum().backward()
        dq_r, dk_r, dv_r, dg_r, _ = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, None, None, None, do, None, None, 16)
    else:
        o, ht = gla.fused_recurrent_gla(qt, kt, vt, gk=gt, output_final_state=True)
        assert o.dtype == torch.float32 and ht.dtype == torch.float32
        o_r, ht_r = O.fused_recurrent_gla(q, k, v, g, None, None, None, True)
        (o * dev(do)).sum().backward()
        dq_r, dk_r, dv_r, dg_r = O.fused_recurrent_gla_bwd(q, k, v, g, None, do, None, None, None)[:4]
    assert qt.grad.dtype == h16 and gt.grad.dtype == torch.float32
    for nm, got, want in (("o", o, o_r), ("ht", ht, ht_r), ("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r),
                          ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r)):
        assert_rel_l2(nm, got, want, 2e-3)


def test_recurrent_k_split(gla):
    """K > 256 takes the K-split path with a workspace reduction."""
    rng = np.random.default_rng(5)
    B, T, H, K, V = 1, 5, 2, 320, 64
    q, k = (rng.standard_normal((B, T, H, K), dtype=np.float32) for _ in range(2))
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    gk = GC.logsigmoid(rng.standard_normal((B, T, H, K))).astype(np.float32)
    o_r, ht_r = O.fused_recurrent_gla(q, k, v, gk, output_final_state=True)
    o, ht = gla.fused_recurrent_gla(dev(q), dev(k), dev(v), gk=dev(gk), output_final_state=True)
    assert_close("o", o, o_r, **FP32)
    assert_close("ht", ht, ht_r, **FP32)


def test_no_device_side_timeouts(gla):
    """No bounded device wait gave up during the tests above (error word stays 0)."""
    from tops import _C
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0


def test_decode_general_shapes(gla):
    """Streaming decode kernel (T == 1): gates on/off, no h0, no ht, several V."""
    rng = np.random.default_rng(31)
    for (B, H, K, V, gk_on, gv_on, h0_on) in [(3, 5, 64, 64, True, True, True), (2, 3, 128, 32, False, False, False),
                                              (4, 2, 32, 256, True, False, True), (1, 7, 128, 128, False, True, True)]:
        q, k = (rng.standard_normal((B, 1, H, K), dtype=np.float32) for _ in range(2))
        v = rng.standard_normal((B, 1, H, V), dtype=np.float32)
        gk = GC.logsigmoid(rng.standard_normal((B, 1, H, K))).astype(np.float32) if gk_on else None
        gv = GC.logsigmoid(rng.standard_normal((B, 1, H, V))).astype(np.float32) if gv_on else None
        h0 = rng.standard_normal((B, H, K, V), dtype=np.float32) if h0_on else None
        o_r, ht_r = O.fused_recurrent_gla(q, k, v, gk, gv, None, h0, True)
        for want_ht in (True, False):
            o, ht = gla.fused_recurrent_gla(dev(q), dev(k), dev(v), gk=dev(gk), gv=dev(gv), initial_state=dev(h0),
                                            output_final_state=want_ht)
            assert_close("o", o, o_r, **FP32)
            if want_ht:
                assert_close("ht", ht, ht_r, **FP32)


# ---------------------------------------------------------------------------
# tensor-core (tcgen05) path: bf16, K in {128, 256}, V % 128 == 0, fixed length
# ---------------------------------------------------------------------------

TC_CASES = [
    dict(B=2, T=640, H=2, K=256, V=512, seed=41),
    dict(B=1, T=333, H=3, K=128, V=256, seed=42, h0=True),
    dict(B=3, T=129, H=1, K=256, V=128, seed=43, h0=True),
    # few (batch, head, V-tile) units and many chunks: the state scans split into spans
    dict(B=1, T=4173, H=2, K=128, V=128, seed=47, h0=True, dht=True),
    dict(B=1, T=16384, H=1, K=128, V=256, seed=48, h0=True),
]


@pytest.mark.parametrize("case", TC_CASES, ids=lambda c: f"B{c['B']}T{c['T']}H{c['H']}K{c['K']}V{c['V']}")
def test_tc_forward_vs_oracle(gla, case):
    from tops import _C
    from tops.ops.gla import _core
    rng = np.random.default_rng(case["seed"])
    B, T, H, K, V = case["B"], case["T"], case["H"], case["K"], case["V"]
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32) if case.get("h0") else None
    bf = torch.bfloat16
    qt, kt, vt = (dev(x, bf) for x in (q, k, v))
    p = _core.make_plan(qt, V, 64, None, K ** -0.5)
    assert _core.saved_size(p, dev(g)) > 0, "case should take the tensor-core path"
    o, ht = gla.chunk_gla(qt, kt, vt, dev(g), initial_state=dev(h0), output_final_state=True, chunk_size=64)
    o_r, ht_r = O.chunk_gla(q, k, v, g, initial_state=h0, output_final_state=True, chunk_size=64)
    assert_rel_l2("o", o, o_r, BF16_L2)
    assert_rel_l2("ht", ht, ht_r, BF16_L2)
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0


@pytest.mark.parametrize("case", TC_CASES + [dict(B=1, T=200, H=2, K=128, V=128, seed=44, h0=True, dht=True)],
                         ids=lambda c: f"B{c['B']}T{c['T']}H{c['H']}K{c['K']}V{c['V']}")
def test_tc_backward_vs_oracle(gla, case):
    """bf16 fwd+bwd on the tensor-core path through torch.autograd vs the fp64 oracle (rel-L2 2e-2)."""
    from tops import _C
    rng = np.random.default_rng(case["seed"] + 100)
    B, T, H, K, V = case["B"], case["T"], case["H"], case["K"], case["V"]
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
    do = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    h0 = rng.standard_normal((B, H, K, V), dtype=np.float32) if case.get("h0") else None
    dht = rng.standard_normal((B, H, K, V), dtype=np.float32) if case.get("dht") else None
    bf = torch.bfloat16
    qt, kt, vt = (dev(x, bf).requires_grad_() for x in (q, k, v))
    gt = dev(g).requires_grad_()
    h0t = dev(h0)
    if h0t is not None:
        h0t.requires_grad_()
    o, ht = gla.chunk_gla(qt, kt, vt, gt, initial_state=h0t, output_final_state=True, chunk_size=64)
    loss = (o.float() * dev(do)).sum() + (0 if dht is None else (ht * dev(dht)).sum())
    loss.backward()
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, h0, None, None, do, dht, None, 64)
    for nm, got, want in (("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r), ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r)):
        assert_rel_l2(nm, got, want, BF16_L2)
    if h0t is not None:
        assert_rel_l2("dh0", h0t.grad, dh0_r, BF16_L2)
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0


def test_tc_with_the_api_default_chunk_size(gla):
    """chunk_gla's default chunk_size (16, as in the reference) on bf16 inputs takes the tensor-core
    path (which chunks by 128 internally: the result does not depend on the chunk size beyond
    rounding); fwd + bwd vs the fp64 oracle at chunk size 16 (rel-L2 2e-2)."""
    from tops import _C
    from tops.ops.gla import _core
    rng = np.random.default_rng(61)
    B, T, H, K, V = 1, 300, 2, 128, 128
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
    do = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    bf = torch.bfloat16
    qt, kt, vt = (dev(x, bf).requires_grad_() for x in (q, k, v))
    gt = dev(g).requires_grad_()
    assert _core.saved_size(_core.make_plan(qt, V, 16, None, K ** -0.5), gt) > 0, "should take the tensor-core path"
    o, ht = gla.chunk_gla(qt, kt, vt, gt, output_final_state=True)
    (o.float() * dev(do)).sum().backward()
    o_r, ht_r = O.chunk_gla(q, k, v, g, output_final_state=True, chunk_size=16)
    dq_r, dk_r, dv_r, dg_r, _ = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, None, None, None, do, None, None, 16)
    for nm, got, want in (("o", o, o_r), ("ht", ht, ht_r), ("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r),
                          ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r)):
        assert_rel_l2(nm, got, want, BF16_L2)
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0


def test_tc_long_sequence_takes_the_span_split_scan(gla):
    """A long single sequence (2 units, 128 chunks) runs its state scans as parallel spans."""
    from tops import _C
    from tops.ops.gla import _core
    torch.manual_seed(0)
    B, T, H, K, V = 1, 16384, 1, 128, 256
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device="cuda", dtype=bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", dtype=bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda")) / 16).contiguous()
    do = torch.randn(B, T, H, V, device="cuda", dtype=bf)
    p = _core.make_plan(q, V, 64, None, K ** -0.5)
    _C.timing_enable(True)
    try:
        o, ht, sv = _core.chunk_fwd(p, q, k, v, g, None, True, save=True)
        _core.chunk_bwd(p, q, k, v, g, None, do, None, block=sv.get("block"), want_dh0=True)
        torch.cuda.synchronize()
    finally:
        _C.timing_enable(False)
    names = {n for n, _ in _C.timing_collect()}
    assert {"tc_scan_span", "tc_span_prefix", "tc_scan_bwd_span"} <= names, names
    # the re-scan that stores the chunk states: fused with the output GEMM (default) or separate
    assert {"tc_scan_out", "tc_scan_out_bwd"} <= names or {"tc_scan", "tc_scan_bwd"} <= names, names
    assert _C.lib().tops_gla_device_error() == 0


@pytest.mark.parametrize("dtype,K,V", [(torch.bfloat16, 128, 128), (torch.float32, 64, 96)],
                         ids=["tensor-core", "cuda-core"])
def test_state_only_modes_match_full_calls(gla, dtype, K, V):
    """C ABI: o == NULL gives the forward's final state alone; all-NULL gradients give dh0 alone."""
    from tops import _C
    from tops.ops.gla import _core
    torch.manual_seed(3)
    B, T, H = 2, 700, 2
    q, k = (torch.randn(B, T, H, K, device="cuda").to(dtype) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda").to(dtype)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda")) / 16).contiguous()
    h0 = torch.randn(B, H, K, V, device="cuda")
    do = torch.randn(B, T, H, V, device="cuda").to(dtype)
    p = _core.make_plan(q, V, 64, None, K ** -0.5)
    o, ht, sv = _core.chunk_fwd(p, q, k, v, g, h0, True, save=True)
    ht_only = _core.final_state(p, q, k, v, g, h0)
    torch.testing.assert_close(ht_only, ht, rtol=1e-5, atol=1e-5)
    full = _core.chunk_bwd(p, q, k, v, g, h0, do, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"),
                           want_dh0=True, block=sv.get("block"))
    dh0 = _core.initial_state_grad(p, q, k, v, g, h0, do, None, block=sv.get("block"))
    torch.testing.assert_close(dh0, full[4], rtol=1e-5, atol=1e-5)
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0


@pytest.mark.parametrize("T,cu", [(5000, None), (3001, [0, 17, 1500, 3001])], ids=["fixed", "varlen"])
def test_span_decay_matches_torch(gla, T, cu):
    """exp(sum of a span's gates) per (sequence, head, K column): the sequence-parallel decay."""
    from tops.ops.gla import _core
    torch.manual_seed(1)
    B = 2 if cu is None else 1
    H, K = 3, 96
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda")) / 16).contiguous()
    q = torch.zeros(B, T, H, K, device="cuda")
    cut = None if cu is None else torch.tensor(cu, dtype=torch.int32, device="cuda")
    p = _core.make_plan(q, 32, 64, cut, 1.0)
    got = _core.span_decay(p, g)
    if cu is None:
        want = torch.exp(g.double().sum(1))
    else:
        want = torch.stack([torch.exp(g[0, a:b].double().sum(0)) for a, b in zip(cu, cu[1:])])
    torch.testing.assert_close(got.double(), want, rtol=1e-5, atol=1e-6)


def test_pinned_host_fwd_bwd_matches_device_calls(gla):
    """chunk_gla_fwd_bwd_pinned (host tensors, sliced over the batch, three streams) gives
    the gradients of the device-side forward + backward."""
    from tops.ops.gla import _core
    torch.manual_seed(9)
    B, T, H, K, V = 3, 520, 2, 128, 256
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K).to(bf).pin_memory() for _ in range(2))
    v = torch.randn(B, T, H, V).to(bf).pin_memory()
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K)) / 16).pin_memory()
    do = torch.randn(B, T, H, V).to(bf).pin_memory()
    got = gla.chunk_gla_fwd_bwd_pinned(q, k, v, g, do, chunk_size=64, slice_batch=1, depth=2)
    torch.cuda.synchronize()
    qd, kd, vd, gd, dod = (x.cuda() for x in (q, k, v, g, do))
    p = _core.make_plan(qd, V, 64, None, K ** -0.5)
    o, _, sv = _core.chunk_fwd(p, qd, kd, vd, gd, None, False, save=True)
    want = _core.chunk_bwd(p, qd, kd, vd, gd, None, dod, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"), False,
                           block=sv.get("block"))
    for nm, a, b in zip(("dq", "dk", "dv", "dg"), got, want[:4]):
        assert not a.is_cuda and a.is_pinned()
        assert_rel_l2(nm, a.float(), b.float().cpu(), 1e-3)


@pytest.mark.parametrize("cu,H,K,V", [([0, 300, 301, 777, 1000], 2, 128, 256), ([0, 640, 1280], 1, 256, 128)],
                         ids=["4seg", "2seg-aligned"])
def test_tc_varlen_fwd_bwd_vs_oracle(gla, cu, H, K, V):
    """Packed varlen (cu_seqlens) on the tensor-core path: segments padded to 128-row blocks
    on the device, the state scans follow the segment boundaries; fwd + bwd vs the oracle."""
    from tops import _C
    from tops.ops.gla import _core
    rng = np.random.default_rng(len(cu) * 7 + K)
    T = cu[-1]
    N = len(cu) - 1
    q, k = (GC.bf16_round(rng.standard_normal((1, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((1, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((1, T, H, K))) / 16).astype(np.float32)
    do = GC.bf16_round(rng.standard_normal((1, T, H, V), dtype=np.float32))
    h0 = rng.standard_normal((N, H, K, V), dtype=np.float32)
    dht = rng.standard_normal((N, H, K, V), dtype=np.float32)
    bf = torch.bfloat16
    cut = torch.tensor(cu, dtype=torch.int32, device="cuda")
    qt, kt, vt = (dev(x, bf).requires_grad_() for x in (q, k, v))
    gt = dev(g).requires_grad_()
    h0t = dev(h0).requires_grad_()
    p = _core.make_plan(qt, V, 64, cut, K ** -0.5)
    assert _core.saved_size(p, gt) > 0, "case should take the tensor-core path"
    o, ht = gla.chunk_gla(qt, kt, vt, gt, initial_state=h0t, output_final_state=True, cu_seqlens=cut, chunk_size=64)
    o_r, ht_r = O.chunk_gla(q, k, v, g, initial_state=h0, output_final_state=True, cu_seqlens=cu, chunk_size=64)
    assert_rel_l2("o", o, o_r, BF16_L2)
    assert_rel_l2("ht", ht, ht_r, BF16_L2)
    ((o.float() * dev(do)).sum() + (ht * dev(dht)).sum()).backward()
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, h0, None, None, do, dht, cu, 64)
    for nm, got, want in (("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r), ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r),
                          ("dh0", h0t.grad, dh0_r)):
        assert_rel_l2(nm, got, want, BF16_L2)
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0


def test_pinned_pipeline_back_to_back_steps(gla):
    """Two steps submitted back to back through one PinnedGLAPipeline (ring slots reused
    across the steps) give each step's own gradients."""
    from tops.ops.gla import _core
    torch.manual_seed(10)
    B, T, H, K, V = 3, 300, 1, 128, 128
    bf = torch.bfloat16

    def inputs():
        q, k = (torch.randn(B, T, H, K).to(bf).pin_memory() for _ in range(2))
        v = torch.randn(B, T, H, V).to(bf).pin_memory()
        g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K)) / 16).pin_memory()
        do = torch.randn(B, T, H, V).to(bf).pin_memory()
        return q, k, v, g, do

    def out_buffers():
        return (torch.empty(B, T, H, K, dtype=bf).pin_memory(), torch.empty(B, T, H, K, dtype=bf).pin_memory(),
                torch.empty(B, T, H, V, dtype=bf).pin_memory(), torch.empty(B, T, H, K).pin_memory())

    steps = [inputs(), inputs()]
    outs = [out_buffers(), out_buffers()]
    pipe = gla.PinnedGLAPipeline(B, T, H, K, V, bf, depth=2)
    for x, o in zip(steps, outs):
        pipe.submit(*x, o)
    pipe.synchronize()
    for x, o in zip(steps, outs):
        qd, kd, vd, gd, dod = (t.cuda() for t in x)
        p = _core.make_plan(qd, V, 64, None, K ** -0.5)
        _, _, sv = _core.chunk_fwd(p, qd, kd, vd, gd, None, False, save=True)
        want = _core.chunk_bwd(p, qd, kd, vd, gd, None, dod, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"),
                               False, block=sv.get("block"))
        for nm, a, b in zip(("dq", "dk", "dv", "dg"), o, want[:4]):
            assert_rel_l2(nm, a.float(), b.float().cpu(), 1e-3)


_UNFUSED_CHILD = r"""
import sys
import numpy as np
import torch
root = sys.argv[1]
sys.path[:0] = [root, root + "/pallas-kernel_b200", root + "/tests", root + "/tests/golden"]
import cases as GC
from oracle import gla_oracle as O
from tops import _C
from tops.ops.gla import _core
B, T, H, K, V = 1, 333, 3, 128, 256
rng = np.random.default_rng(42)
q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
do = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
h0 = rng.standard_normal((B, H, K, V), dtype=np.float32)
dev = lambda x, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dt)
bf = torch.bfloat16
p = _core.make_plan(dev(q, bf), V, 64, None, K ** -0.5)
_C.timing_enable(True)
o, ht, sv = _core.chunk_fwd(p, dev(q, bf), dev(k, bf), dev(v, bf), dev(g), dev(h0), True, save=True)
dq, dk, dv, dg, dh0 = _core.chunk_bwd(p, dev(q, bf), dev(k, bf), dev(v, bf), dev(g), dev(h0), dev(do, bf), None,
                                      sv.get("g_cumsum"), sv.get("A"), sv.get("h"), True, block=sv.get("block"))
torch.cuda.synchronize()
_C.timing_enable(False)
names = {n for n, _ in _C.timing_collect()}
assert {"tc_scan", "tc_out", "tc_scan_bwd", "tc_out_dv"} <= names, names
o_r, ht_r = O.chunk_gla(q, k, v, g, initial_state=h0, output_final_state=True, chunk_size=64)
ref = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, h0, None, None, do, None, None, 64)
rel = lambda a, b: float(np.linalg.norm(a.float().cpu().numpy() - b) / np.linalg.norm(b))
errs = [rel(a, b) for a, b in zip((o, ht, dq, dk, dv, dg, dh0), (o_r, ht_r) + tuple(ref))]
assert max(errs) < 2e-2, errs
assert _C.lib().tops_gla_device_error() == 0
print("UNFUSED_OK", max(errs))
"""


def test_unfused_scan_and_output_path(gla):
    """TOPS_GLA_UNFUSED_OUT=1 selects the separate state scan and k_out GEMM (read once per
    process, so it runs in a child): same results as the oracle, and those kernels ran."""
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = str(Path(__file__).resolve().parents[1])
    env = dict(os.environ, TOPS_GLA_UNFUSED_OUT="1")
    r = subprocess.run([sys.executable, "-c", _UNFUSED_CHILD, root], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "UNFUSED_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_bounded_wait_timeout_is_reported_and_context_survives(gla):
    """Failure path without a GPU fault: a kernel waits on an mbarrier that nothing will
    complete; its bounded wait gives up (about 2 s), records code 1, and returns.  The host
    reads the code, and the next operation runs normally."""
    import ctypes

    from tops import _C
    _C.lib().tops_gla_device_error()  # clear anything earlier tests left
    _C.call("tops_gla_selftest_wait_timeout", ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 1
    rng = np.random.default_rng(5)
    B, T, H, K, V = 1, 256, 2, 128, 128
    q, k = (GC.bf16_round(rng.standard_normal((B, T, H, K), dtype=np.float32)) for _ in range(2))
    v = GC.bf16_round(rng.standard_normal((B, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
    bf = torch.bfloat16
    o, ht = gla.chunk_gla(dev(q, bf), dev(k, bf), dev(v, bf), dev(g), output_final_state=True, chunk_size=64)
    o_r, ht_r = O.chunk_gla(q, k, v, g, output_final_state=True, chunk_size=64)
    assert_rel_l2("o after the timeout", o, o_r, BF16_L2)
    assert _C.lib().tops_gla_device_error() == 0
