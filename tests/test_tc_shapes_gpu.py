"""Tensor-core path for the head sizes the reference pads to 128 (tops/ops/gla/chunk.py:1128-1132)
and for fp16 inputs: K = 64 and V = 64, alone and combined with 128 / 256, in bf16 and fp16,
forward and backward, against the oracle at the 16-bit tolerance (relative L2 2e-2) plus an
element-wise bound relative to each tensor's scale.  Each case asserts that it runs on the
tensor-core path (a saved block exists) and that outputs keep the reference's dtypes (o, dq,
dk, dv in the input dtype; ht, dg, dh0 fp32), and covers an initial state, a final-state
gradient and a ragged last chunk.  The reference's own tests use K = 64 throughout
(tests/ops/gla/test_pallas_chunk_gla.py:24-126).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_max_rel, assert_rel_l2
from oracle import gla_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(scope="module")
def env():
    from tops import _C
    from tops.ops.gla import _core
    import tops.ops.gla as G
    if not _C.lib().tops_gla_has_tcgen05():
        pytest.skip("needs an sm_100 device")
    return _C, _core, G


def _inputs(seed, B, T, H, K, V, dtype):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k = (torch.randn(B, T, H, K, device="cuda", generator=gen).to(dtype) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", generator=gen).to(dtype)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda", generator=gen)) / 16).contiguous()
    h0 = torch.randn(B, H, K, V, device="cuda", generator=gen) * 0.1
    do = torch.randn(B, T, H, V, device="cuda", generator=gen).to(dtype)
    dht = torch.randn(B, H, K, V, device="cuda", generator=gen) * 0.1
    return q, k, v, g, h0, do, dht


SHAPES = [(64, 64), (64, 128), (128, 64), (64, 256), (256, 64), (128, 128)]


@pytest.mark.parametrize("K,V", SHAPES, ids=[f"k{k}v{v}" for k, v in SHAPES])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_tc_head_sizes_fwd_bwd(env, K, V, dtype):
    _C, _core, G = env
    B, T, H, C = 2, 300, 3, 64  # T = 300: a ragged last 128-row block
    q, k, v, g, h0, do, dht = _inputs(K * 7 + V, B, T, H, K, V, dtype)
    plan = _core.make_plan(q, V, C, None, K ** -0.5)
    assert _core.saved_size(plan, g) > 0, "expected the tensor-core path"
    qt, kt, vt, gt = (x.clone().requires_grad_() for x in (q, k, v, g))
    h0t = h0.clone().requires_grad_()
    o, ht = G.chunk_gla(qt, kt, vt, gt, initial_state=h0t, output_final_state=True, chunk_size=C)
    assert o.dtype == dtype and ht.dtype == torch.float32
    ((o.float() * do.float()).sum() + (ht * dht).sum()).backward()
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0
    qn, kn, vn, gn, h0n, don, dhtn = (x.float().cpu().numpy() for x in (q, k, v, g, h0, do, dht))
    o_r, ht_r = O.chunk_gla(qn, kn, vn, gn, initial_state=h0n, output_final_state=True, chunk_size=C)
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(qn, kn, vn, gn, None, K ** -0.5, h0n, None, None, don, dhtn,
                                                    None, C)
    for nm, got, ref in (("o", o, o_r), ("ht", ht, ht_r), ("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r),
                         ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r), ("dh0", h0t.grad, dh0_r)):
        assert got.dtype == (dtype if nm in ("o", "dq", "dk", "dv") else torch.float32), nm
        assert_rel_l2(nm, got, ref, TOL)
        assert_max_rel(nm, got, ref, TOL)


def test_f16_matches_bf16_path_on_shared_values(env):
    """fp16 inputs that are exactly bf16 values must give what the bf16 inputs give (the fp16 path
    widens q, k in registers and copies v, do to bf16; everything after is the same kernels)."""
    _C, _core, G = env
    B, T, H, K, V, C = 1, 512, 2, 128, 128, 64
    q, k, v, g, h0, do, _ = _inputs(3, B, T, H, K, V, torch.bfloat16)
    outs = {}
    for dt in (torch.bfloat16, torch.float16):
        qt, kt, vt = (x.detach().to(dt).clone().requires_grad_() for x in (q, k, v))
        gt = g.clone().requires_grad_()
        o, ht = G.chunk_gla(qt, kt, vt, gt, initial_state=h0, output_final_state=True, chunk_size=C)
        (o.float() * do.float()).sum().backward()
        outs[dt] = (o.float(), ht, qt.grad.float(), kt.grad.float(), vt.grad.float(), gt.grad)
    for nm, a, b in zip(("o", "ht", "dq", "dk", "dv", "dg"), outs[torch.float16], outs[torch.bfloat16]):
        assert_rel_l2(f"{nm} fp16 vs bf16", a, b, 5e-3)  # outputs rounded to fp16 vs bf16 at the end


@pytest.mark.parametrize("K,V", [(64, 64), (64, 256), (256, 64)], ids=["k64v64", "k64v256", "k256v64"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_tc_varlen_head_sizes(env, K, V, dtype):
    """Packed varlen (cu_seqlens, a one-token segment among them) on the tensor-core path with
    padded head sizes and fp16: segments are padded to 128-row blocks on the device, the scans
    follow the segment boundaries; forward + backward against the oracle per the same values."""
    _C, _core, G = env
    cu = [0, 300, 301, 777, 1000]
    T, N, H, C = cu[-1], len(cu) - 1, 2, 64
    q, k, v, g, _, do, _ = _inputs(K + V, 1, T, H, K, V, dtype)
    gen = torch.Generator(device="cuda").manual_seed(5)
    h0 = torch.randn(N, H, K, V, device="cuda", generator=gen) * 0.1
    dht = torch.randn(N, H, K, V, device="cuda", generator=gen) * 0.1
    cut = torch.tensor(cu, dtype=torch.int32, device="cuda")
    plan = _core.make_plan(q, V, C, cut, K ** -0.5)
    assert _core.saved_size(plan, g) > 0, "expected the tensor-core path"
    qt, kt, vt, gt = (x.clone().requires_grad_() for x in (q, k, v, g))
    h0t = h0.clone().requires_grad_()
    o, ht = G.chunk_gla(qt, kt, vt, gt, initial_state=h0t, output_final_state=True, cu_seqlens=cut, chunk_size=C)
    ((o.float() * do.float()).sum() + (ht * dht).sum()).backward()
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0
    qn, kn, vn, gn, h0n, don, dhtn = (x.float().cpu().numpy() for x in (q, k, v, g, h0, do, dht))
    o_r, ht_r = O.chunk_gla(qn, kn, vn, gn, initial_state=h0n, output_final_state=True, cu_seqlens=cu, chunk_size=C)
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(qn, kn, vn, gn, None, K ** -0.5, h0n, None, None, don, dhtn,
                                                    cu, C)
    for nm, got, ref in (("o", o, o_r), ("ht", ht, ht_r), ("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r),
                         ("dv", vt.grad, dv_r), ("dg", gt.grad, dg_r), ("dh0", h0t.grad, dh0_r)):
        assert_rel_l2(nm, got, ref, TOL)
        assert_max_rel(nm, got, ref, TOL)


def test_tc_ungated(env):
    """Neither g nor g_gamma on a tensor-core shape: the library substitutes zero gates (as the
    reference does, chunk.py:1114-1118) and stays on the tensor-core path; fwd + bwd match the
    oracle with g = None, and equal an explicit all-zero gate bit for bit."""
    _C, _core, G = env
    B, T, H, K, V, C = 2, 320, 2, 128, 128, 64
    q, k, v, _, h0, do, dht = _inputs(21, B, T, H, K, V, torch.bfloat16)
    plan = _core.make_plan(q, V, C, None, K ** -0.5)
    assert _core.saved_size(plan, None) > 0, "expected the tensor-core path"
    qt, kt, vt = (x.clone().requires_grad_() for x in (q, k, v))
    h0t = h0.clone().requires_grad_()
    o, ht = G.chunk_gla(qt, kt, vt, initial_state=h0t, output_final_state=True, chunk_size=C)
    ((o.float() * do.float()).sum() + (ht * dht).sum()).backward()
    z = torch.zeros(B, T, H, K, device="cuda")
    o0, ht0 = G.chunk_gla(q, k, v, z, initial_state=h0, output_final_state=True, chunk_size=C)
    assert torch.equal(o.detach(), o0) and torch.equal(ht.detach(), ht0), "ungated differs from g = 0"
    qn, kn, vn, h0n, don, dhtn = (x.float().cpu().numpy() for x in (q, k, v, h0, do, dht))
    o_r, ht_r = O.chunk_gla(qn, kn, vn, None, initial_state=h0n, output_final_state=True, chunk_size=C)
    dq_r, dk_r, dv_r, _, dh0_r = O.chunk_gla_bwd(qn, kn, vn, None, None, K ** -0.5, h0n, None, None, don, dhtn,
                                                 None, C)
    for nm, got, ref in (("o", o, o_r), ("ht", ht, ht_r), ("dq", qt.grad, dq_r), ("dk", kt.grad, dk_r),
                         ("dv", vt.grad, dv_r), ("dh0", h0t.grad, dh0_r)):
        assert_rel_l2(nm, got, ref, TOL)
