"""Parity at BASELINE's full sizes (configs 3 and 4) on one GPU.

Chunked GLA is independent across (sequence, head) pairs, so the oracle run on one (b, h)
slice is the exact reference for that slice of a full-size run.  These tests run the whole
BASELINE workload (forward and backward, tensor-core path, seeded synthetic inputs) and compare
sampled slices of every output and gradient with the float32 oracle at the bf16 tolerance used
by the other tensor-core cases (relative L2 2e-2).  The state split -- a sequence run in two
halves, the second starting from the first half's final state -- must reproduce the one-piece
run at any size.

Every (sequence, head) slice of config 3 (32) and four spread heads of config 4 (the first,
the last and two between) are compared, each against relative L2 2e-2 and an element-wise
bound (max |err| <= 2e-2 x max |ref| of the slice), so one bad tile or head cannot hide in
an average.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_max_rel, assert_rel_l2
from oracle import gla_oracle as O

pytestmark = pytest.mark.gpu

BF16_L2 = 2e-2

CONFIGS = {
    # one 1.3B-model layer
    "cfg3": dict(B=8, T=4096, H=4, K=256, V=512, slices=tuple((b, h) for b in range(8) for h in range(4)), seed=3),
    # long context on one GPU (the state scans run as parallel spans)
    "cfg4": dict(B=1, T=131072, H=16, K=128, V=128, slices=((0, 0), (0, 5), (0, 11), (0, 15)), seed=4),
}


@pytest.fixture(scope="module")
def gla():
    import tops.ops.gla as G
    from tops import _C
    _C.lib()
    return G


def _inputs(c):
    gen = torch.Generator(device="cuda").manual_seed(c["seed"])
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device="cuda", generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", generator=gen).to(bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda", generator=gen)) / 16).contiguous()
    do = torch.randn(B, T, H, V, device="cuda", generator=gen).to(bf)
    return q, k, v, g, do


def _slice(x, b, h):
    return x[b:b + 1, :, h:h + 1].detach().float().cpu().numpy()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_size_slices_vs_oracle(gla, name):
    from tops import _C
    c = CONFIGS[name]
    K = c["K"]
    q, k, v, g, do = _inputs(c)
    qt, kt, vt, gt = (x.clone().requires_grad_() for x in (q, k, v, g))
    o, ht = gla.chunk_gla(qt, kt, vt, gt, output_final_state=True, chunk_size=64)
    (o.float() * do.float()).sum().backward()
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0
    for b, h in c["slices"]:
        qs, ks, vs, gs, dos = (_slice(x, b, h) for x in (q, k, v, g, do))
        o_r, ht_r = O.chunk_gla(qs, ks, vs, gs, output_final_state=True, chunk_size=64, dtype=np.float32)
        dq_r, dk_r, dv_r, dg_r, _ = O.chunk_gla_bwd(qs, ks, vs, gs, None, K ** -0.5, None, None, None, dos, None,
                                                    None, 64, dtype=np.float32)
        at = f"{name} (b={b}, h={h})"
        pairs = [("o", _slice(o, b, h), o_r), ("ht", ht[b:b + 1, h:h + 1], ht_r)]
        pairs += [(nm, _slice(t.grad, b, h), r) for nm, t, r in
                  (("dq", qt, dq_r), ("dk", kt, dk_r), ("dv", vt, dv_r), ("dg", gt, dg_r))]
        for nm, got, ref in pairs:
            assert_rel_l2(f"{nm} {at}", got, ref, BF16_L2)
            assert_max_rel(f"{nm} {at}", got, ref, BF16_L2)


def test_full_size_state_split(gla):
    """Config 3 run in one piece equals the two halves chained through the final state."""
    c = CONFIGS["cfg3"]
    q, k, v, g, _ = _inputs(c)
    h0 = torch.randn(c["B"], c["H"], c["K"], c["V"], device="cuda") * 0.1
    o, ht = gla.chunk_gla(q, k, v, g, initial_state=h0, output_final_state=True, chunk_size=64)
    m = c["T"] // 2
    o1, h1 = gla.chunk_gla(q[:, :m], k[:, :m], v[:, :m], g[:, :m], initial_state=h0, output_final_state=True,
                           chunk_size=64)
    o2, h2 = gla.chunk_gla(q[:, m:].contiguous(), k[:, m:].contiguous(), v[:, m:].contiguous(),
                           g[:, m:].contiguous(), initial_state=h1, output_final_state=True, chunk_size=64)
    assert_rel_l2("o (first half)", o1, o[:, :m], BF16_L2)
    assert_rel_l2("o (second half)", o2, o[:, m:], BF16_L2)
    assert_rel_l2("ht", h2, ht, BF16_L2)
