"""Packed varlen inputs with empty segments (zero-length entries in cu_seqlens).

An empty sequence has no tokens: its final state is its initial state, and the gradient of
its initial state is the gradient of its final state.  Every other segment must come out as if
it ran alone.  Checked on the CUDA-core path (fp32, max-abs/rel 1e-4) and the tensor-core
path (bf16, relative L2 2e-2), forward and backward, against the float64 oracle run on each
non-empty segment by itself.
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
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


CASES = [
    # CUDA-core path: fp32, small K / V, chunk 16
    dict(name="fp32", lens=(0, 23, 0, 40, 0), H=2, K=32, V=48, C=16, dtype=torch.float32),
    # tensor-core path: bf16, K = V = 128 (segments padded to 128-row blocks on the device; the
    # path takes packed inputs while (ceil(T / 128) + N) * 128 <= 2 T + 128, empty segments
    # included in N, so the non-empty ones are long here)
    dict(name="bf16_tc", lens=(0, 600, 0, 700, 0), H=2, K=128, V=128, C=64, dtype=torch.bfloat16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["name"])
def test_varlen_with_empty_segments(gla, case):
    from tops import _C
    from tops.ops.gla import _core
    lens, H, K, V, C, dt = case["lens"], case["H"], case["K"], case["V"], case["C"], case["dtype"]
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    T, N = cu[-1], len(lens)
    rng = np.random.default_rng(sum(lens) + K)
    rnd = GC.bf16_round if dt == torch.bfloat16 else (lambda x: x)
    q, k = (rnd(rng.standard_normal((1, T, H, K), dtype=np.float32)) for _ in range(2))
    v = rnd(rng.standard_normal((1, T, H, V), dtype=np.float32))
    g = (GC.logsigmoid(rng.standard_normal((1, T, H, K))) / 16).astype(np.float32)
    do = rnd(rng.standard_normal((1, T, H, V), dtype=np.float32))
    h0 = rng.standard_normal((N, H, K, V), dtype=np.float32)
    dht = rng.standard_normal((N, H, K, V), dtype=np.float32)
    cut = torch.tensor(cu, dtype=torch.int32, device="cuda")
    qt, kt, vt = (dev(x, dt).requires_grad_() for x in (q, k, v))
    gt = dev(g).requires_grad_()
    h0t = dev(h0).requires_grad_()
    on_tc = _core.saved_size(_core.make_plan(qt, V, C, cut, K ** -0.5), gt) > 0
    assert on_tc == (dt == torch.bfloat16), "the case should take the path it is named after"
    o, ht = gla.chunk_gla(qt, kt, vt, gt, initial_state=h0t, output_final_state=True, cu_seqlens=cut, chunk_size=C)
    ((o.float() * dev(do)).sum() + (ht * dev(dht)).sum()).backward()
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0

    def check(nm, got, want):
        if dt == torch.float32:
            assert_close(nm, got, want, **FP32)
        else:
            assert_rel_l2(nm, got, want, BF16_L2)

    for n in range(N):
        a, b = cu[n], cu[n + 1]
        if a == b:  # empty: the state passes through unchanged, in both directions
            assert torch.equal(ht[n], h0t[n].detach()), f"ht of empty segment {n} is not its initial state"
            assert torch.equal(h0t.grad[n], dev(dht[n])), f"dh0 of empty segment {n} is not its dht"
            continue
        sl = (slice(None), slice(a, b))
        o_r, ht_r = O.chunk_gla(q[sl], k[sl], v[sl], g[sl], initial_state=h0[n:n + 1], output_final_state=True,
                                chunk_size=C)
        dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(q[sl], k[sl], v[sl], g[sl], None, K ** -0.5, h0[n:n + 1],
                                                        None, None, do[sl], dht[n:n + 1], None, C)
        check(f"o[{n}]", o[sl], o_r)
        check(f"ht[{n}]", ht[n:n + 1], ht_r)
        for nm, t, r in (("dq", qt, dq_r), ("dk", kt, dk_r), ("dv", vt, dv_r), ("dg", gt, dg_r)):
            check(f"{nm}[{n}]", t.grad[sl], r)
        check(f"dh0[{n}]", h0t.grad[n:n + 1], dh0_r)
