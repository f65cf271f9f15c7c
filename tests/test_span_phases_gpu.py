"""The two-phase span entry points (tops_gla_chunk_{fwd,bwd}_span_{begin,finish}) on one GPU.

A sequence-parallel run over R ranks is emulated on one device: every span runs its first
phase, the host combines the spans' (local state, decay) and local dh0 with the same prefix /
suffix the ranks use (tops.distributed.prefix_states / suffix_grads), and every span runs its
second phase from its incoming state.  The concatenated outputs and gradients must equal the
whole sequence run in one call (relative L2 1e-2: the same bf16 kernels, state rounding at
different chunk boundaries) and the oracle (relative L2 2e-2, the bf16 tolerance), and each
span's decay must equal exp of its gate sums.  Cases cover spans that the GPU splits further
into parallel scan spans, and spans that run as one scan span (K = V = 256).
The reference has no multi-device code; the state chaining it pins is
tests/ops/gla/test_pallas_chunk_gla.py:223-248.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from _util import assert_close, assert_rel_l2
from oracle import gla_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    from tops import _C
    from tops import distributed as TD
    from tops.ops.gla import _core
    L = _C.lib()
    if not L.tops_gla_has_tcgen05():
        pytest.skip("the span entry points serve the tensor-core path (sm_100)")
    return _C, _core, TD


def _inputs(seed, B, T, H, K, V):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device="cuda", generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", generator=gen).to(bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda", generator=gen)) / 16).contiguous()
    h0 = torch.randn(B, H, K, V, device="cuda", generator=gen) * 0.1
    do = torch.randn(B, T, H, V, device="cuda", generator=gen).to(bf)
    dht = torch.randn(B, H, K, V, device="cuda", generator=gen) * 0.1
    return q, k, v, g, h0, do, dht


@pytest.mark.parametrize("R,shape", [
    (2, (1, 8192, 2, 128, 128)),   # 4096-token spans, each split into 2 scan spans on the GPU
    (4, (1, 16384, 1, 128, 128)),  # four ranks: the prefix / suffix chain more than one hop
    (2, (2, 1024, 2, 256, 256)),   # one scan span per rank span
], ids=["r2_k128", "r4_k128", "r2_k256"])
def test_span_phases_match_whole_sequence(env, R, shape):
    _C, _core, TD = env
    import tops.ops.gla as G
    B, T, H, K, V = shape
    C = 64
    q, k, v, g, h0, do, dht = _inputs(7, B, T, H, K, V)
    Tr = T // R
    parts = [tuple(x[:, r * Tr:(r + 1) * Tr].contiguous() for x in (q, k, v, g, do)) for r in range(R)]
    plan = _core.make_plan(parts[0][0], V, C, None, K ** -0.5)
    assert _core.span_saved_size(plan, parts[0][3]) > 0

    # phase 1 of every span, the host prefix, phase 2
    begun = [_core.fwd_span_begin(plan, *p[:4]) for p in parts]
    S_all = torch.stack([b[0] for b in begun])
    D_all = torch.stack([b[1] for b in begun])
    H_all = TD.prefix_states(S_all, D_all, h0)
    outs = [_core.fwd_span_finish(plan, *p[:4], H_all[r], begun[r][2], want_ht=True) for r, p in enumerate(parts)]
    o_sp = torch.cat([x[0] for x in outs], 1)
    ht_sp = outs[-1][1]
    bw = [_core.bwd_span_begin(plan, *p[:4], p[4], begun[r][2]) for r, p in enumerate(parts)]
    G_all = TD.suffix_grads(torch.stack([b[0] for b in bw]), D_all, dht)
    grads = [_core.bwd_span_finish(plan, *p[:4], p[4], G_all[r], begun[r][2], bw[r][1], want_dh0=(r == 0))
             for r, p in enumerate(parts)]
    torch.cuda.synchronize()
    assert _C.lib().tops_gla_device_error() == 0

    for r, p in enumerate(parts):  # decay = exp of the span's gate sums (long spans underflow to 0)
        assert_close(f"decay of span {r}", D_all[r], torch.exp(p[3].double().sum(1)), atol=1e-30, rtol=1e-4)

    # the whole sequence in one call
    qt, kt, vt, gt = (x.clone().requires_grad_() for x in (q, k, v, g))
    h0t = h0.clone().requires_grad_()
    o, ht = G.chunk_gla(qt, kt, vt, gt, initial_state=h0t, output_final_state=True, chunk_size=C)
    ((o.float() * do.float()).sum() + (ht * dht).sum()).backward()
    assert_rel_l2("o vs one call", o_sp, o, 1e-2)
    assert_rel_l2("ht vs one call", ht_sp, ht, 1e-2)
    for i, (nm, t) in enumerate((("dq", qt), ("dk", kt), ("dv", vt), ("dg", gt))):
        assert_rel_l2(f"{nm} vs one call", torch.cat([x[i] for x in grads], 1), t.grad, 1e-2)
    assert_rel_l2("dh0 vs one call", grads[0][4], h0t.grad, 1e-2)

    # and the oracle
    qn, kn, vn, gn, h0n, don, dhtn = (x.float().cpu().numpy() for x in (q, k, v, g, h0, do, dht))
    o_r, ht_r = O.chunk_gla(qn, kn, vn, gn, initial_state=h0n, output_final_state=True, chunk_size=C,
                            dtype=np.float32)
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(qn, kn, vn, gn, None, K ** -0.5, h0n, None, None, don, dhtn,
                                                    None, C, dtype=np.float32)
    assert_rel_l2("o vs oracle", o_sp, o_r, 2e-2)
    assert_rel_l2("ht vs oracle", ht_sp, ht_r, 2e-2)
    for i, (nm, ref) in enumerate((("dq", dq_r), ("dk", dk_r), ("dv", dv_r), ("dg", dg_r))):
        assert_rel_l2(f"{nm} vs oracle", torch.cat([x[i] for x in grads], 1), ref, 2e-2)
    assert_rel_l2("dh0 vs oracle", grads[0][4], dh0_r, 2e-2)


def test_span_entry_points_reject_what_they_do_not_serve(env):
    _C, _core, _ = env
    import ctypes
    L = _C.lib()
    q = torch.zeros(1, 256, 2, 32, dtype=torch.bfloat16, device="cuda")  # K = 32: CUDA-core path
    plan = _core.make_plan(q, 64, 64, None, None)
    assert L.tops_gla_chunk_span_saved_size(ctypes.byref(plan.shape())) == 0
    a = _C.ChunkFwdArgs(plan.shape(), 1, 1, 1, 1, None, 1, None, None, None, None, None, 0, 1, 1 << 30)
    assert L.tops_gla_chunk_fwd_span_begin(ctypes.byref(a), 1, 1, None) == -2  # TOPS_ERR_UNSUPPORTED
    q = torch.zeros(1, 256, 2, 128, dtype=torch.bfloat16, device="cuda")
    plan = _core.make_plan(q, 128, 64, None, None)
    need = L.tops_gla_chunk_span_saved_size(ctypes.byref(plan.shape()))
    assert need > 0
    a = _C.ChunkFwdArgs(plan.shape(), 1, 1, 1, 1, None, 1, None, None, None, None, None, 0, 1, need - 1)
    assert L.tops_gla_chunk_fwd_span_begin(ctypes.byref(a), 1, 1, None) == -4  # block too small, nothing launched
