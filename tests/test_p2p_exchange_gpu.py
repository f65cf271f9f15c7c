"""The peer-memory state exchange (tops_gla_p2p_exchange) on one GPU.

One rank of a group of two or four runs the real entry point.  The other ranks' parts -- their
packed (state | decay) in their slots of this rank's region and their epoch flags -- are
written into the region beforehand, as their pushes would have left them, so no kernel here
waits for another launch.  The regions are plain device tensors (one process, no IPC); the
others stand in for the other ranks' regions, which this rank's push also writes.  Checked: the forward prefix and total
and the backward suffix against the same arithmetic on the host (fused multiply-add, as the
kernel computes it), the alternating slot parity of consecutive exchanges, and the failure
path -- a flag that nothing sets makes the bounded device wait give up (device error 3,
output left untouched) and the context stays usable.  The two-GPU run over real peer
mappings is in test_seqpar_gpu.py.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CTRL = 4096
MAXW = 64


@pytest.fixture(scope="module")
def C():
    from tops import _C
    _C.lib()
    return _C


def _region(C, world, shape):
    a = C.P2PArgs(0, world, *shape, 0, None, None, None, None, None, None, None, 1000)
    n = int(C.lib().tops_gla_p2p_region_size(ctypes.byref(a)))
    return torch.zeros(n, dtype=torch.uint8, device="cuda")


def _slot(region, world, per, par, rank):
    f = region[CTRL:].view(torch.float32)
    return f[(par * world + rank) * per:(par * world + rank + 1) * per]


def _flags(region):
    return region[:2 * MAXW * 4].view(torch.int32).view(2, MAXW)


def _epoch(region):
    return int(region[1024:1028].view(torch.int32).item())


def _fma_chain(parts, boundary, order):
    """x <- D_r * x + S_r over `order`, in float32 with one rounding per step (fmaf)."""
    x = boundary.astype(np.float64)
    out = {}
    for r in order:
        out[r] = x.astype(np.float32)
        S, D = parts[r]
        x = (D.astype(np.float64)[..., None] * x.astype(np.float32).astype(np.float64) + S.astype(np.float64))
        x = x.astype(np.float32).astype(np.float64)  # fmaf rounds once
    return out, x.astype(np.float32)


def _exchange(C, rank, world, S, D, boundary, regions, own, backward, timeout_ms=2000):
    N, H, K, V = S.shape
    out = torch.full_like(S, float("nan"))
    total = None if backward else torch.full_like(S, float("nan"))
    table = torch.tensor([r.data_ptr() for r in regions], dtype=torch.int64, device="cuda")
    a = C.P2PArgs(rank, world, N, H, K, V, int(backward), C.ptr(S), C.ptr(D), C.ptr(boundary), C.ptr(out),
                  C.ptr(total), C.ptr(table), own.data_ptr(), timeout_ms)
    C.call("tops_gla_p2p_exchange", a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out, total


def _plant(region, world, per, par, rank, S, D, epoch):
    """Leave rank `rank`'s slot and flag in `region` as its push for `epoch` would."""
    _slot(region, world, per, par, rank).copy_(torch.cat([S.reshape(-1), D.reshape(-1)]))
    _flags(region)[par, rank] = epoch


@pytest.mark.parametrize("world,rank,shape", [
    (2, 0, (1, 4, 128, 128)),
    (2, 0, (1, 3, 63, 96)),    # K = 63: the per-element (not 16-byte) push
    (4, 1, (1, 2, 128, 128)),  # a middle rank: prefix over one rank, suffix over two
    (4, 3, (2, 2, 64, 64)),    # the last rank: prefix over three, empty suffix
], ids=["w2r0", "w2r0-scalar", "w4r1", "w4r3"])
def test_p2p_exchange_emulated_ranks(C, world, rank, shape):
    N, H, K, V = shape
    per = N * H * K * V + N * H * K
    gen = torch.Generator(device="cuda").manual_seed(3 + world + rank)
    regions = [_region(C, world, shape) for _ in range(world)]
    own = regions[rank]
    h0 = torch.randn(*shape, device="cuda", generator=gen)
    for e in (1, 2, 3):  # three exchanges: slot parities 1, 0, 1 (forward, backward, forward)
        par = e & 1
        assert _epoch(own) == e - 1
        S = [torch.randn(*shape, device="cuda", generator=gen) for _ in range(world)]
        D = [torch.rand(N, H, K, device="cuda", generator=gen) for _ in range(world)]
        for j in range(world):
            if j != rank:
                _plant(own, world, per, par, j, S[j], D[j], e)
        backward = e == 2
        out, total = _exchange(C, rank, world, S[rank], D[rank], h0, regions, own, backward)
        assert int(C.lib().tops_gla_device_error()) == 0
        for reg in regions:  # this rank's slot and flag went into every region
            got = _slot(reg, world, per, par, rank)
            assert torch.equal(got, torch.cat([S[rank].reshape(-1), D[rank].reshape(-1)]))
            assert int(_flags(reg)[par, rank]) == e
        parts = {r: (S[r].cpu().numpy(), D[r].cpu().numpy()) for r in range(world)}
        b = h0.cpu().numpy()
        if not backward:  # out = incoming state of this rank, total = the whole sequence's final state
            outs, tot = _fma_chain(parts, b, list(range(world)))
            np.testing.assert_allclose(out.cpu().numpy(), outs[rank], rtol=1e-6, atol=1e-6)
            np.testing.assert_allclose(total.cpu().numpy(), tot, rtol=1e-6, atol=1e-6)
        else:  # out = gradient of this rank's final state: the suffix over the later ranks
            _, g = _fma_chain(parts, b, list(range(world - 1, rank, -1)))
            np.testing.assert_allclose(out.cpu().numpy(), g, rtol=1e-6, atol=1e-6)


def test_p2p_exchange_wait_gives_up(C):
    """Rank 1 never writes its flag: the combine's wait runs out after 200 ms, records device
    error 3 and leaves the output as it was; the context keeps working."""
    shape = (1, 2, 64, 64)
    world = 2
    own, stand_in = _region(C, world, shape), _region(C, world, shape)
    S = torch.randn(*shape, device="cuda")
    D = torch.rand(1, 2, 64, device="cuda")
    out, total = _exchange(C, 0, world, S, D, None, [own, stand_in], own, False, timeout_ms=200)
    assert int(C.lib().tops_gla_device_error()) == 3
    assert torch.isnan(out).all() and torch.isnan(total).all()
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum()) == 56.0
    assert int(C.lib().tops_gla_device_error()) == 0


def test_fused_span_push_matches_the_unfused_span_kernels(C):
    """tops_gla_chunk_{fwd,bwd}_span_begin_p2p push exactly what the unfused span entry points
    return -- forward (S | D), backward (L | D with the forward's D) -- into this rank's slot of
    every region, with its epoch flag; tops_gla_p2p_combine then folds them like p2p_exchange
    (rank 1's part planted, as in the tests above)."""
    from tops.ops.gla import _core
    L = C.lib()
    if not L.tops_gla_has_tcgen05():
        pytest.skip("the span entry points serve the tensor-core path (sm_100)")
    B, T, H, K, V = 1, 2048, 2, 128, 128
    gen = torch.Generator(device="cuda").manual_seed(11)
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device="cuda", generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", generator=gen).to(bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda", generator=gen)) / 16).contiguous()
    do = torch.randn(B, T, H, V, device="cuda", generator=gen).to(bf)
    plan = _core.make_plan(q, V, 64, None, K ** -0.5)
    shape, world, rank = (B, H, K, V), 2, 0
    per = B * H * K * V + B * H * K
    regions = [_region(C, world, shape) for _ in range(world)]
    table = torch.tensor([r.data_ptr() for r in regions], dtype=torch.int64, device="cuda")
    x = C.P2PArgs(rank, world, *shape, 0, None, None, None, None, None, C.ptr(table), regions[rank].data_ptr(), 2000)

    S, D, blk = _core.fwd_span_begin(plan, q, k, v, g)  # unfused reference
    D2, blk2 = _core.fwd_span_begin_p2p(plan, q, k, v, g, x)  # epoch 1: slot parity 1
    torch.cuda.synchronize()
    assert int(L.tops_gla_device_error()) == 0
    assert torch.equal(D2, D)
    for reg in regions:
        assert torch.equal(_slot(reg, world, per, 1, rank), torch.cat([S.reshape(-1), D.reshape(-1)]))
        assert int(_flags(reg)[1, rank]) == 1
    S1 = torch.randn(*shape, device="cuda", generator=gen)
    D1 = torch.rand(B, H, K, device="cuda", generator=gen)
    _plant(regions[rank], world, per, 1, 1, S1, D1, 1)
    out, total = torch.full_like(S, float("nan")), torch.full_like(S, float("nan"))
    a = C.P2PArgs(rank, world, *shape, 0, None, None, None, C.ptr(out), C.ptr(total), C.ptr(table),
                  regions[rank].data_ptr(), 2000)
    C.call("tops_gla_p2p_combine", a, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    parts = {0: (S.cpu().numpy(), D.cpu().numpy()), 1: (S1.cpu().numpy(), D1.cpu().numpy())}
    _, tot = _fma_chain(parts, np.zeros(shape, np.float32), [0, 1])
    assert torch.equal(out, torch.zeros_like(out))  # rank 0's incoming state: no h0
    np.testing.assert_allclose(total.cpu().numpy(), tot, rtol=1e-6, atol=1e-6)

    Lloc, ws = _core.bwd_span_begin(plan, q, k, v, g, do, blk)  # unfused reference
    _core.bwd_span_begin_p2p(plan, q, k, v, g, do, blk2, D, x)  # epoch 2: slot parity 0
    torch.cuda.synchronize()
    assert int(L.tops_gla_device_error()) == 0
    for reg in regions:
        assert torch.equal(_slot(reg, world, per, 0, rank), torch.cat([Lloc.reshape(-1), D.reshape(-1)]))
        assert int(_flags(reg)[0, rank]) == 2
