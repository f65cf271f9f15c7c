"""The peer-memory state exchange (tops_gla_p2p_exchange) on one GPU.

Rank 0 of a two-rank group runs the real entry point.  Rank 1's part -- its packed
(state | decay) in its slot of rank 0's region and its epoch flag -- is written into the
region beforehand, as rank 1's push would have left it, so no kernel here waits for another
launch.  The regions are plain device tensors (one process, no IPC); the second one stands in
for rank 1's region, which rank 0's push also writes.  Checked: the forward prefix and total
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


@pytest.mark.parametrize("shape", [(1, 4, 128, 128), (1, 3, 63, 96)], ids=["vec", "scalar"])
def test_p2p_exchange_two_ranks_emulated(C, shape):
    N, H, K, V = shape
    world, per = 2, N * H * K * V + N * H * K
    gen = torch.Generator(device="cuda").manual_seed(3)
    own, stand_in = _region(C, world, shape), _region(C, world, shape)
    h0 = torch.randn(*shape, device="cuda", generator=gen)
    for e in (1, 2, 3):  # three exchanges: slot parities 1, 0, 1
        par = e & 1
        assert _epoch(own) == e - 1
        S = [torch.randn(*shape, device="cuda", generator=gen) for _ in range(world)]
        D = [torch.rand(N, H, K, device="cuda", generator=gen) for _ in range(world)]
        _plant(own, world, per, par, 1, S[1], D[1], e)
        backward = e == 2
        out, total = _exchange(C, 0, world, S[0], D[0], h0, [own, stand_in], own, backward)
        assert int(C.lib().tops_gla_device_error()) == 0
        # rank 0's own slot and flag went into both regions
        for reg in (own, stand_in):
            got = _slot(reg, world, per, par, 0)
            assert torch.equal(got, torch.cat([S[0].reshape(-1), D[0].reshape(-1)]))
            assert int(_flags(reg)[par, 0]) == e
        parts = {r: (S[r].double().cpu().numpy().astype(np.float32), D[r].cpu().numpy()) for r in range(world)}
        b = h0.cpu().numpy()
        if not backward:  # out = incoming state of rank 0 (= h0), total = D1 (D0 h0 + S0) + S1
            outs, tot = _fma_chain(parts, b, [0, 1])
            np.testing.assert_allclose(out.cpu().numpy(), outs[0], rtol=0, atol=0)
            np.testing.assert_allclose(total.cpu().numpy(), tot, rtol=1e-6, atol=1e-6)
        else:  # out = gradient of rank 0's final state: D1 * dht + L1
            _, g = _fma_chain(parts, b, [1])
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
