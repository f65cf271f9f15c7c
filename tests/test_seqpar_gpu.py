"""Sequence parallelism over NCCL (BASELINE config 4's layout) on 2 GPUs: the spans'
outputs, gradients and the final state must equal one GPU running the whole sequence.
Skipped when fewer than 2 GPUs are visible."""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gla():
    sys.path[:0] = [str(ROOT), str(ROOT / "pallas-kernel_b200")]
    import tops.ops.gla as G
    from tops import _C
    _C.lib()
    return G


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(dev):
    gen = torch.Generator(device=dev).manual_seed(5)
    B, T, H, K, V = 1, 8192, 2, 128, 128
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device=dev, generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16
    h0 = torch.randn(B, H, K, V, device=dev, generator=gen)
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    dht = torch.randn(B, H, K, V, device=dev, generator=gen)
    return q, k, v, g.contiguous(), h0, do, dht


def _worker(rank, world, port, out, use_exchange=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path[:0] = [str(ROOT), str(ROOT / "pallas-kernel_b200")]
    import datetime

    import torch.distributed as dist
    from tops import distributed as TD
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", rank)
    q, k, v, g, h0, do, dht = _inputs(dev)
    T = q.shape[1]
    sl = slice(rank * T // world, (rank + 1) * T // world)

    def step(ex):
        qs, ks, vs, gs = (x[:, sl].contiguous().requires_grad_() for x in (q, k, v, g))
        h0r = h0.clone().requires_grad_()
        o, ht = TD.chunk_gla_seq_parallel(qs, ks, vs, gs, initial_state=h0r, chunk_size=64, exchange=ex)
        loss = (o.float() * do[:, sl].float()).sum() + (ht * dht).sum()  # ht and dht are replicated
        loss.backward()
        if ex is not None:  # the bounded host wait returns once the exchanges are done; no peer is lost
            ex.wait(30.0)
            ex.check_peers()
        res = dict(o=o.detach().cpu(), ht=ht.detach().cpu(), dq=qs.grad.cpu(), dk=ks.grad.cpu(), dv=vs.grad.cpu(),
                   dg=gs.grad.cpu())
        if rank == 0:
            res["dh0"] = h0r.grad.cpu()
        return res

    exs = []
    if use_exchange == "nccl":
        exs.append(TD.NcclStateExchange())
    elif use_exchange == "p2p":
        exs.append(TD.P2PStateExchange())
    res = step(exs[0] if exs else None)
    if use_exchange == "p2p":
        # the peer route -- the state pushed by the span kernel that computes it (the default)
        # or by a separate push kernel (fused=False) -- equals the NCCL route bit for bit (the
        # same fold and combine arithmetic); a step's forward and backward exchanges use the two
        # slot parities, and the second fused step reuses both slots
        exs.append(TD.NcclStateExchange())
        ref = step(exs[1])
        again = step(exs[0])
        exs.append(TD.P2PStateExchange(fused=False))
        unfused = step(exs[2])
        res["same_as_nccl"] = all(torch.equal(res[nm], ref[nm]) and torch.equal(again[nm], ref[nm]) and
                                  torch.equal(unfused[nm], ref[nm]) for nm in ref)
    out[rank] = res
    torch.cuda.synchronize()
    for ex in exs:
        ex.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("use_exchange", [None, "nccl", "p2p"],
                         ids=["torch-all-gather", "c-abi-nccl-exchange", "c-abi-peer-memory-exchange"])
def test_seq_parallel_two_gpus_matches_one_gpu(gla, use_exchange):
    world = 2
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out, use_exchange)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=500)
        assert pr.exitcode == 0, "rank failed"
    dev = torch.device("cuda", 0)
    q, k, v, g, h0, do, dht = _inputs(dev)
    qs, ks, vs, gs = (x.clone().requires_grad_() for x in (q, k, v, g))
    h0r = h0.clone().requires_grad_()
    o, ht = gla.chunk_gla(qs, ks, vs, gs, initial_state=h0r, output_final_state=True, chunk_size=64)
    ((o.float() * do.float()).sum() + (ht * dht).sum()).backward()

    def rel(a, b):
        return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-30))

    cat = lambda nm: torch.cat([out[0][nm], out[1][nm]], 1)
    assert rel(cat("o"), o.detach().cpu()) < 1e-2
    for r in range(world):
        assert rel(out[r]["ht"], ht.detach().cpu()) < 1e-2
    for nm, ref in (("dq", qs.grad), ("dk", ks.grad), ("dv", vs.grad), ("dg", gs.grad)):
        assert rel(cat(nm), ref.cpu()) < 2e-2, nm
    assert rel(out[0]["dh0"], h0r.grad.cpu()) < 2e-2
    if use_exchange == "p2p":
        for r in range(world):
            assert out[r]["same_as_nccl"], f"rank {r}: the peer-memory exchange differs from the NCCL one"
