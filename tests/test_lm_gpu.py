"""Config-5 model (GLA blocks + SwiGLU) training step: runs, learns, and its data-parallel
gradients (DDP over NCCL, 2 GPUs) equal the single-GPU gradients of the whole batch."""
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

CFG = dict(vocab_size=512, hidden_size=256, num_layers=2, num_heads=1, intermediate_size=512)


def _model(dtype=torch.bfloat16):
    sys.path[:0] = [str(ROOT), str(ROOT / "pallas-kernel_b200")]
    import tops.layers as L
    torch.manual_seed(0)
    m = L.GLAForCausalLM(L.GLAConfig(**CFG)).cuda()
    m.reset_parameters(torch.Generator(device="cuda").manual_seed(1))
    return L, m.to(dtype)


def _tokens(B, T, seed=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randint(0, CFG["vocab_size"], (B, T), device="cuda", generator=g)


def test_train_steps_reduce_loss():
    L, m = _model()
    opt = L.MasterAdamW(m.parameters(), lr=3e-3, weight_decay=0.0)
    ids = _tokens(4, 256)
    losses = [float(L.train_step(m, opt, ids)) for _ in range(8)]
    assert all(torch.isfinite(torch.tensor(losses)))
    assert losses[-1] < losses[0] - 0.5, losses


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    L, m = _model(torch.float32)
    ddp = torch.nn.parallel.DistributedDataParallel(m, device_ids=[rank])
    ids = _tokens(4, 192)[rank * 2:(rank + 1) * 2]
    loss, _ = ddp(ids, labels=ids)
    loss.backward()
    out[rank] = {n: p.grad.detach().cpu() for n, p in m.named_parameters()}
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ddp_gradients_equal_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=500)
        assert pr.exitcode == 0, "rank failed"
    L, m = _model(torch.float32)
    ids = _tokens(4, 192)
    # the ranks' losses are means over their own half: average of the two halves' grads
    for half in range(2):
        loss, _ = m(ids[half * 2:(half + 1) * 2], labels=ids[half * 2:(half + 1) * 2])
        (loss / 2).backward()
    for n, p in m.named_parameters():
        ref = p.grad.detach().cpu()
        for r in range(world):
            err = float((out[r][n] - ref).norm() / (ref.norm() + 1e-30))
            assert err < 1e-4, (n, r, err)
