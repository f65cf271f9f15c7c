"""Multi-rank logic on CPU ranks (gloo, world sizes 2 and 3): sequence-parallel state
hand-off (with 3 ranks the prefix and suffix chain more than one span) and batch x heads
sharding.  The local compute is the numpy oracle (the
checker); what is tested is the exchange: concatenated rank outputs and gradients
must equal the single-process result."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import cases as GC
from oracle import gla_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(seed=3):
    rng = np.random.default_rng(seed)
    B, T, H, K, V = 2, 96, 2, 8, 12
    q, k = rng.standard_normal((2, B, T, H, K))
    v = rng.standard_normal((B, T, H, V))
    g = GC.logsigmoid(rng.standard_normal((B, T, H, K))) / 4
    h0 = rng.standard_normal((B, H, K, V))
    do = rng.standard_normal((B, T, H, V))
    dht = rng.standard_normal((B, H, K, V))
    return q, k, v, g, h0, do, dht


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "pallas-kernel_b200"), str(root / "tests" / "golden")]
    from tops import distributed as TD
    from oracle import gla_oracle as O2

    dist.init_process_group("gloo", rank=rank, world_size=world)
    q, k, v, g, h0, do, dht = _inputs()
    T = q.shape[1]
    s = slice(rank * T // world, (rank + 1) * T // world)
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x))
    C = 16

    def local_fwd(q_, k_, v_, g_, h_):
        o, ht = O2.chunk_gla(q_.numpy(), k_.numpy(), v_.numpy(), g_.numpy(), initial_state=None if h_ is None else
                             h_.numpy(), output_final_state=True, chunk_size=C)
        return t(o), t(ht)

    def decay(g_):
        return t(np.exp(g_.numpy().sum(1)))  # [B, H, K]

    qs, ks, vs, gs, dos = (t(x[:, s]) for x in (q, k, v, g, do))
    o, H_in, ht = TD.seq_parallel_forward(local_fwd, decay, qs, ks, vs, gs, t(h0))

    def local_bwd(h_in, do_, dht_):
        return tuple(None if x is None else t(x) for x in O2.chunk_gla_bwd(
            qs.numpy(), ks.numpy(), vs.numpy(), gs.numpy(), None, K ** -0.5, h_in.numpy(), None, None, do_.numpy(),
            None if dht_ is None else dht_.numpy(), None, C))

    K = q.shape[-1]
    dq, dk, dv, dg, dh0 = TD.seq_parallel_backward(local_bwd, decay(gs), H_in, dos, t(dht))
    # the two-phase form (begin before the exchange, finish after it) must give the same
    o2, H2, ht2, D2 = TD.seq_parallel_forward_phased(lambda: (local_fwd(qs, ks, vs, gs, None)[1], decay(gs)),
                                                     lambda h_in: local_fwd(qs, ks, vs, gs, h_in)[0], t(h0))
    grads2 = TD.seq_parallel_backward_phased(lambda: local_bwd(H2, dos, None)[-1],
                                             lambda G: local_bwd(H2, dos, G), D2, t(dht))
    phased = dict(o=o2.numpy(), ht=ht2.numpy(), **{nm: x.numpy() for nm, x in zip(("dq", "dk", "dv", "dg", "dh0"),
                                                                                  grads2)})
    # batch sharding: each rank's slice of the batch equals the full run's slice
    ob = None
    if q.shape[0] % world == 0:
        qb, kb, vb, gb = (TD.shard(t(x), rank, world) for x in (q, k, v, g))
        ob, _ = local_fwd(qb, kb, vb, gb, None)
    out[rank] = dict(o=o.numpy(), ht=ht.numpy(), dq=dq.numpy(), dk=dk.numpy(), dv=dv.numpy(), dg=dg.numpy(),
                     dh0=dh0.numpy(), ob=None if ob is None else ob.numpy(), phased=phased)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world", [2, 3])
def test_seq_parallel_and_batch_shard_gloo(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=240)
        assert pr.exitcode == 0, "rank failed"
    q, k, v, g, h0, do, dht = _inputs()
    K = q.shape[-1]
    o_ref, ht_ref = O.chunk_gla(q, k, v, g, initial_state=h0, output_final_state=True, chunk_size=16)
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, h0, None, None, do, dht, None, 16)
    tol = dict(atol=1e-9, rtol=1e-9)
    np.testing.assert_allclose(np.concatenate([out[r]["o"] for r in range(world)], 1), o_ref, **tol)
    for r in range(world):
        np.testing.assert_allclose(out[r]["ht"], ht_ref, **tol)
    for nm, ref in (("dq", dq_r), ("dk", dk_r), ("dv", dv_r), ("dg", dg_r)):
        np.testing.assert_allclose(np.concatenate([out[r][nm] for r in range(world)], 1), ref, **tol)
    np.testing.assert_allclose(out[0]["dh0"], dh0_r, **tol)
    ph = [out[r]["phased"] for r in range(world)]
    np.testing.assert_allclose(np.concatenate([x["o"] for x in ph], 1), o_ref, **tol)
    for nm, ref in (("dq", dq_r), ("dk", dk_r), ("dv", dv_r), ("dg", dg_r)):
        np.testing.assert_allclose(np.concatenate([x[nm] for x in ph], 1), ref, err_msg=f"phased {nm}", **tol)
    for r in range(world):
        np.testing.assert_allclose(ph[r]["ht"], ht_ref, **tol)
    np.testing.assert_allclose(ph[0]["dh0"], dh0_r, **tol)
    if q.shape[0] % world == 0:
        o_nostate, _ = O.chunk_gla(q, k, v, g, chunk_size=16)
        np.testing.assert_allclose(np.concatenate([out[r]["ob"] for r in range(world)], 0), o_nostate, **tol)


def test_prefix_and_suffix_combine_are_linear_maps():
    from tops import distributed as TD
    rng = np.random.default_rng(0)
    S = torch.from_numpy(rng.standard_normal((3, 2, 2, 4, 5)))
    D = torch.from_numpy(rng.uniform(0.1, 1, (3, 2, 2, 4)))
    h0 = torch.from_numpy(rng.standard_normal((2, 2, 4, 5)))
    H = TD.prefix_states(S, D, h0)
    assert torch.allclose(H[0], h0)
    assert torch.allclose(H[2], D[1][..., None] * (D[0][..., None] * h0 + S[0]) + S[1])
    L = torch.from_numpy(rng.standard_normal((3, 2, 2, 4, 5)))
    G = TD.suffix_grads(L, D, None)
    assert torch.allclose(G[2], torch.zeros_like(G[2]))
    assert torch.allclose(G[0], D[1][..., None] * L[2] + L[1])
