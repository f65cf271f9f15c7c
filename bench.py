#!/usr/bin/env python
"""Benchmark of the GLA hot path on B200 (one JSON line on rank 0).

Headline workload: chunk_gla forward + backward at the
GLA-1.3B layer shape B=8, T=4096, H=4, K=256, V=512, chunk 64, bf16 q/k/v/do,
fp32 gates g = logsigmoid(N(0,1))/16, h0 = 0.  One step = fwd (saving what the
backward needs) + bwd -> dq, dk, dv, dg.  Metric: tokens/s (B*T per step, summed
over ranks).  The same line carries the decode step (
fused_recurrent_gla, B=256, T=1, H=16, K=V=128, fp32 state) in HBM GB/s, and the
long-context step (one sequence of T=131072, H=16, K=V=128; on
N GPUs each rank holds T/N tokens and the span states are exchanged over NCCL) and a
training step of the config-5 model (24 GLA layers + SwiGLU, hidden 2048, vocab 32000,
global batch 16 x 2048 tokens, bf16 weights with fp32-master AdamW, data parallel over
NCCL at N>1).

Multi-GPU (torchrun): every rank runs the same per-GPU workload on its own
batch x heads shard -- the units are independent, so there is no collective on
the data path ("scaling": "weak"); timing is max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Inputs (537 MB per step) exceed the 126 MB L2, so no flush is needed between
steps.  `--impl reference` times the CPU restatement of the reference algorithm
(oracle/, float32 numpy, all host threads) on a bounded sample of the workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "pallas-kernel_b200"))

METRIC = "chunk_gla fwd+bwd tokens/s (1-8 B200), % tensor peak; decode step HBM GB/s"
CFG3 = dict(B=8, T=4096, H=4, K=256, V=512, C=64)
CFG2 = dict(B=256, T=1, H=16, K=128, V=128)
CFG4 = dict(B=1, T=131072, H=16, K=128, V=128, C=64)


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=float(d["hbm_gbs"]), bf16=float(d["bf16_tflops"]),
                    bf16_sustained=float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), source="measured")
    return dict(hbm_gbs=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


# Algorithmic work of each kernel per token per head: (flops, compulsory bytes, extra bytes).
# Flops count dense BT x BT intra-chunk tiles (BT = 128 on the tensor-core path).
# Compulsory bytes are the kernel's share of the op's own inputs and outputs, each read or
# written once (bf16 = 2 B, fp32 = 4 B): q, k, g, v, o in the forward; q, k, g, v, do read
# and dq, dk, dv, dg written in the backward.  Extra bytes are the intermediates the kernels
# exchange through HBM and which a fully fused design would not move: the gated copies
# qhat / kdec, the intra-chunk matrix A and the bf16 chunk states h / dh (K*V per BT tokens).
# The roofline fraction is computed on compulsory bytes only; extra bytes are reported beside it.
def kernel_work(name, K, V, BT=128):
    st = 2 * K * V / BT  # one bf16 chunk state per BT tokens
    gated = 2 * K + 2 * K + 2 * BT  # qhat, kdec, A
    return {
        "tc_prep": (2 * BT * K, 2 * K + 2 * K + 4 * K, gated),
        "tc_scan": (2 * K * V, 2 * V, 2 * K + st),
        "tc_out": (2 * K * V + 2 * BT * V, 2 * V + 2 * V, 2 * K + 2 * BT + st),
        "tc_scan_bwd": (2 * K * V, 2 * V, 2 * K + st),
        "tc_out_dv": (2 * K * V + 2 * BT * V, 2 * V + 2 * V, 2 * K + 2 * BT + st),
        # state scan fused with the output GEMM: v (do) in, o (dv) out; gated copies in, states out
        "tc_scan_out": (4 * K * V + 2 * BT * V, 2 * V + 2 * V, gated + st),
        "tc_scan_out_bwd": (4 * K * V + 2 * BT * V, 2 * V + 2 * V, gated + st),
        # do, v, q, k, g in; dq, dk, dg out; the chunk states h and dh in
        "tc_dqk": (2 * BT * V + 4 * K * V + 4 * BT * K,
                   2 * V + 2 * V + 2 * K + 2 * K + 4 * K + 2 * K + 2 * K + 4 * K, 2 * st),
        "recurrent_decode": (None, None, None),
    }.get(name, (None, None, None))


def fwd_bwd_flops_per_token_head(K, V, C):
    return 12 * K * V + 6 * C * (K + V)


def fwd_bwd_bytes_per_token_head(K, V):
    # fwd: q,k (bf16) v (bf16) g (fp32) read, o (bf16) written;
    # bwd: q,k,v,g,do read; dq,dk,dv (bf16), dg (fp32) written
    fwd = 2 * K + 2 * K + 2 * V + 4 * K + 2 * V
    bwd = 2 * K + 2 * K + 2 * V + 4 * K + 2 * V + 2 * K + 2 * K + 2 * V + 4 * K
    return fwd + bwd


class Clocks:
    """nvidia-smi sampler during the timed region (clocks and throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        self.out = ""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.4)  # let the sampler start before the timed region
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = []
        for line in (self.out or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append(dict(sm=float(f[1]), smax=float(f[2]), power=float(f[3]),
                                 hw=f[5], hwt=f[6], swt=f[7], pcap=f[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        load = [r for r in rows if r["power"] > 200] or rows
        reasons = set()
        for r in load:
            for key, nm in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                            ("pcap", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows)}


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    import torch
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (numpy float32 restatement of the reference algorithm)
# ---------------------------------------------------------------------------

# The reference's own CPU path for this op is its Torch restatement (tests/src/ops/gla/chunk.py:450
# forward, :840 backward), which cannot be shipped to the GPU host with this repository.  Timed on
# one 8-core host on the same sample, it ran 13.8 k tokens/s against 4.6 k for this port.
PORT_NOTE = ("CPU restatement of the reference algorithm (the reference's JAX CPU path needs jax, absent); "
             "the reference's own Torch CPU code ran 2.96x faster than this port on one 8-core host, same sample")


def cpu_sample(seconds_budget: float = 20.0, T: int = 4096):
    """One whole config-3 sequence (all heads) through the oracle's fwd + bwd: ~10 s of CPU work."""
    import numpy as np

    from oracle import gla_oracle as O
    c = CFG3
    rng = np.random.default_rng(0)
    B, H, K, V, C = 1, c["H"], c["K"], c["V"], c["C"]
    q, k = (rng.standard_normal((B, T, H, K), dtype=np.float32) for _ in range(2))
    v = rng.standard_normal((B, T, H, V), dtype=np.float32)
    g = (-np.logaddexp(0, -rng.standard_normal((B, T, H, K))) / 16).astype(np.float32)
    do = rng.standard_normal((B, T, H, V), dtype=np.float32)
    runs = []
    t_end = time.perf_counter() + seconds_budget
    while True:
        t0 = time.perf_counter()
        gc, A, h, _, o = O.chunk_gla_fwd(q, k, v, g, None, K ** -0.5, None, False, None, C, dtype=np.float32)
        O.chunk_gla_bwd(q, k, v, g, gc, K ** -0.5, None, h, A, do, None, None, C, dtype=np.float32)
        runs.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(runs) >= 3:
            break
    dt = statistics.median(runs)
    return {"value": B * T / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"oracle fwd+bwd, numpy float32 (BLAS threads = all host cores), 1 sequence x {T} tokens "
                      f"x H={H} at K={K} V={V} C={C}; median of {len(runs)}",
            "note": PORT_NOTE}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    from oracle import gla_oracle as O
    c = CFG3
    T = c["T"]  # one whole config-3 sequence, all heads: the unit the GPU arm's per-token rate is quoted on
    rng = np.random.default_rng(0)
    H, K, V, C = c["H"], c["K"], c["V"], c["C"]
    q, k = (rng.standard_normal((1, T, H, K), dtype=np.float32) for _ in range(2))
    v = rng.standard_normal((1, T, H, V), dtype=np.float32)
    g = (-np.logaddexp(0, -rng.standard_normal((1, T, H, K))) / 16).astype(np.float32)
    do = rng.standard_normal((1, T, H, V), dtype=np.float32)

    def step():
        gc, A, h, _, o = O.chunk_gla_fwd(q, k, v, g, None, K ** -0.5, None, False, None, C, dtype=np.float32)
        O.chunk_gla_bwd(q, k, v, g, gc, K ** -0.5, None, h, A, do, None, None, C, dtype=np.float32)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    val = T / dt
    sample = (f"oracle (CPU restatement of the reference algorithm), numpy float32, all host threads; "
              f"each step = 1 whole sequence of config 3 ({T} tokens x H={H}, K={K}, V={V}, C={C})")
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "chunk_gla fwd+bwd, config 3 shape (B8 T4096 H4 K256 V512 C64), bounded sample",
                       "sample_tokens_per_step": T},
            "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": sample, "note": PORT_NOTE},
            "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    del world
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def make_inputs(dev, seed):
    import torch
    c = CFG3
    gen = torch.Generator(device=dev).manual_seed(seed)
    B, T, H, K, V = c["B"], c["T"], c["H"], c["K"], c["V"]
    bf = torch.bfloat16
    q = torch.randn(B, T, H, K, device=dev, generator=gen).to(bf)
    k = torch.randn(B, T, H, K, device=dev, generator=gen).to(bf)
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    g = torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    return q, k, v, g.contiguous(), do


def run_ours(args):
    import torch

    from tops import _C
    from tops.ops.gla import _core

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    if args.decode_only:
        dec = decode_bench(args, world, local, dev)
        if rank == 0:
            print(json.dumps({"decode_only": True, **dec}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0
    c = CFG3
    B, T, H, K, V, C = c["B"], c["T"], c["H"], c["K"], c["V"], c["C"]
    q, k, v, g, do = make_inputs(dev, 1234 + rank)
    plan = _core.make_plan(q, V, C, None, K ** -0.5)

    def step():
        o, _, sv = _core.chunk_fwd(plan, q, k, v, g, None, False, save=True)
        return _core.chunk_bwd(plan, q, k, v, g, None, do, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"), False,
                               block=sv.get("block"))

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 3)):
        step()
    barrier(world)
    l0 = _C.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = Clocks(local).__enter__()
    barrier(world)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    barrier(world)
    launches = (_C.launch_count() - l0) // max(args.steps, 1)
    ms = ev0.elapsed_time(ev1) / max(args.steps, 1)
    ms = max_over_ranks(ms, world)
    tokens = B * T * world
    value = tokens / (ms * 1e-3)
    if args.kernels_only:
        clk.__exit__()
        if rank == 0:
            print(json.dumps({"kernels_only": True, "ms_per_step": ms, "tokens_per_s": value, "B": B}), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0

    # per-kernel live timing (CUDA events around each launch on its stream)
    _C.timing_enable(True)
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    _C.timing_enable(False)
    rec = _C.timing_collect()
    per = {}
    for nm, t in rec:
        d = per.setdefault(nm, [0.0, 0])
        d[0] += t
        d[1] += 1
    tot = sum(v_[0] for v_ in per.values()) or 1.0
    dom = max(per.items(), key=lambda kv: kv[1][0])
    dom_name, (dom_total, dom_n) = dom
    dom_ms = dom_total / dom_n
    pk = peaks()
    units = B * T * H
    kernels_share = {nm: round(v_[0] / tot, 4) for nm, v_ in sorted(per.items(), key=lambda kv: -kv[1][0])}
    traffic = None
    tj = ROOT / "profiles" / "traffic.txt"
    if tj.exists():
        for line in tj.read_text().splitlines():
            f_ = line.split()
            if len(f_) >= 2 and not line.startswith("#") and f_[0] == dom_name:
                traffic = float(f_[1])
    ridge = pk["bf16_sustained"] * 1e12 / (pk["hbm_gbs"] * 1e9)
    per_kernel = {}
    for nm, (tt, n) in per.items():
        f, by, ex = kernel_work(nm, K, V)
        if f is None:
            continue
        kms = tt / n
        per_kernel[nm] = {"ms": round(kms, 5), "tflops": round(f * units / (kms * 1e-3) / 1e12, 2),
                          "gbs_compulsory": round(by * units / (kms * 1e-3) / 1e9, 1),
                          "gbs_with_extra": round((by + ex) * units / (kms * 1e-3) / 1e9, 1),
                          "intensity": round(f / by, 1)}
    f, by, ex = kernel_work(dom_name, K, V)
    if f is not None and f / by >= ridge:
        roof = {"kernel": dom_name, "bound": "tensor", "unit": "TFLOP/s", "achieved": f * units / (dom_ms * 1e-3) / 1e12,
                "peak": pk["bf16_sustained"], "peak_source": f"{pk['source']} bf16 sustained (kernel timed inside a step)"}
    elif f is not None:
        roof = {"kernel": dom_name, "bound": "hbm", "unit": "GB/s", "achieved": by * units / (dom_ms * 1e-3) / 1e9,
                "peak": pk["hbm_gbs"], "peak_source": f"{pk['source']} HBM copy bandwidth"}
    else:
        roof = {"kernel": dom_name, "bound": "hbm", "unit": "GB/s", "achieved": None, "peak": pk["hbm_gbs"],
                "peak_source": pk["source"]}
    roof["frac"] = roof["achieved"] / roof["peak"] if roof["achieved"] else None
    alg = None if by is None else by * units
    extra = None if ex is None else ex * units
    roof.update({"traffic": traffic, "traffic_unit": "bytes per launch (ncu dram read+write)",
                 "algorithmic_bytes_per_launch": alg,
                 "algorithmic_bytes_basis": "compulsory: the op's inputs read once and outputs written once",
                 "extra_bytes_per_launch": extra,
                 "extra_bytes_basis": "bf16 chunk states h and dh (and gated copies) exchanged through HBM",
                 "traffic_over_algorithmic": (traffic / alg) if (traffic and alg) else None,
                 "frac_with_extra_bytes": ((by + ex) * units / (dom_ms * 1e-3) / 1e9 / pk["hbm_gbs"])
                 if (by is not None and roof["bound"] == "hbm") else None,
                 "algorithmic_flops_per_launch": None if f is None else f * units,
                 "kernel_ms": dom_ms, "kernel_shares": kernels_share, "per_kernel": per_kernel})
    step_flops = fwd_bwd_flops_per_token_head(K, V, C) * units
    step_bytes = fwd_bwd_bytes_per_token_head(K, V) * units
    step_roof = {"tflops": step_flops / (ms * 1e-3) / 1e12, "tensor_frac": step_flops / (ms * 1e-3) / 1e12 / pk["bf16"],
                 "gbs": step_bytes / (ms * 1e-3) / 1e9, "hbm_frac": step_bytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"],
                 "binding_roof_frac": max(step_flops / (pk["bf16"] * 1e12), step_bytes / (pk["hbm_gbs"] * 1e9))
                 / (ms * 1e-3)}

    # ---- decode step (config 2) -------------------------------------------------
    dec = decode_bench(args, world, local, dev)

    # ---- long context (config 4) ---------------------------------------------------
    lc = long_context_bench(args, world, rank, local, dev)

    # ---- configs 3 and 2 at their stated global sizes split over the ranks (strong) ----
    strong = {}
    if world > 1:
        strong["cfg3"] = strong_cfg3_bench(args, world, rank, dev)
        if CFG2["B"] % world == 0:
            d2 = decode_bench(args, world, local, dev, B=CFG2["B"] // world)
            strong["cfg2"] = {**d2, "scaling": "strong",
                              "metric": "fused_recurrent_gla decode step, global B=256 split over the ranks"}
    else:
        strong["note"] = "at one GPU the strong-scaling legs are the headline (config 3) and decode (config 2)"

    # ---- K = V = 64 heads: tensor-core path next to the CUDA-core kernels ----------------
    h64 = head64_bench(args, world, rank, dev)

    # ---- config-5 model training step (GLA layers + SwiGLU, data parallel) -----------
    torch.cuda.empty_cache()
    lm = None if args.no_model else model_bench(args, world, rank, local, dev)
    torch.cuda.empty_cache()

    # ---- end to end through the public API with host buffers ---------------------
    e2e = e2e_bench(args, world, dev, q, k, v, g, do, plan)
    clk.__exit__()

    clocks = clk.summary()
    if rank == 0:
        cpu = cpu_sample() if world == 1 else None
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "chunk_gla fwd+bwd (BASELINE config 3)", "B_per_gpu": B, "T": T, "H": H,
                           "K": K, "V": V, "chunk_size": C, "global_batch": B * world,
                           "parallelism": f"batch x heads shards, {world} GPU(s), no collective",
                           "l2": "inputs (537 MB/step) larger than L2; no flush"},
                "roofline": roof, "step_roofline": step_roof, "decode": dec, "long_context": lc,
                "strong_scaling": strong, "head64": h64, "model_dp": lm,
                "e2e": e2e,
                "gpu_launches": int(launches), "clocks": clocks, "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def decode_bench(args, world, local, dev, B=None):
    import torch

    from tops.ops.gla import _core
    c = CFG2
    B, T, H, K, V = c["B"] if B is None else B, c["T"], c["H"], c["K"], c["V"]
    gen = torch.Generator(device=dev).manual_seed(7)
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device=dev, generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    gk = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16).contiguous()
    h0 = torch.randn(B, H, K, V, device=dev, generator=gen) * 0.1
    scale = K ** -0.5

    def step():
        return _core.recurrent_fwd(q, k, v, gk, None, h0, scale, True, False, None, B)

    for _ in range(5):
        step()
    steps = max(args.steps, 20)

    def timed(run):
        barrier(world)
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        run()
        e1.record(s)
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1) / steps, world)

    def eager():  # each step's outputs are dropped at once, so the allocator reuses them
        for _ in range(steps):
            step()

    eager_ms = timed(eager)
    # a serving loop replays its decode steps as a CUDA graph (no launch gaps between steps)
    graph = None
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(steps):
                step()
        graph.replay()
        torch.cuda.synchronize(dev)
    except Exception:  # capture unavailable: report the eager loop
        graph = None
    # every rank times two loops (the same barriers on every rank, whatever capture did)
    ms = timed(graph.replay if graph is not None else eager)
    nbytes = 2 * B * H * K * V * 4 + B * T * H * (2 * K * 2 + 2 * V + 4 * K + 4 * V)
    pk = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"metric": "fused_recurrent_gla decode step HBM GB/s (BASELINE config 2)", "value": gbs * world,
            "unit": "GB/s", "per_gpu_gbs": gbs, "us_per_step": ms * 1e3, "bytes_per_step": nbytes,
            "timing": "CUDA graph of the timed steps" if graph is not None else "eager launches",
            "eager_us_per_step": eager_ms * 1e3,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / pk["hbm_gbs"], "peak_source": pk["source"], "kernel": "recurrent_fwd"},
            "config": {"B": B, "T": T, "H": H, "K": K, "V": V, "state": "fp32", "inputs": "bf16 q/k/v, fp32 gk"}}


def long_context_bench(args, world, rank, local, dev):
    """Config 4: chunk_gla fwd+bwd over one long sequence.  1 GPU: the whole sequence (state
    scans split into parallel spans).  N GPUs: rank r holds tokens [r T/N, (r+1) T/N) and runs
    tops.distributed.chunk_gla_seq_parallel with the C ABI's NCCL state exchange: the forward's
    first phase (gating, zero-state span scans) yields the span's (final state, decay), one
    all-gather + prefix gives its incoming state, the second phase finishes the scan and the
    output; the backward does the same with the span's dh0."""
    import torch

    from tops.ops.gla import _core
    c = CFG4
    B, T, H, K, V, C = c["B"], c["T"], c["H"], c["K"], c["V"], c["C"]
    Tr = T // world
    gen = torch.Generator(device=dev).manual_seed(21 + rank)
    bf = torch.bfloat16
    q, k = (torch.randn(B, Tr, H, K, device=dev, generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, Tr, H, V, device=dev, generator=gen).to(bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, Tr, H, K, device=dev, generator=gen)) / 16).contiguous()
    do = torch.randn(B, Tr, H, V, device=dev, generator=gen).to(bf)
    plan = _core.make_plan(q, V, C, None, K ** -0.5)

    if world == 1:
        def step():
            o, _, sv = _core.chunk_fwd(plan, q, k, v, g, None, False, save=True)
            return _core.chunk_bwd(plan, q, k, v, g, None, do, None, block=sv.get("block"))
    else:
        from tops import distributed as TD
        for x in (q, k, v, g):
            x.requires_grad_()

        def step_with(ex):
            def step():
                o, _ = TD.chunk_gla_seq_parallel(q, k, v, g, chunk_size=C, exchange=ex)
                return torch.autograd.grad(o, (q, k, v, g), do)
            return step

    steps = max(3, min(args.steps, 5))

    def timed(run):
        barrier(world)
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            run()
        e1.record(s)
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1) / steps, world)

    def measure(step):
        """-> (ms per step, eager ms per step, per-launch ms of one eager step, graph used)."""
        for _ in range(3):
            step()
        ms = eager_ms = timed(step)
        # per-launch device times of one eager step (rank 0's), after the timed region
        from tops import _C
        _C.timing_enable(True)
        step()
        torch.cuda.synchronize()
        _C.timing_enable(False)
        kern = {}
        for nm, t in _C.timing_collect():
            kern[nm] = round(kern.get(nm, 0.0) + t, 4)
        graph_used = False
        if world > 1:
            # A training loop replays a step this small (a rank's span is 1/N of the sequence)
            # as a CUDA graph, so the host's launch and autograd work stops adding to the step.
            # The graph holds the same kernels and exchanges; every rank replays only if every
            # rank captured (the exchanges must pair up), and the graph is released before the
            # exchange and the process group.
            import torch.distributed as dist
            graph, ok = None, 1
            try:
                side = torch.cuda.Stream(dev)
                side.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(side):
                    for _ in range(2):
                        step()
                torch.cuda.current_stream(dev).wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    step()
                graph.replay()
                torch.cuda.synchronize(dev)
            except Exception:
                graph, ok = None, 0
            flag = torch.tensor([ok], device=dev, dtype=torch.int32)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()) == 1:
                ms = timed(graph.replay)
                graph_used = True
            del graph
            torch.cuda.synchronize()
        return ms, eager_ms, kern, graph_used

    route, nccl_route, p2p_unfused_route = "none (1 GPU)", None, None
    if world == 1:
        ms, eager_ms, kern, graph_used = measure(step)
    else:
        # the product route: the state exchange through peer memory (two kernels, NVLink
        # stores); the C ABI's NCCL all-gather route is timed the same way beside it
        ex = None
        try:  # construction and region setup are collective and fail on every rank together
            ex = TD.P2PStateExchange()
            ex.prepare((B, H, K, V))
            route = "peer memory (tops_gla_p2p_exchange)"
        except (ValueError, RuntimeError):
            if ex is not None:
                ex.close()
            ex = TD.NcclStateExchange()
            route = "NCCL all-gather (tops_gla_state_exchange)"
        ms, eager_ms, kern, graph_used = measure(step_with(ex))
        ex.close()
        if isinstance(ex, TD.P2PStateExchange):
            route = "peer memory, pushed by the span kernel that computes the state (tops_gla_chunk_*_span_begin_p2p)"

            def other(make):
                e2 = make()
                o_ms, o_eager, o_kern, o_graph = measure(step_with(e2))
                e2.close()
                return {"ms_per_step": o_ms, "eager_ms_per_step": o_eager,
                        "timing": "CUDA graph of one step, replayed" if o_graph else "eager launches",
                        "exchange_kernel_ms": {k_: v_ for k_, v_ in o_kern.items() if k_.startswith("exchange")}}
            p2p_unfused_route = other(lambda: TD.P2PStateExchange(fused=False))
            nccl_route = other(TD.NcclStateExchange)
    del q, k, v, g, do
    return {"metric": "chunk_gla fwd+bwd tokens/s, long context (BASELINE config 4)", "value": B * T / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "scaling": "strong",
            "timing": "CUDA graph of one step, replayed" if graph_used else "eager launches",
            "eager_ms_per_step": eager_ms, "kernel_ms": kern, "kernel_ms_sum": round(sum(kern.values()), 4),
            "exchange": route, "p2p_unfused_route": p2p_unfused_route, "nccl_route": nccl_route,
            "config": {"B": B, "T": T, "H": H, "K": K, "V": V, "chunk_size": C, "T_per_gpu": Tr,
                       "parallelism": "1 GPU (state scans in parallel spans)" if world == 1 else
                       f"sequence spans over {world} GPUs, two-phase span fwd/bwd, one exchange of "
                       "(state, decay) per direction"}}


def strong_cfg3_bench(args, world, rank, dev):
    """Config 3 at its stated global size, B = 8 sequences split over the ranks (strong
    scaling: B/N sequences per GPU, no collective).  At N = 8 a GPU holds one sequence (16
    (head, V-tile) scan units), so the state scans run in parallel spans."""
    import torch

    from tops.ops.gla import _core
    c = CFG3
    Bg, T, H, K, V, C = 8, c["T"], c["H"], c["K"], c["V"], c["C"]
    if Bg % world:
        return None
    B = Bg // world
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device=dev, generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16).contiguous()
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    plan = _core.make_plan(q, V, C, None, K ** -0.5)

    def step():
        o, _, sv = _core.chunk_fwd(plan, q, k, v, g, None, False, save=True)
        return _core.chunk_bwd(plan, q, k, v, g, None, do, None, block=sv.get("block"))

    for _ in range(3):
        step()
    steps = max(5, args.steps)
    barrier(world)
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        step()
    e1.record(s)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    return {"metric": "chunk_gla fwd+bwd tokens/s, config 3 at its global size (strong scaling)",
            "value": Bg * T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "scaling": "strong", "config": {"global_batch": Bg, "B_per_gpu": B, "T": T, "H": H, "K": K, "V": V,
                                            "chunk_size": C, "inputs_bytes_per_gpu": B * T * H * (6 * K + 4 * V)}}


def head64_bench(args, world, rank, dev):
    """K = V = 64 heads (the size the reference's tests use, which it pads to 128) on the
    tensor-core path, timed next to the CUDA-core kernels on the same inputs: chunk_gla fwd+bwd,
    B=4, T=4096, H=16, bf16.  The CUDA-core path is selected through the same C ABI by asking
    for the sub-function intermediates (g_cumsum, A, h), which only it returns."""
    import torch

    from tops import _C
    from tops.ops.gla import _core
    B, T, H, K, V, C = 4, 4096, 16, 64, 64, 64
    gen = torch.Generator(device=dev).manual_seed(64 + rank)
    bf = torch.bfloat16
    q, k = (torch.randn(B, T, H, K, device=dev, generator=gen).to(bf) for _ in range(2))
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16).contiguous()
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    plan = _core.make_plan(q, V, C, None, K ** -0.5)
    assert _core.saved_size(plan, g) > 0

    def tc_step():
        o, _, sv = _core.chunk_fwd(plan, q, k, v, g, None, False, save=True)
        return _core.chunk_bwd(plan, q, k, v, g, None, do, None, block=sv.get("block"))

    gc = torch.empty(B, T, H, K, dtype=torch.float32, device=dev)
    A = torch.empty(B, T, H, C, dtype=torch.float32, device=dev)
    h = torch.empty(plan.NT, H, K, V, dtype=torch.float32, device=dev)
    o = torch.empty(B, T, H, V, dtype=bf, device=dev)
    fa = _C.ChunkFwdArgs(plan.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), None, _C.ptr(o), None,
                         _C.ptr(gc), _C.ptr(A), _C.ptr(h), None, 0, None, 0)
    fws = torch.empty(max(int(_C.lib().tops_gla_chunk_fwd_workspace_size(fa)), 1), dtype=torch.uint8, device=dev)
    fa.workspace, fa.workspace_bytes = _C.ptr(fws), fws.numel()
    grads = [torch.empty_like(x) for x in (q, k, v)] + [torch.empty_like(g)]
    ba = _C.ChunkBwdArgs(plan.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), None, _C.ptr(do), None,
                         _C.ptr(gc), _C.ptr(A), _C.ptr(h), *(_C.ptr(x) for x in grads), None, None, 0, None, 0)
    bws = torch.empty(max(int(_C.lib().tops_gla_chunk_bwd_workspace_size(ba)), 1), dtype=torch.uint8, device=dev)
    ba.workspace, ba.workspace_bytes = _C.ptr(bws), bws.numel()

    def simt_step():
        st = _C.stream_of(q)
        _C.call("tops_gla_chunk_fwd", fa, st)
        _C.call("tops_gla_chunk_bwd", ba, st)

    out = {}
    for name, fn in (("tensor_core", tc_step), ("cuda_core", simt_step)):
        for _ in range(3):
            fn()
        steps = max(3, min(args.steps, 10))
        barrier(world)
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(steps):
            fn()
        e1.record(s)
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
        out[name] = {"ms_per_step": ms, "tokens_per_s": B * T * world / (ms * 1e-3)}
    out["speedup_tensor_core"] = out["cuda_core"]["ms_per_step"] / out["tensor_core"]["ms_per_step"]
    out["config"] = {"B_per_gpu": B, "T": T, "H": H, "K": K, "V": V, "chunk_size": C, "dtype": "bf16",
                     "workload": "chunk_gla fwd+bwd at K = V = 64"}
    return out


def op_only(args):
    """One small case of a named op, run a few times: the command the per-kernel ncu summaries
    of the kernels outside the config-3 step (recurrence backward, CUDA-core chunk kernels,
    layer kernels) are taken from."""
    import torch

    from tops.ops.gla import _core
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    gen = torch.Generator(device=dev).manual_seed(9)
    bf = torch.bfloat16
    # sizes: each case's tensors exceed the 126 MB L2 and stay a few hundred MB in all
    if args.op == "recurrent_bwd":  # BASELINE config 2's head shape over T = 64 steps, B = 64
        B, T, H, K, V = 64, 64, 16, 128, 128
        q, k = (torch.randn(B, T, H, K, device=dev, generator=gen).to(bf) for _ in range(2))
        v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
        gk = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16).contiguous()
        h0 = torch.randn(B, H, K, V, device=dev, generator=gen) * 0.1
        do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)  # the C ABI reads do in q's dtype
        o, _ = _core.recurrent_fwd(q, k, v, gk, None, h0, K ** -0.5, False, False, None, B)

        def run():
            return _core.recurrent_bwd(q, k, v, gk, None, h0, o, do, None, K ** -0.5, False, None, B)
    elif args.op == "simt_chunk":  # fp32 chunk_gla fwd+bwd (CUDA-core kernels), config-1 layout scaled up
        B, T, H, K, V, C = 8, 4096, 4, 64, 64, 64
        q, k = (torch.randn(B, T, H, K, device=dev, generator=gen) for _ in range(2))
        v = torch.randn(B, T, H, V, device=dev, generator=gen)
        g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device=dev, generator=gen)) / 16).contiguous()
        do = torch.randn(B, T, H, V, device=dev, generator=gen)
        plan = _core.make_plan(q, V, C, None, K ** -0.5)

        def run():
            o, _, sv = _core.chunk_fwd(plan, q, k, v, g, None, False, save=True)
            return _core.chunk_bwd(plan, q, k, v, g, None, do, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"))
    elif args.op == "layer":  # the GLA layer's fused kernels: gate logsigmoid and RMSNorm x swish gate
        import tops.layers as L
        cfg = L.GLAConfig()
        with torch.device(dev):
            layer = L.GatedLinearAttention(hidden_size=cfg.hidden_size, num_heads=cfg.num_heads, expand_k=0.5,
                                           expand_v=1.0, mode="chunk", layer_idx=0).to(bf)
        x = torch.randn(4, 2048, cfg.hidden_size, device=dev, generator=gen).to(bf).requires_grad_()

        def run():
            y = layer(x)[0]
            y.float().sum().backward()
    else:
        raise SystemExit(f"unknown --op {args.op}")
    for _ in range(max(args.steps, 1)):
        run()
    torch.cuda.synchronize()
    print(json.dumps({"op": args.op, "ok": True}), flush=True)
    return 0


def model_bench(args, world, rank, local, dev):
    """Config 5: one training step (forward, next-token loss, backward, gradient all-reduce
    when N>1, fp32-master AdamW) of the 24-layer GLA + SwiGLU model on synthetic tokens
    U[0, vocab); global batch 16 x 2048 split over the ranks."""
    import torch

    import tops.layers as L
    cfg = L.GLAConfig()
    B, T = max(1, 16 // world), 2048
    with torch.device(dev):
        model = L.GLAForCausalLM(cfg)
    model.reset_parameters(torch.Generator(device=dev).manual_seed(5))
    model = model.to(torch.bfloat16)
    n_params = sum(p.numel() for p in model.parameters())
    opt = L.MasterAdamW(model.parameters())
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local], bucket_cap_mb=100)
    gen = torch.Generator(device=dev).manual_seed(31 + rank)
    ids = torch.randint(0, cfg.vocab_size, (B, T), device=dev, generator=gen)
    for _ in range(2):
        L.train_step(net, opt, ids)
    steps = max(2, min(args.steps, 3))
    barrier(world)
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        loss = L.train_step(net, opt, ids)
    e1.record(s)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    tokens = B * T * world
    K, V, H = int(cfg.hidden_size * cfg.expand_k) // cfg.num_heads, int(cfg.hidden_size * cfg.expand_v) // cfg.num_heads, cfg.num_heads
    flops = 6 * n_params * tokens + cfg.num_layers * fwd_bwd_flops_per_token_head(K, V, 64) * H * tokens
    pk = peaks()
    out = {"metric": "GLA LM training tokens/s (BASELINE config 5)", "value": tokens / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms, "steps": steps, "scaling": "strong", "loss": float(loss),
           "params": n_params, "model_tflops": flops / (ms * 1e-3) / 1e12,
           "tensor_frac": flops / (ms * 1e-3) / 1e12 / pk["bf16_sustained"],
           "config": {"layers": cfg.num_layers, "hidden": cfg.hidden_size, "heads": H, "K": K, "V": V,
                      "mlp": cfg.intermediate_size, "vocab": cfg.vocab_size, "global_batch": B * world, "T": T,
                      "dtype": "bf16 weights/activations, fp32 master AdamW",
                      "parallelism": "1 GPU" if world == 1 else f"data parallel x{world} (DDP all-reduce, NCCL)"}}
    del net, model, opt, ids
    return out


def e2e_bench(args, world, dev, q, k, v, g, do, plan):
    """Public API with HOST buffers: ``tops.ops.gla.PinnedGLAPipeline`` copies q, k, v, g, do
    in from pinned memory and dq, dk, dv, dg back out every step, one sequence slice at a
    time on three streams (copy-in, compute, copy-out overlap, also across steps); the
    timed region ends when the last step's gradients are in host memory."""
    import torch

    from tops.ops.gla import PinnedGLAPipeline
    hq, hk, hv, hg, hdo = (x.cpu().pin_memory() for x in (q, k, v, g, do))
    outs = tuple(torch.empty(x.shape, dtype=x.dtype).pin_memory() for x in (q, k, v, g))
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hg, hdo))
    d2h = sum(x.numel() * x.element_size() for x in outs)
    pipe = PinnedGLAPipeline(plan.B, plan.T, plan.H, plan.K, plan.V, q.dtype, plan.scale, plan.C, device=dev)

    for _ in range(2):
        pipe.submit(hq, hk, hv, hg, hdo, outs)
    pipe.synchronize()
    steps = max(3, min(args.steps, 10))
    barrier(world)
    s = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(steps):
        pipe.submit(hq, hk, hv, hg, hdo, outs)
    pipe.synchronize()  # the current stream now waits for the last copy-out
    e1.record(s)
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    tokens = plan.B * plan.T * world
    return {"value": tokens / (ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "path": "tops.ops.gla.PinnedGLAPipeline (C ABI chunk fwd+bwd per sequence slice; "
            "pinned host inputs/outputs; copy-in / compute / copy-out on three streams, overlapped across steps)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=None, help="override B per GPU (profiling runs on a smaller case)")
    ap.add_argument("--no-model", action="store_true", help="skip the config-5 model training leg")
    ap.add_argument("--decode-only", action="store_true", help="only the config-2 decode leg (for ncu captures)")
    ap.add_argument("--kernels-only", action="store_true",
                    help="only the timed fwd+bwd loop (no decode / e2e / CPU legs); for ncu launch lists")
    ap.add_argument("--op", choices=("recurrent_bwd", "simt_chunk", "layer"), default=None,
                    help="run only a small case of one op --steps times (for ncu captures of its kernels)")
    args = ap.parse_args()
    if args.batch is not None:
        CFG3["B"] = int(args.batch)
    if args.impl == "reference":
        return run_reference(args)
    if args.op is not None:
        return op_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
