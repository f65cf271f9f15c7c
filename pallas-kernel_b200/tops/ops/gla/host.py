"""chunk_gla forward + backward on HOST (pinned) tensors, streamed through the GPU.

No counterpart in the reference (whose arrays live on the accelerator): this is the
entry point for callers that keep activations in host memory (offloaded training,
a host-side framework).  The batch is cut into slices of whole sequences; three CUDA
streams overlap the host->device copy of slice i+1, the fused forward + backward of
slice i on this library's kernels, and the device->host copy of slice i-1's gradients,
so a step costs about the slower PCIe direction instead of the sum of both directions
plus the compute.  ``PinnedGLAPipeline`` keeps its device ring and streams between
calls, so consecutive steps overlap too (step n+1's inputs go in while step n's
gradients come out).  Sequences are independent, so slicing is exact.
"""
from __future__ import annotations

import torch

from . import _core

__all__ = ["chunk_gla_fwd_bwd_pinned", "PinnedGLAPipeline"]


class PinnedGLAPipeline:
    """Reusable copy-in / compute / copy-out pipeline for one problem shape.

    ``submit(q, k, v, g, do, out)`` enqueues one step (host tensors, pinned) and returns
    at once; ``synchronize()`` waits until every submitted step's gradients are in
    ``out``.  Slices of ``slice_batch`` sequences rotate through ``depth`` device slots.
    The default slice is half the batch (rounded up): consecutive steps overlap each other,
    so two slices per step keep both copy directions busy, and fewer, larger copies pay the
    per-copy start cost less often (config 3 on one B200: 11.2 ms per step against 11.6 ms
    with one-sequence slices; both copy directions at once take 10.5 ms).
    """

    def __init__(self, B, T, H, K, V, dtype=torch.bfloat16, scale=None, chunk_size: int = 64,
                 slice_batch: int | None = None, depth: int = 3, device=None):
        self.dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.B, self.T, self.H, self.K, self.V = B, T, H, K, V
        self.dtype = dtype
        self.scale = K ** -0.5 if scale is None else scale
        self.C = chunk_size
        self.sb = max(1, min((B + 1) // 2 if slice_batch is None else slice_batch, B))
        self.depth = max(1, depth)
        sb, dev = self.sb, self.dev
        mk = lambda d, dt: torch.empty(sb, T, H, d, dtype=dt, device=dev)
        self.ins = [[mk(K, dtype), mk(K, dtype), mk(V, dtype), mk(K, torch.float32), mk(V, dtype)]
                    for _ in range(self.depth)]
        self.outs = [[mk(K, dtype), mk(K, dtype), mk(V, dtype), mk(K, torch.float32)] for _ in range(self.depth)]
        self.s_in, self.s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self.s_comp = torch.cuda.Stream(dev)
        self.ev_in = [torch.cuda.Event() for _ in range(self.depth)]
        self.ev_comp = [torch.cuda.Event() for _ in range(self.depth)]
        self.ev_out = [torch.cuda.Event() for _ in range(self.depth)]
        self.used = [False] * self.depth
        self.count = 0  # slices submitted so far
        self.plans = {}

    def _plan(self, qd, n):
        p = self.plans.get(n)
        if p is None:
            p = self.plans[n] = _core.make_plan(qd, self.V, self.C, None, self.scale)
        return p

    def submit(self, q, k, v, g, do, out):
        B = q.shape[0]
        if tuple(q.shape) != (self.B, self.T, self.H, self.K):
            raise ValueError(f"pipeline built for {(self.B, self.T, self.H, self.K)}, got {tuple(q.shape)}")
        dq_h, dk_h, dv_h, dg_h = out
        for b0 in range(0, B, self.sb):
            b1 = min(B, b0 + self.sb)
            n = b1 - b0
            slot = self.count % self.depth
            # host -> device (the slot is free once the compute that last read it is done)
            with torch.cuda.stream(self.s_in):
                if self.used[slot]:
                    self.s_in.wait_event(self.ev_comp[slot])
                dst = [t[:n] for t in self.ins[slot]]
                for d, src in zip(dst, (q, k, v, g, do)):
                    d.copy_(src[b0:b1], non_blocking=True)
                self.ev_in[slot].record(self.s_in)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(self.ev_in[slot])
                if self.used[slot]:
                    self.s_comp.wait_event(self.ev_out[slot])  # its last gradients have left the slot
                qd, kd, vd, gd, dod = dst
                p = self._plan(qd, n)
                o, _, sv = _core.chunk_fwd(p, qd, kd, vd, gd, None, False, save=True)
                ob = [t[:n] for t in self.outs[slot]]
                _core.chunk_bwd(p, qd, kd, vd, gd, None, dod, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"),
                                False, block=sv.get("block"), out=ob)
                self.ev_comp[slot].record(self.s_comp)
            # device -> host
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(self.ev_comp[slot])
                for d, src in zip((dq_h, dk_h, dv_h, dg_h), ob):
                    d[b0:b1].copy_(src, non_blocking=True)
                self.ev_out[slot].record(self.s_out)
            self.used[slot] = True
            self.count += 1
        return out

    def synchronize(self):
        self.s_out.synchronize()
        cur = torch.cuda.current_stream(self.dev)
        cur.wait_stream(self.s_out)


def chunk_gla_fwd_bwd_pinned(q, k, v, g, do, scale=None, chunk_size: int = 64, slice_batch: int = 1,
                             out=None, device=None, depth: int = 3):
    """dq, dk, dv, dg of ``sum(chunk_gla(q, k, v, g)[0] * do)`` for host tensors.

    q, k [B,T,H,K], v, do [B,T,H,V] (bf16/fp32), g [B,T,H,K] fp32 log-space gates, all in
    pinned host memory.  ``out``: optional pinned (dq, dk, dv, dg) to write into.  Returns
    pinned host tensors; on return the copies are complete.  ``slice_batch`` sequences per
    slice; ``depth`` slices in flight on the device.
    """
    if q.is_cuda:
        raise ValueError("chunk_gla_fwd_bwd_pinned takes host tensors; use chunk_gla for device tensors")
    for name, t in (("q", q), ("k", k), ("v", v), ("g", g), ("do", do)):
        if not t.is_pinned():
            raise ValueError(f"{name} must be in pinned host memory")
    B, T, H, K = q.shape
    V = v.shape[-1]
    if out is None:
        out = (torch.empty_like(q).pin_memory(), torch.empty_like(k).pin_memory(), torch.empty_like(v).pin_memory(),
               torch.empty(B, T, H, K, dtype=torch.float32).pin_memory())
    pipe = PinnedGLAPipeline(B, T, H, K, V, q.dtype, scale, chunk_size, slice_batch,
                             min(depth, (B + slice_batch - 1) // max(1, slice_batch)), device)
    pipe.submit(q, k, v, g, do, out)
    pipe.synchronize()
    return out
