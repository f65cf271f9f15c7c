"""chunk_gla forward + backward on HOST (pinned) tensors, streamed through the GPU.

No counterpart in the reference (whose arrays live on the accelerator): this is the
entry point for callers that keep activations in host memory (offloaded training,
a host-side framework).  The batch is cut into slices of whole sequences; three CUDA
streams overlap the host->device copy of slice i+1, the fused forward + backward of
slice i on this library's kernels, and the device->host copy of slice i-1's gradients,
so the step costs about the slower PCIe direction instead of the sum of both
directions plus the compute.  Sequences are independent, so slicing is exact.
"""
from __future__ import annotations

import torch

from . import _core

__all__ = ["chunk_gla_fwd_bwd_pinned"]


class _Ring:
    """`depth` device copies of a set of per-slice buffers."""

    def __init__(self, shapes_dtypes, depth, dev):
        self.bufs = [[torch.empty(s, dtype=d, device=dev) for s, d in shapes_dtypes] for _ in range(depth)]

    def __getitem__(self, i):
        return self.bufs[i % len(self.bufs)]


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
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    if out is None:
        out = (torch.empty_like(q).pin_memory(), torch.empty_like(k).pin_memory(), torch.empty_like(v).pin_memory(),
               torch.empty(B, T, H, K, dtype=torch.float32).pin_memory())
    dq_h, dk_h, dv_h, dg_h = out
    sb = max(1, min(slice_batch, B))
    nsl = (B + sb - 1) // sb
    depth = max(1, min(depth, nsl))
    ins = _Ring([((sb, T, H, K), q.dtype), ((sb, T, H, K), k.dtype), ((sb, T, H, V), v.dtype),
                 ((sb, T, H, K), torch.float32), ((sb, T, H, V), do.dtype)], depth, dev)
    outs = _Ring([((sb, T, H, K), q.dtype), ((sb, T, H, K), k.dtype), ((sb, T, H, V), v.dtype),
                  ((sb, T, H, K), torch.float32)], depth, dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp = torch.cuda.current_stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(nsl)]
    ev_comp = [torch.cuda.Event() for _ in range(nsl)]
    ev_out = [torch.cuda.Event() for _ in range(nsl)]
    plans = {}
    for i in range(nsl):
        b0, b1 = i * sb, min(B, (i + 1) * sb)
        n = b1 - b0
        # host -> device (slot i % depth is free once slice i - depth's compute has read it)
        with torch.cuda.stream(s_in):
            if i >= depth:
                s_in.wait_event(ev_comp[i - depth])
            dst = [t[:n] for t in ins[i]]
            for d, src in zip(dst, (q, k, v, g, do)):
                d.copy_(src[b0:b1], non_blocking=True)
            ev_in[i].record(s_in)
        # compute on the current stream
        s_comp.wait_event(ev_in[i])
        if i >= depth:
            s_comp.wait_event(ev_out[i - depth])  # slice i - depth's gradients have left the ring slot
        qd, kd, vd, gd, dod = dst
        p = plans.get(n)
        if p is None:
            p = plans[n] = _core.make_plan(qd, V, chunk_size, None, scale)
        o, _, sv = _core.chunk_fwd(p, qd, kd, vd, gd, None, False, save=True)
        ob = [t[:n] for t in outs[i]]
        _core.chunk_bwd(p, qd, kd, vd, gd, None, dod, None, sv.get("g_cumsum"), sv.get("A"), sv.get("h"), False,
                        block=sv.get("block"), out=ob)
        ev_comp[i].record(s_comp)
        # device -> host
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[i])
            for d, src in zip((dq_h, dk_h, dv_h, dg_h), ob):
                d[b0:b1].copy_(src, non_blocking=True)
            ev_out[i].record(s_out)
    s_comp.wait_stream(s_out)
    s_out.synchronize()
    return dq_h, dk_h, dv_h, dg_h
