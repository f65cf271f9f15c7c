"""Tensor-level wrappers of the libtops_gla C ABI (torch CUDA tensors in, out).

Everything here is plumbing: shape checks, output allocation, the varlen chunk
map (computed on the host exactly like the reference's ``prepare_chunk_indices``,
``tops/utils.py:70-89``) and one C call per operation on the current CUDA stream.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ... import _C


def _cuda(name: str, t: torch.Tensor | None) -> torch.Tensor | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the GLA ops run only on the GPU), got {t.device}")
    return t.contiguous()


def _f32(name: str, t: torch.Tensor | None) -> torch.Tensor | None:
    t = _cuda(name, t)
    return None if t is None else t.float().contiguous()


@dataclass
class Plan:
    """Problem geometry shared by the chunked entry points."""
    B: int
    T: int
    H: int
    K: int
    V: int
    N: int
    NT: int
    C: int
    dtype: torch.dtype
    scale: float
    cu_host: list | None
    cu_dev: torch.Tensor | None
    offs_dev: torch.Tensor | None

    def shape(self) -> _C.Shape:
        return _C.Shape(self.B, self.T, self.H, self.K, self.V, self.N, self.NT, self.C, _C.dtype_code(self.dtype),
                        float(self.scale), _C.ptr(self.cu_dev), _C.ptr(self.offs_dev))

    @property
    def nchunk_per_seq(self) -> int:
        return (self.T + self.C - 1) // self.C


def host_cu(cu_seqlens) -> list | None:
    if cu_seqlens is None:
        return None
    if isinstance(cu_seqlens, torch.Tensor):
        return [int(x) for x in cu_seqlens.detach().cpu().tolist()]
    return [int(x) for x in cu_seqlens]


def make_plan(q: torch.Tensor, V: int, chunk_size: int, cu_seqlens, scale: float | None) -> Plan:
    B, T, H, K = q.shape
    C = int(chunk_size)
    assert C > 0 and (C & (C - 1)) == 0, f"chunk_size must be a power of 2, got {C}"
    cu = host_cu(cu_seqlens)
    if cu is None:
        N, NT, cu_dev, offs_dev = B, B * ((T + C - 1) // C), None, None
    else:
        assert B == 1, f"Batch size must be 1 when using cu_seqlens, got {B}"
        assert len(cu) >= 2 and cu[0] == 0 and cu[-1] == T, f"cu_seqlens must run from 0 to T={T}, got {cu}"
        assert all(b >= a for a, b in zip(cu, cu[1:])), "cu_seqlens must be non-decreasing"
        N = len(cu) - 1
        offs = [0]
        for a, b in zip(cu, cu[1:]):
            offs.append(offs[-1] + (b - a + C - 1) // C)
        NT = offs[-1]
        cu_dev = torch.tensor(cu, dtype=torch.int32, device=q.device)
        offs_dev = torch.tensor(offs, dtype=torch.int32, device=q.device)
    if scale is None:
        scale = K ** -0.5
    return Plan(B, T, H, K, V, N, NT, C, q.dtype, float(scale), cu, cu_dev, offs_dev)


def _ws(nbytes: int, dev) -> torch.Tensor | None:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev) if nbytes else None


# ---------------------------------------------------------------------------
# fused forward / backward
# ---------------------------------------------------------------------------

def saved_size(p: Plan, g) -> int:
    """Bytes of the tensor-core path's saved block (0 when the problem runs on CUDA cores).
    Ungated problems (g None) take the tensor-core path too: the library substitutes zero gates."""
    s = p.shape()
    return int(_C.lib().tops_gla_chunk_saved_size(s))


def chunk_fwd(p: Plan, q, k, v, g, h0, output_final_state: bool, save: bool):
    """-> o, ht|None, saved; saved = {"block": uint8 tensor} (tensor-core path) or
    {"g_cumsum", "A", "h"} (CUDA-core path) when ``save`` else None."""
    dev = q.device
    o = torch.empty(p.B, p.T, p.H, p.V, dtype=q.dtype, device=dev)
    ht = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev) if output_final_state else None
    gc = A = h = blk = None
    nblk = saved_size(p, g)
    if save and nblk:
        blk = torch.empty(nblk, dtype=torch.uint8, device=dev)
    elif save:
        gc = torch.empty(p.B, p.T, p.H, p.K, dtype=torch.float32, device=dev)
        A = torch.empty(p.B, p.T, p.H, p.C, dtype=torch.float32, device=dev)
        h = torch.empty(p.NT, p.H, p.K, p.V, dtype=torch.float32, device=dev)
    a = _C.ChunkFwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(o), _C.ptr(ht),
                        _C.ptr(gc), _C.ptr(A), _C.ptr(h), None, 0, _C.ptr(blk), 0 if blk is None else blk.numel())
    ws = _ws(_C.lib().tops_gla_chunk_fwd_workspace_size(a), dev)
    a.workspace, a.workspace_bytes = _C.ptr(ws), (ws.numel() if ws is not None else 0)
    _C.call("tops_gla_chunk_fwd", a, _C.stream_of(q))
    if not save:
        return o, ht, None
    return o, ht, ({"block": blk} if blk is not None else {"g_cumsum": gc, "A": A, "h": h})


def chunk_bwd(p: Plan, q, k, v, g, h0, do, dht, gc=None, A=None, h=None, want_dh0: bool = False, block=None,
              out=None):
    """-> dq, dk, dv, dg, dh0|None; ``out`` = preallocated (dq, dk, dv, dg) to write into."""
    dev = q.device
    if out is not None:
        dq, dk, dv, dg = out
    else:
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        dg = torch.empty(p.B, p.T, p.H, p.K, dtype=torch.float32, device=dev)
    dh0 = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev) if want_dh0 else None
    a = _C.ChunkBwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(do), _C.ptr(dht),
                        _C.ptr(gc), _C.ptr(A), _C.ptr(h), _C.ptr(dq), _C.ptr(dk), _C.ptr(dv), _C.ptr(dg),
                        _C.ptr(dh0), None, 0, _C.ptr(block), 0 if block is None else block.numel())
    ws = _ws(_C.lib().tops_gla_chunk_bwd_workspace_size(a), dev)
    a.workspace, a.workspace_bytes = _C.ptr(ws), (ws.numel() if ws is not None else 0)
    _C.call("tops_gla_chunk_bwd", a, _C.stream_of(q))
    return dq, dk, dv, dg, dh0


def final_state(p: Plan, q, k, v, g, h0):
    """Final state only (the state scan without the output GEMM): the first pass of a
    sequence-parallel forward.  -> [N, H, K, V] fp32."""
    dev = q.device
    ht = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev)
    a = _C.ChunkFwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), None, _C.ptr(ht),
                        None, None, None, None, 0, None, 0)
    ws = _ws(_C.lib().tops_gla_chunk_fwd_workspace_size(a), dev)
    a.workspace, a.workspace_bytes = _C.ptr(ws), (ws.numel() if ws is not None else 0)
    _C.call("tops_gla_chunk_fwd", a, _C.stream_of(q))
    return ht


def initial_state_grad(p: Plan, q, k, v, g, h0, do, dht, block=None):
    """dL/dh0 only (the reverse state scan): the first pass of a sequence-parallel
    backward.  ``block`` is the forward's saved block when it ran on the tensor-core path."""
    dev = q.device
    dh0 = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev)
    a = _C.ChunkBwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(do), _C.ptr(dht),
                        None, None, None, None, None, None, None, _C.ptr(dh0), None, 0, _C.ptr(block),
                        0 if block is None else block.numel())
    ws = _ws(_C.lib().tops_gla_chunk_bwd_workspace_size(a), dev)
    a.workspace, a.workspace_bytes = _C.ptr(ws), (ws.numel() if ws is not None else 0)
    _C.call("tops_gla_chunk_bwd", a, _C.stream_of(q))
    return dh0


# ---------------------------------------------------------------------------
# two-phase span forward / backward (one rank's span of a sequence-parallel problem)
# ---------------------------------------------------------------------------

def span_saved_size(p: Plan, g) -> int:
    """Bytes of the saved block of the two-phase span entry points (0: not served, i.e. the
    problem does not run on the tensor-core path or is variable-length)."""
    if g is None or p.cu_dev is not None:
        return 0
    return int(_C.lib().tops_gla_chunk_span_saved_size(p.shape()))


def fwd_span_begin(p: Plan, q, k, v, g):
    """Phase 1 of a span's forward -> (local_state [N,H,K,V] from a zero state, decay [N,H,K],
    saved block)."""
    dev = q.device
    blk = torch.empty(span_saved_size(p, g), dtype=torch.uint8, device=dev)
    S = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev)
    D = torch.empty(p.N, p.H, p.K, dtype=torch.float32, device=dev)
    a = _C.ChunkFwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), None, None, None,
                        None, None, None, None, 0, _C.ptr(blk), blk.numel())
    _C.call("tops_gla_chunk_fwd_span_begin", a, _C.ptr(S), _C.ptr(D), _C.stream_of(q))
    return S, D, blk


def fwd_span_begin_p2p(p: Plan, q, k, v, g, x):
    """Phase 1 with the state exchange's push fused into the kernel that computes the span's
    state (``x``: a ``_C.P2PArgs`` naming the group's peer regions) -> (decay [N,H,K], saved
    block).  The state itself goes only to the regions."""
    dev = q.device
    blk = torch.empty(span_saved_size(p, g), dtype=torch.uint8, device=dev)
    D = torch.empty(p.N, p.H, p.K, dtype=torch.float32, device=dev)
    a = _C.ChunkFwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), None, None, None,
                        None, None, None, None, 0, _C.ptr(blk), blk.numel())
    _C.call("tops_gla_chunk_fwd_span_begin_p2p", a, _C.ptr(D), x, _C.stream_of(q))
    return D, blk


def fwd_span_finish(p: Plan, q, k, v, g, h_in, blk, want_ht: bool = False):
    """Phase 2: the span's output from its incoming state ``h_in`` -> (o, ht|None)."""
    dev = q.device
    o = torch.empty(p.B, p.T, p.H, p.V, dtype=q.dtype, device=dev)
    ht = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev) if want_ht else None
    a = _C.ChunkFwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h_in), _C.ptr(o), _C.ptr(ht),
                        None, None, None, None, 0, _C.ptr(blk), blk.numel())
    _C.call("tops_gla_chunk_fwd_span_finish", a, _C.stream_of(q))
    return o, ht


def _span_bwd_args(p: Plan, q, k, v, g, do, dht, blk, outs=(None,) * 5):
    dq, dk, dv, dg, dh0 = outs
    return _C.ChunkBwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), None, _C.ptr(do), _C.ptr(dht),
                           None, None, None, _C.ptr(dq), _C.ptr(dk), _C.ptr(dv), _C.ptr(dg), _C.ptr(dh0), None, 0,
                           _C.ptr(blk), blk.numel())


def bwd_span_begin(p: Plan, q, k, v, g, do, blk):
    """Phase 1 of a span's backward -> (local dh0 of the span's own loss, workspace to pass on)."""
    a = _span_bwd_args(p, q, k, v, g, do, None, blk)
    ws = torch.empty(max(int(_C.lib().tops_gla_chunk_bwd_span_workspace_size(a)), 1), dtype=torch.uint8,
                     device=q.device)
    a.workspace, a.workspace_bytes = _C.ptr(ws), ws.numel()
    L = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=q.device)
    _C.call("tops_gla_chunk_bwd_span_begin", a, _C.ptr(L), _C.stream_of(q))
    return L, ws


def bwd_span_begin_p2p(p: Plan, q, k, v, g, do, blk, D, x):
    """Phase 1 of the backward with the exchange's push fused in: the span's local dh0 and
    the forward's decay ``D`` go straight to the peer regions named by ``x`` -> workspace."""
    a = _span_bwd_args(p, q, k, v, g, do, None, blk)
    ws = torch.empty(max(int(_C.lib().tops_gla_chunk_bwd_span_workspace_size(a)), 1), dtype=torch.uint8,
                     device=q.device)
    a.workspace, a.workspace_bytes = _C.ptr(ws), ws.numel()
    _C.call("tops_gla_chunk_bwd_span_begin_p2p", a, _C.ptr(D.contiguous()), x, _C.stream_of(q))
    return ws


def bwd_span_finish(p: Plan, q, k, v, g, do, dht_in, blk, ws, want_dh0: bool = False):
    """Phase 2: gradients from the final-state gradient ``dht_in`` -> (dq, dk, dv, dg, dh0|None)."""
    dev = q.device
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(p.B, p.T, p.H, p.K, dtype=torch.float32, device=dev)
    dh0 = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev) if want_dh0 else None
    a = _span_bwd_args(p, q, k, v, g, do, dht_in, blk, (dq, dk, dv, dg, dh0))
    a.workspace, a.workspace_bytes = _C.ptr(ws), ws.numel()
    _C.call("tops_gla_chunk_bwd_span_finish", a, _C.stream_of(q))
    return dq, dk, dv, dg, dh0


# ---------------------------------------------------------------------------
# sub-functions
# ---------------------------------------------------------------------------

def cumsum(p: Plan, g, reverse=False, scale=1.0):
    out = torch.empty(p.B, p.T, p.H, p.K, dtype=torch.float32, device=g.device)
    s = p.shape()
    _C.call("tops_gla_chunk_local_cumsum", s, _C.ptr(g), _C.ptr(out), int(bool(reverse)), float(scale),
            _C.stream_of(g))
    return out


def fwd_h(p: Plan, k, v, gc, h0, want_h=True, want_ht=True):
    dev = k.device
    h = torch.empty(p.NT, p.H, p.K, p.V, dtype=torch.float32, device=dev) if want_h else None
    ht = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev) if want_ht else None
    _C.call("tops_gla_chunk_fwd_h", p.shape(), _C.ptr(k), _C.ptr(v), _C.ptr(gc), _C.ptr(h0), _C.ptr(h), _C.ptr(ht),
            _C.stream_of(k))
    return h, ht


def bwd_dh(p: Plan, q, gc, do, dht, want_dh0):
    dev = q.device
    dh = torch.empty(p.NT, p.H, p.K, p.V, dtype=torch.float32, device=dev)
    dh0 = torch.empty(p.N, p.H, p.K, p.V, dtype=torch.float32, device=dev) if want_dh0 else None
    _C.call("tops_gla_chunk_bwd_dh", p.shape(), _C.ptr(q), _C.ptr(gc), _C.ptr(do), _C.ptr(dht), _C.ptr(dh),
            _C.ptr(dh0), _C.stream_of(q))
    return dh, dh0


def intra(p: Plan, q, k, gc, causal: bool):
    A = torch.empty(p.B, p.T, p.H, p.C, dtype=torch.float32, device=q.device)
    _C.call("tops_gla_chunk_fwd_intra", p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(gc), int(bool(causal)), _C.ptr(A),
            _C.stream_of(q))
    return A


def fwd_o(p: Plan, q, v, gc, A, h):
    o = torch.empty(p.B, p.T, p.H, p.V, dtype=q.dtype, device=q.device)
    _C.call("tops_gla_chunk_fwd_o", p.shape(), _C.ptr(q), _C.ptr(v), _C.ptr(gc), _C.ptr(A), _C.ptr(h), _C.ptr(o),
            _C.stream_of(q))
    return o


def bwd_dA(p: Plan, v, do):
    dA = torch.empty(p.B, p.T, p.H, p.C, dtype=torch.float32, device=v.device)
    _C.call("tops_gla_chunk_bwd_dA", p.shape(), _C.ptr(v), _C.ptr(do), _C.ptr(dA), _C.stream_of(v))
    return dA


def bwd_dv(p: Plan, k, gc, A, do, dh):
    dv = torch.empty(p.B, p.T, p.H, p.V, dtype=torch.float32, device=k.device)
    _C.call("tops_gla_chunk_bwd_dv", p.shape(), _C.ptr(k), _C.ptr(gc), _C.ptr(A), _C.ptr(do), _C.ptr(dh), _C.ptr(dv),
            _C.stream_of(k))
    return dv


def bwd_dqk_intra(p: Plan, q, k, gc, dA):
    dq = torch.empty(p.B, p.T, p.H, p.K, dtype=torch.float32, device=q.device)
    dk = torch.empty_like(dq)
    _C.call("tops_gla_chunk_bwd_dqk_intra", p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(gc), _C.ptr(dA), _C.ptr(dq),
            _C.ptr(dk), _C.stream_of(q))
    return dq, dk


def bwd_dqkg(p: Plan, q, k, v, h, gc, do, dh, dq_in, dk_in, out_dtype=torch.float32):
    dq = torch.empty(p.B, p.T, p.H, p.K, dtype=out_dtype, device=q.device)
    dk = torch.empty_like(dq)
    dg = torch.empty(p.B, p.T, p.H, p.K, dtype=torch.float32, device=q.device)
    _C.call("tops_gla_chunk_bwd_dqkg", p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(h), _C.ptr(gc), _C.ptr(do),
            _C.ptr(dh), _C.ptr(dq_in), _C.ptr(dk_in), _C.ptr(dq), _C.ptr(dk), _C.dtype_code(out_dtype), _C.ptr(dg),
            _C.stream_of(q))
    return dq, dk, dg


def span_decay(p: Plan, g):
    d = torch.empty(p.N, p.H, p.K, dtype=torch.float32, device=g.device)
    _C.call("tops_gla_span_decay", p.shape(), _C.ptr(g), _C.ptr(d), _C.stream_of(g))
    return d


def state_combine(decay, h_in, s_local, out=None):
    N, H, K, V = s_local.shape
    out = torch.empty_like(s_local) if out is None else out
    _C.call("tops_gla_state_combine", N, H, K, V, _C.ptr(decay), _C.ptr(h_in), _C.ptr(s_local), _C.ptr(out),
            _C.stream_of(s_local))
    return out


# ---------------------------------------------------------------------------
# recurrent
# ---------------------------------------------------------------------------

def _rec_args(q, k, v, gk, gv, h0, scale, reverse, cu_dev, N, o=None, ht=None):
    B, T, H, K = q.shape
    V = v.shape[-1]
    return _C.RecArgs(B, T, H, K, V, N, _C.dtype_code(q.dtype), float(scale), int(bool(reverse)), _C.ptr(cu_dev),
                      _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(gk), _C.ptr(gv), _C.ptr(h0), _C.ptr(o), _C.ptr(ht),
                      None, 0)


def recurrent_fwd(q, k, v, gk, gv, h0, scale, output_final_state, reverse, cu_dev, N):
    B, T, H, K = q.shape
    V = v.shape[-1]
    dev = q.device
    o = (torch.zeros if cu_dev is not None else torch.empty)(B, T, H, V, dtype=torch.float32, device=dev)
    ht = torch.empty(N, H, K, V, dtype=torch.float32, device=dev) if output_final_state else None
    a = _rec_args(q, k, v, gk, gv, h0, scale, reverse, cu_dev, N, o, ht)
    ws = _ws(_C.lib().tops_gla_recurrent_fwd_workspace_size(a), dev)
    a.workspace, a.workspace_bytes = _C.ptr(ws), (ws.numel() if ws is not None else 0)
    _C.call("tops_gla_recurrent_fwd", a, _C.stream_of(q))
    return o, ht


def recurrent_bwd(q, k, v, gk, gv, h0, o, do, dht, scale, reverse, cu_dev, N):
    B, T, H, K = q.shape
    V = v.shape[-1]
    dev = q.device
    z = torch.zeros if cu_dev is not None else torch.empty
    dq = z(B, T, H, K, dtype=torch.float32, device=dev)
    dk = z(B, T, H, K, dtype=torch.float32, device=dev)
    dv = z(B, T, H, V, dtype=torch.float32, device=dev)
    dgk = z(B, T, H, K, dtype=torch.float32, device=dev) if gk is not None else None
    dgv = z(B, T, H, V, dtype=torch.float32, device=dev) if gv is not None else None
    dh0 = torch.empty(N, H, K, V, dtype=torch.float32, device=dev) if h0 is not None else None
    f = _rec_args(q, k, v, gk, gv, h0, scale, reverse, cu_dev, N)
    a = _C.RecBwdArgs(f, _C.ptr(o), _C.ptr(do), _C.ptr(dht), _C.ptr(dq), _C.ptr(dk), _C.ptr(dv), _C.ptr(dgk),
                      _C.ptr(dgv), _C.ptr(dh0))
    ws = _ws(_C.lib().tops_gla_recurrent_bwd_workspace_size(a), dev)
    a.f.workspace, a.f.workspace_bytes = _C.ptr(ws), (ws.numel() if ws is not None else 0)
    _C.call("tops_gla_recurrent_bwd", a, _C.stream_of(q))
    return dq, dk, dv, dgk, dgv, dh0

