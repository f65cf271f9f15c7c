"""Chunked Gated Linear Attention on B200 -- the API of ``tops.ops.gla.chunk``.

Same names, arguments, return values and assertion behaviour as the reference
module (primatrix/pallas-kernel ``tops/ops/gla/chunk.py``); arrays are torch CUDA
tensors instead of JAX arrays and every computation runs in ``libtops_gla.so``
(hand-written sm_100a CUDA).  ``chunk_gla`` is differentiable through
``torch.autograd`` (the analogue of a ``jax.custom_vjp``): its backward calls the
fused chunk backward of the library.

Layout: q, k, g ``[B, T, H, K]``; v, o ``[B, T, H, V]``; states ``[N, H, K, V]``.
"""
from __future__ import annotations

import torch

from . import _core
from ._core import _cuda, _f32, make_plan

__all__ = [
    "chunk_gla",
    "chunk_gla_fwd",
    "chunk_gla_bwd",
    "chunk_local_cumsum_vector",
    "chunk_local_cumsum_ref",
    "chunk_fwd_h_ref",
    "chunk_gla_fwd_intra_gk",
    "chunk_gla_fwd_intra_gk_ref",
    "chunk_gla_fwd_o_gk",
    "chunk_gla_fwd_o_gk_ref",
    "chunk_gla_bwd_dA_ref",
    "chunk_gla_bwd_dv_ref",
    "chunk_gla_bwd_dqk_intra_ref",
    "chunk_gla_bwd_dqkg_ref",
]


def _check_qkv(q, k, v):
    assert q.dim() == 4, f"q must be [B, T, H, K], got {tuple(q.shape)}"
    B, T, H, K = q.shape
    assert k.shape == (B, T, H, K), f"Expected k shape {(B, T, H, K)}, got {tuple(k.shape)}"
    assert v.dim() == 4 and v.shape[:3] == (B, T, H), f"Expected v shape {(B, T, H, '*')}, got {tuple(v.shape)}"
    assert q.dtype == k.dtype == v.dtype, f"q, k, v must share a dtype, got {q.dtype}, {k.dtype}, {v.dtype}"


def _gates(q, g, g_gamma):
    """g is used when given; otherwise g_gamma broadcast to q.shape; otherwise zeros (chunk.py:1114-1118)."""
    if g is not None:
        assert g.shape == q.shape, f"Expected g shape {tuple(q.shape)}, got {tuple(g.shape)}"
        return _f32("g", g)
    if g_gamma is not None:
        return _f32("g_gamma", torch.broadcast_to(g_gamma.float(), q.shape))
    return None


def _reduce_to(dg, g_gamma):
    """Sum-reduce a full gate gradient to g_gamma's shape (chunk.py:966-975)."""
    for i, (d_full, d_gamma) in enumerate(zip(dg.shape[::-1], g_gamma.shape[::-1])):
        if d_full != d_gamma:
            dg = dg.sum(dim=dg.dim() - 1 - i, keepdim=True)
    missing = dg.dim() - g_gamma.dim()
    if missing > 0:
        dg = dg.sum(dim=tuple(range(missing)))
    return dg.reshape(g_gamma.shape)


class _ChunkGLA(torch.autograd.Function):
    """o, ht = chunk_gla(...) with the library's fused backward as the VJP."""

    @staticmethod
    def forward(ctx, q, k, v, g, h0, g_gamma, scale, output_final_state, cu_seqlens, chunk_size):
        p = make_plan(q, v.shape[-1], chunk_size, cu_seqlens, scale)
        gg = _gates(q, g, g_gamma)
        h0c = _f32("initial_state", h0)
        save = any(ctx.needs_input_grad[:6])
        o, ht, saved = _core.chunk_fwd(p, q, k, v, gg, h0c, output_final_state, save)
        if save:
            ctx.save_for_backward(q, k, v, gg, h0c, saved.get("g_cumsum"), saved.get("A"), saved.get("h"),
                                  saved.get("block"))
            ctx.plan = p
            ctx.g_shape = None if g is not None else (g_gamma.shape if g_gamma is not None else None)
            ctx.g_dtype = g.dtype if g is not None else (g_gamma.dtype if g_gamma is not None else None)
        if ht is None:
            return o
        return o, ht

    @staticmethod
    def backward(ctx, do, dht=None):
        q, k, v, gg, h0c, gc, A, h, blk = ctx.saved_tensors
        p = ctx.plan
        do = do.contiguous().to(q.dtype)
        dht = None if dht is None else dht.float().contiguous()
        want_dh0 = h0c is not None
        dq, dk, dv, dg, dh0 = _core.chunk_bwd(p, q, k, v, gg, h0c, do, dht, gc, A, h, want_dh0, block=blk)
        d_g = d_gamma = None
        if ctx.needs_input_grad[3]:
            d_g = dg.to(ctx.g_dtype)
        if ctx.needs_input_grad[5]:
            d_gamma = _reduce_to(dg, torch.empty(ctx.g_shape, device="meta")).to(ctx.g_dtype)
        return dq, dk, dv, d_g, dh0, d_gamma, None, None, None, None


def chunk_gla(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor | None = None,
    g_gamma: torch.Tensor | None = None,
    scale: float | None = None,
    initial_state: torch.Tensor | None = None,
    output_final_state: bool = False,
    cu_seqlens=None,
    chunk_size: int = 16,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Chunked GLA forward (differentiable).  Mirrors ``tops.ops.gla.chunk_gla`` (chunk.py:1187).

    Args:
        q: [B, T, H, K] queries; k: [B, T, H, K] keys; v: [B, T, H, V] values.
        g: [B, T, H, K] log-space gates (after logsigmoid) or None.
        g_gamma: gate broadcastable to [B, T, H, K], used only when g is None.
        scale: attention scale, default K ** -0.5.
        initial_state: [N, H, K, V] initial recurrent state (fp32) or None.
        output_final_state: also return the final state [N, H, K, V] (fp32).
        cu_seqlens: [N+1] cumulative sequence lengths (varlen; B must be 1).
        chunk_size: block size of the chunked algorithm (power of 2).
    Returns:
        o: [B, T, H, V] in q's dtype; final_state: [N, H, K, V] fp32 or None.
    """
    _check_qkv(q, k, v)
    B, T, H, K = q.shape
    V = v.shape[-1]
    N = B if cu_seqlens is None else len(_core.host_cu(cu_seqlens)) - 1
    if initial_state is not None:
        assert initial_state.shape == (N, H, K, V), \
            f"Expected initial_state shape {(N, H, K, V)}, got {tuple(initial_state.shape)}"
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    gamma = None
    if g is None and g_gamma is not None:
        gamma = g_gamma
    out = _ChunkGLA.apply(q, k, v, g, initial_state, gamma, scale, bool(output_final_state), cu_seqlens,
                          int(chunk_size))
    if output_final_state:
        o, ht = out
        return o, ht
    return out, None


def chunk_gla_fwd(q, k, v, g, g_gamma, g_cumsum, scale, initial_state, output_final_state, cu_seqlens=None,
                  chunk_size: int = 64):
    """Forward orchestrator returning ``(g_cumsum, A, h, ht, o)``.  Mirrors chunk.py:1083.

    ``A`` is the causal intra-chunk matrix [B, T, H, C] (fp32), ``h`` the state at the
    start of every chunk [B, NT, H, K, V] (varlen: [1, NT_total, ...]) in k's dtype,
    ``ht`` the final state (fp32) or None.
    """
    _check_qkv(q, k, v)
    p = make_plan(q, v.shape[-1], chunk_size, cu_seqlens, scale)
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    gg = _gates(q, g, g_gamma)
    if g_cumsum is not None:
        gc = _f32("g_cumsum", g_cumsum)
        h, ht = _core.fwd_h(p, k, v, gc, _f32("initial_state", initial_state), True, bool(output_final_state))
        A = _core.intra(p, q, k, gc, causal=True)
        o = _core.fwd_o(p, q, v, gc, A, h)
    else:
        gc = _core.cumsum(p, gg) if gg is not None else torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        h, ht = _core.fwd_h(p, k, v, gc, _f32("initial_state", initial_state), True, bool(output_final_state))
        A = _core.intra(p, q, k, gc, causal=True)
        o = _core.fwd_o(p, q, v, gc, A, h)
    h = h.view(1 if p.cu_host is not None else p.B, -1, p.H, p.K, p.V).to(k.dtype)
    return gc, A, h, (ht if output_final_state else None), o


def chunk_gla_bwd(q, k, v, g, g_gamma, g_cumsum, scale, initial_state, h, A, do, dht, cu_seqlens=None,
                  chunk_size: int = 64):
    """Backward orchestrator returning ``(dq, dk, dv, dg, dh0)``.  Mirrors chunk.py:815.

    ``h``/``A``/``g_cumsum`` from the forward may be passed (else recomputed).  ``dh0``
    is returned when ``initial_state`` or ``dht`` is given (chunk_h.py:448-452).
    With ``g=None`` and ``g_gamma`` given, dg is sum-reduced to g_gamma's shape.
    """
    _check_qkv(q, k, v)
    assert do.shape == v.shape, f"Expected do shape {tuple(v.shape)}, got {tuple(do.shape)}"
    p = make_plan(q, v.shape[-1], chunk_size, cu_seqlens, scale)
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    gg = _gates(q, g, g_gamma)
    do = _cuda("do", do).to(q.dtype)
    hh = None if h is None else _f32("h", h).reshape(p.NT, p.H, p.K, p.V)
    dq, dk, dv, dg, dh0 = _core.chunk_bwd(p, q, k, v, gg, _f32("initial_state", initial_state), do,
                                          _f32("dht", dht), _f32("g_cumsum", g_cumsum), _f32("A", A), hh,
                                          want_dh0=(initial_state is not None or dht is not None))
    if g is None and g_gamma is not None:
        dg = _reduce_to(dg, g_gamma)
    return dq, dk, dv, dg, dh0


# ---------------------------------------------------------------------------
# sub-functions (exported by tops.ops.gla; tops/ops/gla/__init__.py:2-14)
# ---------------------------------------------------------------------------

def chunk_local_cumsum_vector(g, chunk_size: int, reverse: bool = False, scale: float | None = None,
                              cu_seqlens=None, head_first: bool = False, output_dtype=torch.float32,
                              chunk_indices=None):
    """Chunk-local cumsum of gates.  Mirrors chunk.py:110 (``chunk_local_cumsum``)."""
    assert chunk_size == 2 ** (chunk_size.bit_length() - 1), "chunk_size must be power of 2"
    if head_first:
        g = g.transpose(1, 2)
    B, T, H, K = g.shape
    p = make_plan(g, 1, chunk_size, cu_seqlens, 1.0)
    out = _core.cumsum(p, _f32("g", g), reverse=reverse, scale=1.0 if scale is None else scale)
    if head_first:
        out = out.transpose(1, 2)
    return out.to(output_dtype or g.dtype)


def chunk_local_cumsum_ref(g, chunk_size: int, scale: float | None = None, reverse: bool = False,
                           cu_seqlens_cpu=None):
    """Mirrors chunk.py:20 (forward cumsum only, like the reference)."""
    assert reverse is False, "Reverse mode not supported in chunk_local_cumsum"
    return chunk_local_cumsum_vector(g, chunk_size, scale=scale, cu_seqlens=cu_seqlens_cpu)


def chunk_fwd_h_ref(k, v, gk=None, h0=None, output_final_state: bool = False, cu_seqlens_cpu=None,
                    chunk_size: int = 64):
    """State at the start of each chunk.  Mirrors chunk.py:206 (exported as ``chunk_fwd_h``).

    Returns h [B, NT, H, K, V] (k's dtype; varlen [1, NT_total, ...]) and ht [N, H, K, V]
    (fp32; zeros when output_final_state is False, as in the reference).
    """
    assert k.dim() == 4 and v.dim() == 4 and v.shape[:3] == k.shape[:3]
    p = make_plan(k, v.shape[-1], chunk_size, cu_seqlens_cpu, 1.0)
    k, v = _cuda("k", k), _cuda("v", v)
    gc = _f32("gk", gk) if gk is not None else torch.zeros(k.shape, dtype=torch.float32, device=k.device)
    h, ht = _core.fwd_h(p, k, v, gc, _f32("h0", h0), True, True)
    if not output_final_state:
        ht = torch.zeros_like(ht)
    return h.view(1 if p.cu_host is not None else p.B, -1, p.H, p.K, p.V).to(k.dtype), ht


def chunk_gla_fwd_intra_gk(q, k, g, scale, chunk_size: int):
    """Full (non-causal) intra-chunk matrix A[i, j] = scale (q_i e^{g_i}) . (k_j e^{-g_j}), [B, T, H, C].

    Mirrors the exported Pallas launcher chunk.py:386 (kernel :350).
    """
    _check_qkv(q, k, k)
    p = make_plan(q, q.shape[-1], chunk_size, None, scale)
    return _core.intra(p, _cuda("q", q), _cuda("k", k), _f32("g", g), causal=False)


def chunk_gla_fwd_intra_gk_ref(q, k, g, scale, cu_seqlens=None, chunk_size: int = 64):
    """Mirrors chunk.py:300 (first-row reference point; full C x C block)."""
    p = make_plan(q, q.shape[-1], chunk_size, cu_seqlens, scale)
    return _core.intra(p, _cuda("q", q), _cuda("k", k), _f32("g", g), causal=False)


def chunk_gla_fwd_o_gk(q, v, g, A, h, scale, cu_seqlens=None, chunk_indices=None, chunk_size: int = 64,
                       use_exp2: bool = False):
    """o = scale (q e^g) h + tril(A) v.  Mirrors chunk.py:1387 (kernel :1259).  Output in v's dtype."""
    p = make_plan(q, v.shape[-1], chunk_size, cu_seqlens, scale)
    g = _f32("g", g)
    if use_exp2:
        g = g * 0.6931471805599453
    o = _core.fwd_o(p, _cuda("q", q).to(v.dtype), _cuda("v", v), g, _f32("A", A),
                    _f32("h", h).reshape(p.NT, p.H, p.K, p.V))
    return o


def chunk_gla_fwd_o_gk_ref(q, v, gk, A, h, scale, cu_seqlens_cpu=None, chunk_size: int = 64):
    """Mirrors chunk.py:441."""
    return chunk_gla_fwd_o_gk(q, v, gk, A, h, scale, cu_seqlens=cu_seqlens_cpu, chunk_size=chunk_size)


def chunk_gla_bwd_dA_ref(v, do, scale, cu_seqlens_cpu=None, chunk_size: int = 64):
    """dA = tril(scale do v^T) per chunk, [B, T, H, C].  Mirrors chunk.py:504."""
    p = make_plan(v, v.shape[-1], chunk_size, cu_seqlens_cpu, scale)
    v = _cuda("v", v)
    return _core.bwd_dA(p, v, _cuda("do", do).to(v.dtype))


def chunk_gla_bwd_dv_ref(k, g_cumsum, A, do, dh, cu_seqlens_cpu=None, chunk_size: int = 64):
    """dv = tril(A)^T do + (k e^{G_last-G}) dh.  Mirrors chunk.py:547."""
    p = make_plan(k, do.shape[-1], chunk_size, cu_seqlens_cpu, 1.0)
    k = _cuda("k", k)
    return _core.bwd_dv(p, k, _f32("g_cumsum", g_cumsum), _f32("A", A), _cuda("do", do).to(k.dtype),
                        _f32("dh", dh).reshape(p.NT, p.H, p.K, p.V))


def chunk_gla_bwd_dqk_intra_ref(q, k, g_cumsum, dA, cu_seqlens_cpu=None, chunk_size: int = 64):
    """Intra-chunk dq, dk from dA.  Mirrors chunk.py:603."""
    p = make_plan(q, q.shape[-1], chunk_size, cu_seqlens_cpu, 1.0)
    return _core.bwd_dqk_intra(p, _cuda("q", q), _cuda("k", k), _f32("g_cumsum", g_cumsum), _f32("dA", dA))


def chunk_gla_bwd_dqkg_ref(q, k, v, h, g_cumsum, do, dh, dq, dk, scale, cu_seqlens_cpu=None, chunk_size: int = 64):
    """Inter-chunk dq, dk (added to the given intra parts) and dg.  Mirrors chunk.py:656."""
    p = make_plan(q, v.shape[-1], chunk_size, cu_seqlens_cpu, scale)
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    return _core.bwd_dqkg(p, q, k, v, _f32("h", h).reshape(p.NT, p.H, p.K, p.V), _f32("g_cumsum", g_cumsum),
                          _cuda("do", do).to(q.dtype), _f32("dh", dh).reshape(p.NT, p.H, p.K, p.V),
                          _f32("dq", dq), _f32("dk", dk), out_dtype=torch.float32)
