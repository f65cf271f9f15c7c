"""CPU oracle for the Gated Linear Attention (GLA) operators -- TEST INFRASTRUCTURE.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The CUDA library (``libtops_gla.so``) never calls into it, and the product
path raises when the CUDA extension is missing instead of falling back here.

It is a numpy restatement of the reference's algorithm (primatrix/pallas-kernel,
package ``tops``).  Each function cites the reference file:line it follows.
Arithmetic runs in ``dtype`` (float64 by default, so the oracle is closer to the
exact answer than any fp32 implementation; ``bench.py`` times it in float32,
which is what the reference computes in).

Layout convention (same as the reference, FLA style):
    q, k, g : [B, T, H, K]      v, o, do : [B, T, H, V]
    states  : [N, H, K, V]      per-chunk states h / dh : [B, NT, H, K, V]
    varlen  : B == 1, ``cu_seqlens`` = [N+1] host integers; each segment is
              padded to a multiple of the chunk size on its own and per-chunk
              tensors are concatenated in segment order.

Parity is pinned against fixtures produced by the reference's own Torch CPU
restatement (``tests/golden/make_golden.py``); see ``tests/test_oracle.py``.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "chunk_local_cumsum",
    "chunk_fwd_h",
    "chunk_bwd_dh",
    "chunk_gla_fwd_intra_gk",
    "chunk_gla_fwd_o_gk",
    "chunk_gla_fwd",
    "chunk_gla_bwd_dA",
    "chunk_gla_bwd_dv",
    "chunk_gla_bwd_dqk_intra",
    "chunk_gla_bwd_dqkg",
    "chunk_gla_bwd",
    "chunk_gla",
    "fused_recurrent_gla",
    "fused_recurrent_gla_bwd",
    "naive_recurrent_gla",
    "seq_bounds",
]


def _f(x, dt):
    return None if x is None else np.asarray(x, dtype=dt)


def _contract(spec, a, b):
    """Two-operand einsum (single-letter indices) evaluated as a batched ``np.matmul``.

    numpy's einsum keeps contractions whose batch index appears in both operands and
    the output (the per-head index ``h`` here) on its element loop, which is ~20x
    slower than BLAS at these sizes; this routes them through matmul.  Only the
    summation order differs from the plain sum.
    """
    ins, out = spec.split("->")
    sa, sb = ins.split(",")
    batch = [c for c in out if c in sa and c in sb]
    contr = [c for c in sa if c in sb and c not in out]
    fa = [c for c in sa if c not in sb]
    fb = [c for c in sb if c not in sa]
    dim = {c: a.shape[sa.index(c)] for c in sa}
    dim.update({c: b.shape[sb.index(c)] for c in sb})
    n = lambda cs: int(np.prod([dim[c] for c in cs])) if cs else 1
    bsh = [dim[c] for c in batch]
    at = a.transpose([sa.index(c) for c in batch + fa + contr]).reshape(bsh + [n(fa), n(contr)])
    bt = b.transpose([sb.index(c) for c in batch + contr + fb]).reshape(bsh + [n(contr), n(fb)])
    r = np.matmul(at, bt).reshape(bsh + [dim[c] for c in fa] + [dim[c] for c in fb])
    order = batch + fa + fb
    return r.transpose([order.index(c) for c in out])


def seq_bounds(B: int, T: int, cu_seqlens):
    """(bos, eos) row ranges of every sequence in the flattened [B*T] row space.

    Mirrors the bos/eos selection of ``tops/ops/common/chunk_h.py:324-330``.
    """
    if cu_seqlens is None:
        return [(n * T, (n + 1) * T) for n in range(B)]
    cu = [int(c) for c in cu_seqlens]
    return [(cu[i], cu[i + 1]) for i in range(len(cu) - 1)]


def _pad_rows(x, bounds, C):
    """Pad every segment of a [R, ...] row array to a multiple of C.

    Restates ``_pad_varlen_seqs_jax`` (``tops/ops/gla/chunk.py:751-793``) and the
    fixed-length T padding of ``chunk_gla_fwd`` (``chunk.py:1120-1126``).
    Returns the padded array and the padded (bos, eos) bounds.
    """
    parts, nb, off = [], [], 0
    for bos, eos in bounds:
        L = eos - bos
        PL = ((L + C - 1) // C) * C
        seg = x[bos:eos]
        if PL > L:
            seg = np.concatenate([seg, np.zeros((PL - L,) + x.shape[1:], x.dtype)], 0)
        parts.append(seg)
        nb.append((off, off + PL))
        off += PL
    return np.concatenate(parts, 0) if parts else x[:0], nb


def _unpad_rows(x, bounds, pbounds):
    """Inverse of ``_pad_rows`` (``chunk.py:796-807``)."""
    return np.concatenate([x[pb:pb + (e - b)] for (b, e), (pb, _) in zip(bounds, pbounds)], 0)


# ---------------------------------------------------------------------------
# Sub-function 1: chunk-local cumsum
# ---------------------------------------------------------------------------

def chunk_local_cumsum(g, chunk_size, cu_seqlens=None, dtype=np.float64):
    """Chunk-local inclusive prefix sum of log-gates along time.

    Follows ``chunk_local_cumsum_ref`` (``tops/ops/gla/chunk.py:20-52``) and the
    kernel ``chunk_cumsum_kernel`` (``chunk.py:55-107``).  Ragged last chunks are
    handled as if zero-padded (equivalent to the reference's padding).
    g: [B, T, H, K] -> [B, T, H, K]
    """
    g = _f(g, dtype)
    B, T, H, K = g.shape
    C = chunk_size
    flat = g.reshape(B * T, H, K)
    out = np.empty_like(flat)
    for bos, eos in seq_bounds(B, T, cu_seqlens):
        for s in range(bos, eos, C):
            e = min(s + C, eos)
            out[s:e] = np.cumsum(flat[s:e], axis=0)
    return out.reshape(B, T, H, K)


# ---------------------------------------------------------------------------
# Sub-function 2: inter-chunk state scan (forward)
# ---------------------------------------------------------------------------

def chunk_fwd_h(k, v, gk, h0=None, output_final_state=False, cu_seqlens=None,
                chunk_size=64, dtype=np.float64):
    """State at the start of every chunk: h_{c+1} = diag(e^{G_last}) h_c + (k e^{G_last-G})^T v.

    Follows ``chunk_fwd_h_ref`` (``tops/ops/common/chunk_h.py:277-396``, gk path
    ``:372-386``).  ``gk`` is the chunk-local cumsum.  T need not be a multiple of
    chunk_size (ragged chunks act as zero padding).
    Returns h [B, NT, H, K, V] (varlen: [1, NT_total, ...]) and ht [N, H, K, V] or None.
    """
    k, v, gk, h0 = (_f(x, dtype) for x in (k, v, gk, h0))
    B, T, H, K = k.shape
    V = v.shape[-1]
    C = chunk_size
    bounds = seq_bounds(B, T, cu_seqlens)
    kf, vf, gf = k.reshape(-1, H, K), v.reshape(-1, H, V), gk.reshape(-1, H, K)
    hs, hts = [], []
    for n, (bos, eos) in enumerate(bounds):
        h = np.zeros((H, K, V), dtype) if h0 is None else h0[n].copy()
        for s in range(bos, eos, C):
            e = min(s + C, eos)
            hs.append(h.copy())
            gc = gf[s:e]
            gl = gc[-1]                                   # [H, K]
            kd = kf[s:e] * np.exp(gl[None] - gc)          # [L, H, K]
            h = h * np.exp(gl)[:, :, None] + _contract("lhk,lhv->hkv", kd, vf[s:e])
        hts.append(h)
    h_all = np.stack(hs, 0) if hs else np.zeros((0, H, K, V), dtype)
    h_all = h_all.reshape((1, -1, H, K, V) if cu_seqlens is not None else (B, -1, H, K, V))
    ht = np.stack(hts, 0) if output_final_state else None
    return h_all, ht


# ---------------------------------------------------------------------------
# Sub-function 3: intra-chunk attention matrix
# ---------------------------------------------------------------------------

def chunk_gla_fwd_intra_gk(q, k, g, scale, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """A_ij = scale * sum_k q_ik k_jk exp(G_ik - G_jk), causal (j <= i) within a chunk.

    Follows ``chunk_gla_fwd_intra_gk_ref`` (``tops/ops/gla/chunk.py:300-345``,
    first-row reference point ``:330-332``) plus the causal mask applied by the
    orchestrator (``tests`` oracle ``chunk.py:476-478`` / Pallas ``chunk.py:1309-1311``).
    Returns A [B, T, H, C]; column j of row i refers to position j of i's chunk.
    """
    q, k, g = (_f(x, dtype) for x in (q, k, g))
    B, T, H, K = q.shape
    C = chunk_size
    qf, kf, gf = q.reshape(-1, H, K), k.reshape(-1, H, K), g.reshape(-1, H, K)
    A = np.zeros((B * T, H, C), dtype)
    for bos, eos in seq_bounds(B, T, cu_seqlens):
        for s in range(bos, eos, C):
            e = min(s + C, eos)
            L = e - s
            gn = gf[s:s + 1]
            qg = qf[s:e] * np.exp(gf[s:e] - gn)
            kg = kf[s:e] * np.exp(gn - gf[s:e])
            a = _contract("ihk,jhk->ihj", qg, kg) * scale  # [L, H, L]
            mask = np.tril(np.ones((L, L), bool))
            a = np.where(mask[:, None, :], a, 0.0)
            A[s:e, :, :L] = a
    return A.reshape(B, T, H, C)


# ---------------------------------------------------------------------------
# Sub-function 4: output
# ---------------------------------------------------------------------------

def chunk_gla_fwd_o_gk(q, v, g, A, h, scale, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """o = scale (q e^{G}) h_c + tril(A) v, per chunk.

    Follows ``chunk_gla_fwd_o_gk_ref`` (``tops/ops/gla/chunk.py:441-497``) and the
    kernel ``chunk_gla_fwd_o_gk_pl_kernel`` (``chunk.py:1259-1312``).
    h: per-chunk start states in chunk order ([B, NT, ...] or [1, NT_total, ...]).
    """
    q, v, g, A, h = (_f(x, dtype) for x in (q, v, g, A, h))
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    qf, vf, gf = q.reshape(-1, H, K), v.reshape(-1, H, V), g.reshape(-1, H, K)
    Af = A.reshape(-1, H, C)
    hf = h.reshape(-1, H, K, V)
    o = np.zeros((B * T, H, V), dtype)
    ci = 0
    for bos, eos in seq_bounds(B, T, cu_seqlens):
        for s in range(bos, eos, C):
            e = min(s + C, eos)
            L = e - s
            qg = qf[s:e] * np.exp(gf[s:e])
            o_inter = scale * _contract("lhk,hkv->lhv", qg, hf[ci])
            a = np.tril(np.ones((L, L)))[:, None, :] * Af[s:e, :, :L]
            o_intra = _contract("ihj,jhv->ihv", a, vf[s:e])
            o[s:e] = o_inter + o_intra
            ci += 1
    return o.reshape(B, T, H, V)


# ---------------------------------------------------------------------------
# Forward orchestrator and public op
# ---------------------------------------------------------------------------

def chunk_gla_fwd(q, k, v, g, g_cumsum=None, scale=None, initial_state=None,
                  output_final_state=False, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """cumsum -> h -> A -> o.  Returns (g_cumsum, A, h, ht, o).

    Follows ``chunk_gla_fwd`` (``tops/ops/gla/chunk.py:1083-1179``).  ``g=None``
    means zero gates (``chunk.py:1114-1118``).
    """
    q, k, v = (_f(x, dtype) for x in (q, k, v))
    g = np.zeros_like(q) if g is None else _f(g, dtype)
    K = q.shape[-1]
    if scale is None:
        scale = K ** -0.5
    gc = chunk_local_cumsum(g, chunk_size, cu_seqlens, dtype) if g_cumsum is None else _f(g_cumsum, dtype)
    h, ht = chunk_fwd_h(k, v, gc, initial_state, output_final_state, cu_seqlens, chunk_size, dtype)
    A = chunk_gla_fwd_intra_gk(q, k, gc, scale, cu_seqlens, chunk_size, dtype)
    o = chunk_gla_fwd_o_gk(q, v, gc, A, h, scale, cu_seqlens, chunk_size, dtype)
    return gc, A, h, ht, o


def chunk_gla(q, k, v, g=None, g_gamma=None, scale=None, initial_state=None,
              output_final_state=False, cu_seqlens=None, chunk_size=16, dtype=np.float64):
    """Public chunked GLA forward: returns (o, final_state or None).

    Follows ``chunk_gla`` (``tops/ops/gla/chunk.py:1187-1251``): inputs computed
    in floating point of ``dtype`` regardless of their storage type;
    ``g_gamma`` (broadcastable to q.shape) is used when ``g`` is None.
    """
    q = _f(q, dtype)
    if g is None:
        g = np.broadcast_to(_f(g_gamma, dtype), q.shape).copy() if g_gamma is not None else np.zeros_like(q)
    _, _, _, ht, o = chunk_gla_fwd(q, k, v, g, None, scale, initial_state, output_final_state,
                                   cu_seqlens, chunk_size, dtype)
    return o, (ht if output_final_state else None)


# ---------------------------------------------------------------------------
# Backward sub-functions
# ---------------------------------------------------------------------------

def chunk_bwd_dh(q, k, v, gk, do, h0=None, dht=None, scale=1.0, cu_seqlens=None,
                 chunk_size=64, dtype=np.float64):
    """Reverse state-gradient scan: dh_{c-1} = diag(e^{G_last}) dh_c + (scale q e^{G})^T do.

    Follows ``chunk_bwd_dh_ref`` (``tops/ops/common/chunk_h.py:399-492``).  The
    stored dh of chunk c is the gradient w.r.t. the state at the END of chunk c.
    Returns dh [B, NT, H, K, V] (varlen [1, NT_total, ...]) and dh0 [N, H, K, V]
    when ``h0`` or ``dht`` is given (``chunk_h.py:448-452``), else None.
    """
    q, do, gk, dht = (_f(x, dtype) for x in (q, do, gk, dht))
    B, T, H, K = q.shape
    V = do.shape[-1]
    C = chunk_size
    qf, dof, gf = q.reshape(-1, H, K), do.reshape(-1, H, V), gk.reshape(-1, H, K)
    per_seq, dh0s = [], []
    for n, (bos, eos) in enumerate(seq_bounds(B, T, cu_seqlens)):
        dh = np.zeros((H, K, V), dtype) if dht is None else dht[n].copy()
        starts = list(range(bos, eos, C))
        out = [None] * len(starts)
        for i in range(len(starts) - 1, -1, -1):
            s = starts[i]
            e = min(s + C, eos)
            out[i] = dh.copy()
            gc = gf[s:e]
            qh = qf[s:e] * np.exp(gc) * scale
            dh = dh * np.exp(gc[-1])[:, :, None] + _contract("lhk,lhv->hkv", qh, dof[s:e])
        per_seq.extend(out)
        dh0s.append(dh)
    dh_all = np.stack(per_seq, 0) if per_seq else np.zeros((0, H, K, V), dtype)
    dh_all = dh_all.reshape((1, -1, H, K, V) if cu_seqlens is not None else (B, -1, H, K, V))
    dh0 = np.stack(dh0s, 0) if (h0 is not None or dht is not None) else None
    return dh_all, dh0


def _chunks(B, T, cu_seqlens, C):
    ci = 0
    for bos, eos in seq_bounds(B, T, cu_seqlens):
        for s in range(bos, eos, C):
            yield ci, s, min(s + C, eos)
            ci += 1


def chunk_gla_bwd_dA(v, do, scale, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """dA_ij = scale * do_i . v_j for j <= i.  ``chunk_gla_bwd_dA_ref`` (``chunk.py:504-540``)."""
    v, do = _f(v, dtype), _f(do, dtype)
    B, T, H, V = v.shape
    C = chunk_size
    vf, dof = v.reshape(-1, H, V), do.reshape(-1, H, V)
    dA = np.zeros((B * T, H, C), dtype)
    for _, s, e in _chunks(B, T, cu_seqlens, C):
        L = e - s
        a = _contract("ihv,jhv->ihj", dof[s:e], vf[s:e]) * scale
        dA[s:e, :, :L] = np.where(np.tril(np.ones((L, L), bool))[:, None, :], a, 0.0)
    return dA.reshape(B, T, H, C)


def chunk_gla_bwd_dv(k, g_cumsum, A, do, dh, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """dv = tril(A)^T do + (k e^{G_last - G}) dh.  ``chunk_gla_bwd_dv_ref`` (``chunk.py:547-596``)."""
    k, gc, A, do, dh = (_f(x, dtype) for x in (k, g_cumsum, A, do, dh))
    B, T, H, K = k.shape
    V = do.shape[-1]
    C = chunk_size
    kf, gf, dof = k.reshape(-1, H, K), gc.reshape(-1, H, K), do.reshape(-1, H, V)
    Af, dhf = A.reshape(-1, H, C), dh.reshape(-1, H, K, V)
    dv = np.zeros((B * T, H, V), dtype)
    for ci, s, e in _chunks(B, T, cu_seqlens, C):
        L = e - s
        a = np.tril(np.ones((L, L)))[:, None, :] * Af[s:e, :, :L]
        dv_intra = _contract("ihj,ihv->jhv", a, dof[s:e])
        kd = kf[s:e] * np.exp(gf[e - 1][None] - gf[s:e])
        dv[s:e] = dv_intra + _contract("lhk,hkv->lhv", kd, dhf[ci])
    return dv.reshape(B, T, H, V)


def chunk_gla_bwd_dqk_intra(q, k, g_cumsum, dA, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """Intra-chunk dq/dk from dA.  ``chunk_gla_bwd_dqk_intra_ref`` (``chunk.py:603-649``).

    dq_i = e^{G_i} sum_{j<=i} dA_ij k_j e^{-G_j};  dk_j = e^{-G_j} sum_{i>=j} dA_ij q_i e^{G_i}.
    """
    q, k, gc, dA = (_f(x, dtype) for x in (q, k, g_cumsum, dA))
    B, T, H, K = q.shape
    C = chunk_size
    qf, kf, gf, dAf = q.reshape(-1, H, K), k.reshape(-1, H, K), gc.reshape(-1, H, K), dA.reshape(-1, H, C)
    dq, dk = np.zeros_like(qf), np.zeros_like(kf)
    for _, s, e in _chunks(B, T, cu_seqlens, C):
        L = e - s
        d = dAf[s:e, :, :L]
        dq[s:e] = np.exp(gf[s:e]) * _contract("ihj,jhk->ihk", d, kf[s:e] * np.exp(-gf[s:e]))
        dk[s:e] = np.exp(-gf[s:e]) * _contract("ihj,ihk->jhk", d, qf[s:e] * np.exp(gf[s:e]))
    return dq.reshape(B, T, H, K), dk.reshape(B, T, H, K)


def chunk_gla_bwd_dqkg(q, k, v, h, g_cumsum, do, dh, dq, dk, scale, cu_seqlens=None,
                       chunk_size=64, dtype=np.float64):
    """Inter-chunk dq/dk and the gate gradient.  ``chunk_gla_bwd_dqkg_ref`` (``chunk.py:656-743``).

    dg = revcumsum_t(q dq - k dk) + e^{G_last} sum_v(h dh) + sum_t(dk_inter k).
    """
    q, k, v, h, gc, do, dh, dq, dk = (_f(x, dtype) for x in (q, k, v, h, g_cumsum, do, dh, dq, dk))
    B, T, H, K = q.shape
    V = v.shape[-1]
    C = chunk_size
    qf, kf, vf, gf, dof = (x.reshape(-1, H, x.shape[-1]) for x in (q, k, v, gc, do))
    dqf, dkf = dq.reshape(-1, H, K), dk.reshape(-1, H, K)
    hf, dhf = h.reshape(-1, H, K, V), dh.reshape(-1, H, K, V)
    dq_o, dk_o, dg_o = np.zeros_like(qf), np.zeros_like(kf), np.zeros_like(qf)
    for ci, s, e in _chunks(B, T, cu_seqlens, C):
        gcs = gf[s:e]
        gn = gcs[-1]
        dq_inter = scale * np.exp(gcs) * _contract("lhv,hkv->lhk", dof[s:e], hf[ci])
        dk_inter = np.exp(gn[None] - gcs) * _contract("lhv,hkv->lhk", vf[s:e], dhf[ci])
        dqt = dqf[s:e] + dq_inter
        dkt = dkf[s:e] + dk_inter
        dgk_inter = np.exp(gn) * _contract("hkv,hkv->hk", hf[ci], dhf[ci]) + (dk_inter * kf[s:e]).sum(0)
        dg_raw = qf[s:e] * dqt - kf[s:e] * dkt
        dg = np.cumsum(dg_raw[::-1], axis=0)[::-1] + dgk_inter[None]
        dq_o[s:e], dk_o[s:e], dg_o[s:e] = dqt, dkt, dg
    return dq_o.reshape(B, T, H, K), dk_o.reshape(B, T, H, K), dg_o.reshape(B, T, H, K)


def chunk_gla_bwd(q, k, v, g, g_cumsum=None, scale=None, initial_state=None, h=None, A=None,
                  do=None, dht=None, cu_seqlens=None, chunk_size=64, dtype=np.float64):
    """Backward orchestrator -> (dq, dk, dv, dg, dh0).

    Follows ``chunk_gla_bwd`` (``tops/ops/gla/chunk.py:815-977``): recompute
    g_cumsum/h/A when not given, reverse dh scan, dv, dA, intra dq/dk, inter
    dq/dk + dg.  ``dh0`` is returned when ``initial_state`` or ``dht`` is given.
    """
    q, k, v, do = (_f(x, dtype) for x in (q, k, v, do))
    g = np.zeros_like(q) if g is None else _f(g, dtype)
    K = q.shape[-1]
    if scale is None:
        scale = K ** -0.5
    C = chunk_size
    gc = chunk_local_cumsum(g, C, cu_seqlens, dtype) if g_cumsum is None else _f(g_cumsum, dtype)
    if h is None:
        h, _ = chunk_fwd_h(k, v, gc, initial_state, False, cu_seqlens, C, dtype)
    dh, dh0 = chunk_bwd_dh(q, k, v, gc, do, initial_state, dht, scale, cu_seqlens, C, dtype)
    if A is None:
        A = chunk_gla_fwd_intra_gk(q, k, gc, scale, cu_seqlens, C, dtype)
    dv = chunk_gla_bwd_dv(k, gc, A, do, dh, cu_seqlens, C, dtype)
    dA = chunk_gla_bwd_dA(v, do, scale, cu_seqlens, C, dtype)
    dq, dk = chunk_gla_bwd_dqk_intra(q, k, gc, dA, cu_seqlens, C, dtype)
    dq, dk, dg = chunk_gla_bwd_dqkg(q, k, v, h, gc, do, dh, dq, dk, scale, cu_seqlens, C, dtype)
    return dq, dk, dv, dg, dh0


# ---------------------------------------------------------------------------
# Recurrent forms
# ---------------------------------------------------------------------------

def fused_recurrent_gla(q, k, v, gk=None, gv=None, scale=None, initial_state=None,
                        output_final_state=False, reverse=False, cu_seqlens=None,
                        dtype=np.float64):
    """Token-by-token recurrence: h_t = h_{t-1} e^{gk_t} e^{gv_t} + k_t^T v_t, o_t = (scale q_t)^T h_t.

    Follows ``fused_recurrent_gla_fwd_ref`` (``tops/ops/gla/fused_recurrent.py:17-132``);
    ``o`` and ``ht`` are floating point of ``dtype`` whatever the input type
    (the reference returns fp32 for both, ``fused_recurrent.py:261-263``).
    """
    q, k, v, gk, gv, h0 = (_f(x, dtype) for x in (q, k, v, gk, gv, initial_state))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    qf, kf, vf = q.reshape(-1, H, K), k.reshape(-1, H, K), v.reshape(-1, H, V)
    gkf = gk.reshape(-1, H, K) if gk is not None else None
    gvf = gv.reshape(-1, H, V) if gv is not None else None
    o = np.zeros((B * T, H, V), dtype)
    hts = []
    for n, (bos, eos) in enumerate(seq_bounds(B, T, cu_seqlens)):
        h = np.zeros((H, K, V), dtype) if h0 is None else h0[n].copy()
        ts = range(eos - 1, bos - 1, -1) if reverse else range(bos, eos)
        for t in ts:
            if gkf is not None:
                h = h * np.exp(gkf[t])[:, :, None]
            if gvf is not None:
                h = h * np.exp(gvf[t])[:, None, :]
            h = h + kf[t][:, :, None] * vf[t][:, None, :]
            o[t] = (h * (qf[t] * scale)[:, :, None]).sum(1)
        hts.append(h)
    ht = np.stack(hts, 0) if output_final_state else None
    return o.reshape(B, T, H, V), ht


def fused_recurrent_gla_bwd(q, k, v, gk=None, gv=None, do=None, dht=None, scale=None,
                            initial_state=None, reverse=False, cu_seqlens=None, dtype=np.float64):
    """Gradients of ``fused_recurrent_gla`` -> (dq, dk, dv, dgk, dgv, dh0).

    Follows the step derivation of the reference's CPU backward
    (``tests/src/ops/common/fused_recurrent.py:118-305``) and the gate-gradient
    formulation of ``tops/ops/gla/fused_recurrent.py:798-876``:
    dgk_t[k] = sum_v dh_t[k,v] (e^{gk_t} h_{t-1})[k,v] (gated previous state).
    dh0 is returned when ``initial_state`` is given.
    """
    q, k, v, gk, gv, do, dht, h0 = (_f(x, dtype) for x in (q, k, v, gk, gv, do, dht, initial_state))
    B, T, H, K = q.shape
    V = v.shape[-1]
    if scale is None:
        scale = K ** -0.5
    qf, kf, vf, dof = q.reshape(-1, H, K), k.reshape(-1, H, K), v.reshape(-1, H, V), do.reshape(-1, H, V)
    gkf = gk.reshape(-1, H, K) if gk is not None else None
    gvf = gv.reshape(-1, H, V) if gv is not None else None
    dq, dk = np.zeros_like(qf), np.zeros_like(kf)
    dv = np.zeros_like(vf)
    dgk = np.zeros_like(qf) if gk is not None else None
    dgv = np.zeros_like(vf) if gv is not None else None
    dh0s = []
    for n, (bos, eos) in enumerate(seq_bounds(B, T, cu_seqlens)):
        h = np.zeros((H, K, V), dtype) if h0 is None else h0[n].copy()
        order = list(range(eos - 1, bos - 1, -1)) if reverse else list(range(bos, eos))
        gated = {}
        for t in order:
            hg = h
            if gkf is not None:
                hg = hg * np.exp(gkf[t])[:, :, None]
            if gvf is not None:
                hg = hg * np.exp(gvf[t])[:, None, :]
            gated[t] = hg
            h = hg + kf[t][:, :, None] * vf[t][:, None, :]
            dq[t] = scale * (h * dof[t][:, None, :]).sum(-1)
        dh = np.zeros((H, K, V), dtype) if dht is None else dht[n].copy()
        for t in reversed(order):
            dh = dh + scale * qf[t][:, :, None] * dof[t][:, None, :]
            dk[t] = (dh * vf[t][:, None, :]).sum(-1)
            dv[t] = (dh * kf[t][:, :, None]).sum(-2)
            if gkf is not None:
                dgk[t] = (dh * gated[t]).sum(-1)
            if gvf is not None:
                dgv[t] = (dh * gated[t]).sum(-2)
            if gvf is not None:
                dh = dh * np.exp(gvf[t])[:, None, :]
            if gkf is not None:
                dh = dh * np.exp(gkf[t])[:, :, None]
        dh0s.append(dh)
    rs = lambda x, D: None if x is None else x.reshape(B, T, H, D)
    dh0 = np.stack(dh0s, 0) if h0 is not None else None
    return rs(dq, K), rs(dk, K), rs(dv, V), rs(dgk, K), rs(dgv, V), dh0


def naive_recurrent_gla(q, k, v, gk, scale=None, initial_state=None, output_final_state=False,
                        cu_seqlens=None, dtype=np.float64):
    """Definition of GLA as a step loop.  ``tops/ops/gla/naive.py:5-99``."""
    return fused_recurrent_gla(q, k, v, gk=gk, scale=scale, initial_state=initial_state,
                               output_final_state=output_final_state, cu_seqlens=cu_seqlens,
                               dtype=dtype)
