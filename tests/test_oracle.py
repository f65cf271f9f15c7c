"""Pin the numpy oracle against the reference's own outputs (CPU only).

Every fixture under ``tests/golden`` was produced by the reference's Torch CPU
restatement (``tests/golden/make_golden.py``).  The oracle must reproduce it
within fp32 rounding: the oracle runs in float64, the reference in float32.
"""
from __future__ import annotations

import numpy as np
import pytest

import cases as GC
from oracle import gla_oracle as O

FWD_TOL = dict(atol=2e-5, rtol=2e-5)
BWD_TOL = dict(atol=1e-4, rtol=1e-4)


def _close(name, got, want, atol, rtol):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{name}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    bound = atol + rtol * np.abs(want)
    bad = err > bound
    assert not bad.any(), f"{name}: max err {err.max():.3e} (worst ratio {(err / bound).max():.2f})"


@pytest.mark.parametrize("case", GC.CHUNK_CASES, ids=lambda c: c["name"])
def test_oracle_chunk_matches_reference(case):
    c, inp, fx = GC.load("chunk", case["name"])
    gc, A, h, ht, o = O.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g"], None, inp["scale"], inp["h0"],
                                      True, inp["cu"], inp["C"])
    _close("o", o, fx["o"], **FWD_TOL)
    _close("ht", ht, fx["ht"], **FWD_TOL)
    if "h" in fx:
        _close("g_cumsum", gc, fx["g_cumsum"], **FWD_TOL)
        _close("A", A, fx["A"], **FWD_TOL)
        _close("h", h, fx["h"], **FWD_TOL)
    if "dq" not in fx:
        return
    dq, dk, dv, dg, dh0 = O.chunk_gla_bwd(inp["q"], inp["k"], inp["v"], inp["g"], None, inp["scale"], inp["h0"],
                                          None, None, inp["do"], inp["dht"], inp["cu"], inp["C"])
    for nm, got in (("dq", dq), ("dk", dk), ("dv", dv), ("dg", dg)):
        _close(nm, got, fx[nm], **BWD_TOL)
    assert (dh0 is None) == ("dh0" not in fx)
    if dh0 is not None:
        _close("dh0", dh0, fx["dh0"], **BWD_TOL)
    if "dh" in fx:
        dh, _ = O.chunk_bwd_dh(inp["q"], inp["k"], inp["v"], gc, inp["do"], inp["h0"], inp["dht"], inp["scale"],
                               inp["cu"], inp["C"])
        _close("dh", dh, fx["dh"], **BWD_TOL)


@pytest.mark.parametrize("case", GC.REC_CASES, ids=lambda c: c["name"])
def test_oracle_recurrent_matches_reference(case):
    c, inp, fx = GC.load("rec", case["name"])
    o, ht = O.fused_recurrent_gla(inp["q"], inp["k"], inp["v"], inp["gk"], inp["gv"], inp["scale"], inp["h0"],
                                  True, inp["reverse"], inp["cu"])
    _close("o", o, fx["o"], **FWD_TOL)
    _close("ht", ht, fx["ht"], **FWD_TOL)
    dq, dk, dv, dgk, dgv, dh0 = O.fused_recurrent_gla_bwd(inp["q"], inp["k"], inp["v"], inp["gk"], inp["gv"],
                                                          inp["do"], inp["dht"], inp["scale"], inp["h0"],
                                                          inp["reverse"], inp["cu"])
    for nm, got in (("dq", dq), ("dk", dk), ("dv", dv), ("dgk", dgk), ("dgv", dgv), ("dh0", dh0)):
        if nm in fx:
            _close(nm, got, fx[nm], **BWD_TOL)
        else:
            assert got is None, nm
    if "naive_o" in fx:
        on, hn = O.naive_recurrent_gla(inp["q"], inp["k"], inp["v"], inp["gk"], inp["scale"], inp["h0"], True,
                                       inp["cu"])
        _close("naive_o", on, fx["naive_o"], **FWD_TOL)
        _close("naive_ht", hn, fx["naive_ht"], **FWD_TOL)


def test_oracle_chunk_equals_recurrent():
    """chunk == naive recurrence on a case with strong (un-normalised) gates."""
    rng = np.random.default_rng(5)
    B, T, H, K, V = 2, 77, 3, 16, 24
    q, k = rng.standard_normal((2, B, T, H, K))
    v = rng.standard_normal((B, T, H, V))
    g = GC.logsigmoid(rng.standard_normal((B, T, H, K)))
    h0 = rng.standard_normal((B, H, K, V))
    for C in (4, 16, 64):
        o1, s1 = O.chunk_gla(q, k, v, g, initial_state=h0, output_final_state=True, chunk_size=C)
        o2, s2 = O.naive_recurrent_gla(q, k, v, g, initial_state=h0, output_final_state=True)
        np.testing.assert_allclose(o1, o2, atol=1e-9, rtol=1e-9)
        np.testing.assert_allclose(s1, s2, atol=1e-9, rtol=1e-9)


def test_oracle_state_split():
    """Running two halves with the first half's final state equals the full run
    (the reference's ``test_state_split_pallas``)."""
    rng = np.random.default_rng(77)
    B, T, H, K, V = 1, 40, 2, 16, 32
    q, k = rng.standard_normal((2, B, T, H, K))
    v = rng.standard_normal((B, T, H, V))
    g = GC.logsigmoid(rng.standard_normal((B, T, H, K)))
    o, s = O.chunk_gla(q, k, v, g, output_final_state=True)
    o1, s1 = O.chunk_gla(q[:, :20], k[:, :20], v[:, :20], g[:, :20], output_final_state=True)
    o2, s2 = O.chunk_gla(q[:, 20:], k[:, 20:], v[:, 20:], g[:, 20:], initial_state=s1, output_final_state=True)
    np.testing.assert_allclose(np.concatenate([o1, o2], 1), o, atol=1e-10)
    np.testing.assert_allclose(s2, s, atol=1e-10)


def test_oracle_bwd_matches_finite_difference():
    """Gradients of the chunk form agree with central differences of the forward."""
    rng = np.random.default_rng(3)
    B, T, H, K, V, C = 1, 11, 1, 3, 2, 4
    q, k = rng.standard_normal((2, B, T, H, K))
    v = rng.standard_normal((B, T, H, V))
    g = GC.logsigmoid(rng.standard_normal((B, T, H, K)))
    h0 = rng.standard_normal((B, H, K, V))
    do = rng.standard_normal((B, T, H, V))
    dht = rng.standard_normal((B, H, K, V))

    def loss(q_, k_, v_, g_, h0_):
        o, s = O.chunk_gla(q_, k_, v_, g_, initial_state=h0_, output_final_state=True, chunk_size=C)
        return (o * do).sum() + (s * dht).sum()

    dq, dk, dv, dg, dh0 = O.chunk_gla_bwd(q, k, v, g, None, K ** -0.5, h0, None, None, do, dht, None, C)
    args = [q, k, v, g, h0]
    for i, grad in enumerate((dq, dk, dv, dg, dh0)):
        x = args[i]
        for idx in [tuple(rng.integers(0, s) for s in x.shape) for _ in range(6)]:
            e = 1e-6
            xp, xm = x.copy(), x.copy()
            xp[idx] += e
            xm[idx] -= e
            ap, am = list(args), list(args)
            ap[i], am[i] = xp, xm
            fd = (loss(*ap) - loss(*am)) / (2 * e)
            assert abs(fd - grad[idx]) < 1e-5 * max(1.0, abs(fd)), (i, idx, fd, grad[idx])
