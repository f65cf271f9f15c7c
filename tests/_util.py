"""Comparison helpers shared by the tests (tolerances are stated at each call site)."""
from __future__ import annotations

import numpy as np


def to_np(x):
    if x is None:
        return None
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().float().cpu().numpy().astype(np.float64)
    except ImportError:
        pass
    return np.asarray(x, dtype=np.float64)


def assert_close(name, got, want, atol, rtol):
    """|got - want| <= atol + rtol * |want| elementwise (max-abs/rel criterion)."""
    g, w = to_np(got), to_np(want)
    assert g is not None and w is not None, f"{name}: missing tensor"
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    assert np.isfinite(g).all(), f"{name}: non-finite values"
    err = np.abs(g - w)
    bound = atol + rtol * np.abs(w)
    worst = float((err / bound).max()) if err.size else 0.0
    assert worst <= 1.0, f"{name}: max abs err {err.max():.3e}, worst err/tol ratio {worst:.2f}"


def rel_l2(got, want) -> float:
    g, w = to_np(got), to_np(want)
    return float(np.linalg.norm((g - w).ravel()) / max(np.linalg.norm(w.ravel()), 1e-30))


def assert_rel_l2(name, got, want, tol):
    g, w = to_np(got), to_np(want)
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    assert np.isfinite(g).all(), f"{name}: non-finite values"
    r = rel_l2(g, w)
    assert r <= tol, f"{name}: relative L2 error {r:.3e} > {tol}"


def assert_max_rel(name, got, want, tol):
    """Element-wise bound relative to the tensor's scale: max |got - want| <= tol * max |want|.
    Catches one bad tile or row that a relative-L2 check over a large tensor would average away."""
    g, w = to_np(got), to_np(want)
    assert g.shape == w.shape, f"{name}: shape {g.shape} != {w.shape}"
    assert np.isfinite(g).all(), f"{name}: non-finite values"
    err = float(np.abs(g - w).max()) if g.size else 0.0
    scale = float(np.abs(w).max()) if w.size else 0.0
    assert err <= tol * max(scale, 1e-30), f"{name}: max abs error {err:.3e} > {tol} x max |ref| {scale:.3e}"
