"""Token-by-token GLA (decode path) -- the API of ``tops.ops.gla.fused_recurrent``.

Mirrors the reference module (primatrix/pallas-kernel ``tops/ops/gla/fused_recurrent.py``):
``fused_recurrent_gla`` (:438), ``fused_recurrent_gla_fwd`` (:379) and
``fused_recurrent_gla_bwd`` (:879).  ``o`` and the final state are fp32 whatever
the input dtype, as in the reference (:261-263).  Differentiable through
``torch.autograd`` with the library's recurrent backward.
"""
from __future__ import annotations

import torch

from . import _core
from ._core import _cuda, _f32

__all__ = ["fused_recurrent_gla", "fused_recurrent_gla_fwd", "fused_recurrent_gla_bwd"]


def _bwd_operands(q, k, v, do):
    """q, k, v, do for the backward kernel, which takes do in the storage type of q, k, v.

    The forward output o is fp32, so its gradient arrives in fp32; the reference's backward
    reads that gradient as it is (fused_recurrent.py:626-790).  Rather than round it to a
    16-bit input type, the 16-bit q, k, v are widened to fp32 (exactly) and the kernel runs in
    fp32 on the same values.
    """
    if do.dtype == torch.float32 and q.dtype != torch.float32:
        return q.float(), k.float(), v.float(), do.contiguous()
    return q, k, v, do.contiguous().to(q.dtype)


def _validate(q, k, v, gk, gv, initial_state, cu_seqlens):
    B, T, H, K = q.shape
    V = v.shape[-1]
    cu = _core.host_cu(cu_seqlens)
    N = len(cu) - 1 if cu is not None else B
    assert k.shape == (B, T, H, K), f"Expected k shape {(B, T, H, K)}, got {tuple(k.shape)}"
    assert v.shape == (B, T, H, V), f"Expected v shape {(B, T, H, V)}, got {tuple(v.shape)}"
    assert (gk is None) or (gk.shape == (B, T, H, K)), f"Expected gk shape {(B, T, H, K)}, got {tuple(gk.shape)}"
    assert (gv is None) or (gv.shape == (B, T, H, V)), f"Expected gv shape {(B, T, H, V)}, got {tuple(gv.shape)}"
    assert (initial_state is None) or (initial_state.shape == (N, H, K, V)), \
        f"Expected initial_state shape {(N, H, K, V)}, got {tuple(initial_state.shape)}"
    assert (cu is None) or (B == 1), f"Batch size must be 1 when using cu_seqlens, got {B}"
    if cu is not None:
        assert cu[0] == 0 and cu[-1] == T, f"cu_seqlens must run from 0 to T={T}"
    cu_dev = None if cu is None else torch.tensor(cu, dtype=torch.int32, device=q.device)
    return N, cu_dev


class _FusedRecurrentGLA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, gk, gv, h0, scale, output_final_state, reverse, N, cu_dev):
        gkc, gvc, h0c = _f32("gk", gk), _f32("gv", gv), _f32("initial_state", h0)
        o, ht = _core.recurrent_fwd(q, k, v, gkc, gvc, h0c, scale, output_final_state, reverse, cu_dev, N)
        ctx.save_for_backward(q, k, v, gkc, gvc, h0c, o, cu_dev)
        ctx.meta = (scale, reverse, N, gk is not None and gk.dtype, gv is not None and gv.dtype)
        return (o, ht) if ht is not None else o

    @staticmethod
    def backward(ctx, do, dht=None):
        q, k, v, gkc, gvc, h0c, o, cu_dev = ctx.saved_tensors
        scale, reverse, N, gk_dt, gv_dt = ctx.meta
        qb, kb, vb, dob = _bwd_operands(q, k, v, do)
        dq, dk, dv, dgk, dgv, dh0 = _core.recurrent_bwd(qb, kb, vb, gkc, gvc, h0c, o, dob,
                                                        None if dht is None else dht.float().contiguous(), scale,
                                                        reverse, cu_dev, N)
        dq, dk, dv = dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)
        dgk = None if dgk is None else dgk.to(gk_dt)
        dgv = None if dgv is None else dgv.to(gv_dt)
        return dq, dk, dv, dgk, dgv, dh0, None, None, None, None, None


def fused_recurrent_gla_fwd(q, k, v, gk=None, gv=None, scale=None, initial_state=None, output_final_state=False,
                            reverse=False, cu_seqlens=None):
    """Validated forward: returns (o [B,T,H,V] fp32, ht [N,H,K,V] fp32 or None).  Mirrors :379."""
    N, cu_dev = _validate(q, k, v, gk, gv, initial_state, cu_seqlens)
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    out = _FusedRecurrentGLA.apply(q, k, v, gk, gv, initial_state, float(scale), bool(output_final_state),
                                   bool(reverse), N, cu_dev)
    if output_final_state:
        return out
    return out, None


def fused_recurrent_gla(q, k, v, gk=None, gv=None, scale=None, initial_state=None, output_final_state=False,
                        reverse=False, cu_seqlens=None):
    """Fused recurrent GLA (public API, FLA signature).  Mirrors tops/ops/gla/fused_recurrent.py:438.

    Args:
        q, k: [B, T, H, K]; v: [B, T, H, V]
        gk: [B, T, H, K] key-wise log-gate (optional); gv: [B, T, H, V] value-wise log-gate (optional)
        scale: default K ** -0.5; initial_state: [N, H, K, V]
        output_final_state: return the final state; reverse: iterate t = T-1 .. 0
        cu_seqlens: [N+1] cumulative lengths (B must be 1)
    Returns:
        o: [B, T, H, V] fp32; ht: [N, H, K, V] fp32 or None
    """
    return fused_recurrent_gla_fwd(q, k, v, gk=gk, gv=gv, scale=scale, initial_state=initial_state,
                                   output_final_state=output_final_state, reverse=reverse, cu_seqlens=cu_seqlens)


def fused_recurrent_gla_bwd(q, k, v, gk=None, gv=None, o=None, do=None, dht=None, scale=None, initial_state=None,
                            reverse=False, cu_seqlens=None):
    """Gradients (dq, dk, dv, dgk, dgv, dh0) of the recurrence.  Mirrors :879.

    ``o`` (the forward output) is required when ``gv`` is given, as in the reference.
    dq/dk/dv/dgk/dgv are fp32; dh0 is returned when initial_state is given.
    """
    N, cu_dev = _validate(q, k, v, gk, gv, initial_state, cu_seqlens)
    B, T, H, K = q.shape
    assert do is not None and do.shape == v.shape, f"Expected do shape {tuple(v.shape)}"
    assert (dht is None) or (dht.shape == (N, H, K, v.shape[-1])), "bad dht shape"
    assert gv is None or o is not None, "o (forward output) is required when gv is used"
    scale = scale if scale is not None else K ** -0.5
    q, k, v = (_cuda(n, x) for n, x in (("q", q), ("k", k), ("v", v)))
    q, k, v, do = _bwd_operands(q, k, v, _cuda("do", do))
    return _core.recurrent_bwd(q, k, v, _f32("gk", gk), _f32("gv", gv), _f32("initial_state", initial_state),
                               _f32("o", o), do, _f32("dht", dht), float(scale), bool(reverse), cu_dev, N)
