"""jax.custom_vjp wiring of the B200 GLA kernels via XLA custom calls.

Targets the JAX version the reference pins (jax 0.6.2, ``uv.lock``).  JAX is not
installable on the build/test machines of this repository, so this module is
import-guarded and exercised only by hosts that have JAX; the C entry points it
calls (``tops_gla_xla_chunk_fwd/bwd``, ``tops_gla_xla_recurrent_fwd``) are tested
for export and layout on CPU, and the kernels behind them by the torch frontend.

Buffer conventions (see csrc/xla_custom_call.cu): the opaque descriptor carries
the shape, dtype, scale and flags; the forward returns (o, ht, saved, workspace)
where ``saved`` is the opaque block the backward consumes as a residual.
"""
from __future__ import annotations

import ctypes
import functools

import jax  # noqa: F401  (ImportError here means: no JAX on this host)
import jax.numpy as jnp
from jax.interpreters import mlir

from .. import _C

_DT = {jnp.dtype(jnp.float32): _C.F32, jnp.dtype(jnp.bfloat16): _C.BF16, jnp.dtype(jnp.float16): _C.F16}
_REGISTERED = False


def _register():
    global _REGISTERED
    if _REGISTERED:
        return
    lib = _C.lib()
    for name in ("tops_gla_xla_chunk_fwd", "tops_gla_xla_chunk_bwd", "tops_gla_xla_recurrent_fwd"):
        fn = ctypes.cast(getattr(lib, name), ctypes.c_void_p).value
        capsule = jax.ffi.pycapsule(ctypes.cast(fn, ctypes.CFUNCTYPE(None)))
        jax.ffi.register_ffi_target(name, capsule, platform="CUDA", api_version=0)
    _REGISTERED = True


def _desc(**kw) -> bytes:
    d = _C.XlaDesc(**kw)
    return bytes(memoryview(d).cast("B"))


def _sizes(B, T, H, K, V, C, dtype, has_g):
    """(saved bytes, fwd workspace bytes, bwd workspace bytes) from the library's own queries."""
    s = _C.Shape(B, T, H, K, V, B, B * ((T + C - 1) // C), C, dtype, 0.0, None, None)
    lib = _C.lib()
    saved = int(lib.tops_gla_chunk_saved_size(ctypes.byref(s))) if has_g else 0
    fa = _C.ChunkFwdArgs(s, 1, 1, 1, 1 if has_g else None, None, 1, None, None, None, None, None, 0,
                         1 if saved else None, saved)
    ba = _C.ChunkBwdArgs(s, 1, 1, 1, 1 if has_g else None, None, 1, None, None, None, None, 1, 1, 1, 1, None, None,
                         0, 1 if saved else None, saved)
    return saved, int(lib.tops_gla_chunk_fwd_workspace_size(ctypes.byref(fa))), \
        int(lib.tops_gla_chunk_bwd_workspace_size(ctypes.byref(ba)))


def _custom_call(name, operands, result_avals, opaque):
    def lowering(ctx, *args):
        out_types = [mlir.aval_to_ir_type(a) for a in ctx.avals_out]
        return mlir.custom_call(name, result_types=out_types, operands=list(args), backend_config=opaque,
                                api_version=2).results

    prim = jax.extend.core.Primitive(name + "_" + str(abs(hash(opaque))))
    prim.multiple_results = True
    prim.def_impl(functools.partial(jax.interpreters.xla.apply_primitive, prim))
    prim.def_abstract_eval(lambda *a: result_avals)
    mlir.register_lowering(prim, lowering, platform="cuda")
    return prim.bind(*operands)


@functools.partial(jax.custom_vjp, nondiff_argnums=(5, 6, 7))
def _chunk_gla(q, k, v, g, h0, scale, output_final_state, chunk_size):
    o, ht, _ = _chunk_fwd(q, k, v, g, h0, scale, output_final_state, chunk_size)
    return o, ht


def _chunk_fwd(q, k, v, g, h0, scale, output_final_state, chunk_size):
    _register()
    B, T, H, K = q.shape
    V = v.shape[-1]
    dt = _DT[jnp.dtype(q.dtype)]
    saved, ws_f, _ = _sizes(B, T, H, K, V, chunk_size, dt, True)
    opaque = _desc(B=B, T=T, H=H, K=K, V=V, chunk_size=chunk_size, dtype=dt, scale=scale, has_g=1,
                   has_h0=int(h0 is not None), out_final=1, saved_bytes=saved, workspace_bytes=ws_f)
    ops = [q, k, v, g.astype(jnp.float32)] + ([h0.astype(jnp.float32)] if h0 is not None else [])
    avals = [jax.core.ShapedArray((B, T, H, V), q.dtype), jax.core.ShapedArray((B, H, K, V), jnp.float32),
             jax.core.ShapedArray((max(saved, 1),), jnp.uint8), jax.core.ShapedArray((max(ws_f, 1),), jnp.uint8)]
    o, ht, blk, _ = _custom_call("tops_gla_xla_chunk_fwd", ops, avals, opaque)
    return o, (ht if output_final_state else None), blk


def _chunk_gla_fwd(q, k, v, g, h0, scale, output_final_state, chunk_size):
    o, ht, blk = _chunk_fwd(q, k, v, g, h0, scale, output_final_state, chunk_size)
    return (o, ht), (q, k, v, g, h0, blk)


def _chunk_gla_bwd(scale, output_final_state, chunk_size, res, cts):
    q, k, v, g, h0, blk = res
    do, dht = cts
    B, T, H, K = q.shape
    V = v.shape[-1]
    dt = _DT[jnp.dtype(q.dtype)]
    saved, _, ws_b = _sizes(B, T, H, K, V, chunk_size, dt, True)
    want_dh0 = h0 is not None
    opaque = _desc(B=B, T=T, H=H, K=K, V=V, chunk_size=chunk_size, dtype=dt, scale=scale, has_g=1,
                   has_h0=int(want_dh0), has_dht=int(dht is not None), want_dh0=int(want_dh0),
                   saved_bytes=saved, workspace_bytes=ws_b)
    ops = [q, k, v, g.astype(jnp.float32)] + ([h0.astype(jnp.float32)] if want_dh0 else []) + [do.astype(q.dtype)]
    ops += ([dht.astype(jnp.float32)] if dht is not None else []) + [blk]
    avals = [jax.core.ShapedArray(q.shape, q.dtype), jax.core.ShapedArray(k.shape, k.dtype),
             jax.core.ShapedArray(v.shape, v.dtype), jax.core.ShapedArray(q.shape, jnp.float32)]
    if want_dh0:
        avals.append(jax.core.ShapedArray((B, H, K, V), jnp.float32))
    avals.append(jax.core.ShapedArray((max(ws_b, 1),), jnp.uint8))
    res_ = _custom_call("tops_gla_xla_chunk_bwd", ops, avals, opaque)
    dq, dk, dv, dg = res_[:4]
    dh0 = res_[4] if want_dh0 else None
    return dq, dk, dv, dg.astype(g.dtype), dh0


_chunk_gla.defvjp(_chunk_gla_fwd, _chunk_gla_bwd)


def chunk_gla(q, k, v, g=None, g_gamma=None, scale=None, initial_state=None, output_final_state=False,
              cu_seqlens=None, chunk_size=16):
    """Same contract as the reference's tops.ops.gla.chunk_gla (tops/ops/gla/chunk.py:1187).

    Variable-length input (cu_seqlens) is served by the torch frontend only.
    """
    assert cu_seqlens is None, "cu_seqlens is not wired through the JAX custom call"
    if g is None:
        g = jnp.broadcast_to(g_gamma, q.shape) if g_gamma is not None else jnp.zeros(q.shape, jnp.float32)
    if scale is None:
        scale = q.shape[-1] ** -0.5
    o, ht = _chunk_gla(q, k, v, g, initial_state, float(scale), bool(output_final_state), int(chunk_size))
    return o, (ht if output_final_state else None)


def fused_chunk_gla(q, k, v, g, scale=None, initial_state=None, output_final_state=False, cu_seqlens=None,
                    chunk_size=16):
    """Alias of chunk_gla (reference tops/ops/gla/fused_chunk.py:4)."""
    return chunk_gla(q, k, v, g, scale=scale, initial_state=initial_state, output_final_state=output_final_state,
                     cu_seqlens=cu_seqlens, chunk_size=chunk_size)


def fused_recurrent_gla(q, k, v, gk=None, gv=None, scale=None, initial_state=None, output_final_state=False,
                        reverse=False, cu_seqlens=None):
    """Forward of the recurrence (reference tops/ops/gla/fused_recurrent.py:438); o and ht are fp32."""
    assert gv is None and cu_seqlens is None, "gv / cu_seqlens are served by the torch frontend only"
    _register()
    B, T, H, K = q.shape
    V = v.shape[-1]
    dt = _DT[jnp.dtype(q.dtype)]
    if scale is None:
        scale = K ** -0.5
    a = _C.RecArgs(B, T, H, K, V, B, dt, float(scale), int(reverse), None, 1, 1, 1, 1 if gk is not None else None,
                   None, None, 1, None, None, 0)
    ws = int(_C.lib().tops_gla_recurrent_fwd_workspace_size(ctypes.byref(a)))
    opaque = _desc(B=B, T=T, H=H, K=K, V=V, chunk_size=1, dtype=dt, scale=float(scale), has_g=int(gk is not None),
                   has_h0=int(initial_state is not None), out_final=1, reverse=int(reverse), workspace_bytes=ws)
    ops = [q, k, v] + ([gk.astype(jnp.float32)] if gk is not None else []) + \
        ([initial_state.astype(jnp.float32)] if initial_state is not None else [])
    avals = [jax.core.ShapedArray((B, T, H, V), jnp.float32), jax.core.ShapedArray((B, H, K, V), jnp.float32),
             jax.core.ShapedArray((max(ws, 1),), jnp.uint8)]
    o, ht, _ = _custom_call("tops_gla_xla_recurrent_fwd", ops, avals, opaque)
    return o, (ht if output_final_state else None)

