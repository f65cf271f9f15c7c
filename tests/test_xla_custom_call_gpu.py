"""The XLA custom-call targets (the JAX frontend's boundary), driven through ctypes.

JAX is not installable on this image or the B200 pool, so the custom calls are invoked
the way XLA invokes a status-returning legacy custom call: the stream, a `void*` array
holding the operand buffers followed by the result buffers, the opaque descriptor bytes
(a packed `tops_gla_xla_desc`) and an `XlaCustomCallStatus*`.  The library resolves
`XlaCustomCallStatusSetFailure` from the hosting process at run time; here a two-line C
stand-in (compiled with gcc into the test's temporary directory and loaded globally)
records what the library reports, so a failing call is seen as a failure and not only
as wrong outputs.  Buffer order follows csrc/xla_custom_call.cu (documented in
INTEGRATION.md).  Outputs and gradients are checked against the oracle: bf16 within
relative L2 2e-2 (tensor-core path), fp32 within max-abs/rel 1e-4 (CUDA-core path).
Reference boundary: tops/ops/gla/__init__.py:1-34, tops/ops/gla/chunk.py:1187-1251.
"""
from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest
import torch

from _util import assert_close, assert_rel_l2
from oracle import gla_oracle as O

pytestmark = pytest.mark.gpu

BF16_L2 = 2e-2
FP32 = dict(atol=1e-4, rtol=1e-4)

_STATUS_SRC = r"""
#include <stddef.h>
#include <string.h>
/* stand-in for XLA's status setter: status points at a 256-byte buffer, byte 0 = failed */
void XlaCustomCallStatusSetFailure(void* status, const char* msg, size_t len) {
  char* s = (char*)status;
  size_t n = len < 254 ? len : 254;
  s[0] = 1;
  memcpy(s + 1, msg, n);
  s[1 + n] = 0;
}
"""


@pytest.fixture(scope="module")
def xla(tmp_path_factory):
    from tops import _C
    L = _C.lib()
    d = tmp_path_factory.mktemp("xla_status")
    src, so = d / "status.c", d / "libxla_status_standin.so"
    src.write_text(_STATUS_SRC)
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", str(src), "-o", str(so)], check=True)
    keep = ctypes.CDLL(str(so), mode=ctypes.RTLD_GLOBAL)  # visible to dlsym(RTLD_DEFAULT, ...)
    return _C, L, keep


class Status:
    def __init__(self):
        self.buf = ctypes.create_string_buffer(256)

    @property
    def ptr(self):
        return ctypes.cast(self.buf, ctypes.c_void_p)

    def check(self, what):
        assert self.buf.raw[0] == 0, f"{what} reported failure: {self.buf.raw[1:].split(b'\x00')[0].decode()}"


def _call(L, name, stream, bufs, desc):
    arr = (ctypes.c_void_p * len(bufs))(*[None if b is None else b for b in bufs])
    st = Status()
    raw = bytes(desc)
    getattr(L, name)(ctypes.c_void_p(stream), ctypes.cast(arr, ctypes.c_void_p), raw, len(raw), st.ptr)
    torch.cuda.synchronize()
    return st


def _inputs(seed, B, T, H, K, V, dtype):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k = (torch.randn(B, T, H, K, device="cuda", generator=gen).to(dtype) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", generator=gen).to(dtype)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda", generator=gen)) / 16).contiguous()
    h0 = torch.randn(B, H, K, V, device="cuda", generator=gen) * 0.1
    do = torch.randn(B, T, H, V, device="cuda", generator=gen).to(dtype)
    dht = torch.randn(B, H, K, V, device="cuda", generator=gen) * 0.1
    return q, k, v, g, h0, do, dht


def _np(x):
    return x.detach().float().cpu().numpy()


@pytest.mark.parametrize("dtype,shape", [
    (torch.bfloat16, (2, 256, 2, 128, 128)),   # tensor-core path
    (torch.float32, (2, 100, 3, 64, 48)),      # CUDA-core path, ragged last chunk
], ids=["bf16_tc", "f32_simt"])
def test_xla_chunk_fwd_bwd(xla, dtype, shape):
    _C, L, _ = xla
    B, T, H, K, V = shape
    C = 64
    scale = K ** -0.5
    q, k, v, g, h0, do, dht = _inputs(11, B, T, H, K, V, dtype)
    dt = _C._DTYPE[dtype]
    stream = torch.cuda.current_stream().cuda_stream
    # sizes the host (XLA's lowering) asks the library for, through the regular entry points
    sh = _C.Shape(B, T, H, K, V, B, B * ((T + C - 1) // C), C, dt, scale, None, None)
    saved_bytes = L.tops_gla_chunk_saved_size(ctypes.byref(sh))
    saved = torch.empty(max(saved_bytes, 1), dtype=torch.uint8, device="cuda")
    fa = _C.ChunkFwdArgs(sh, 1, 1, 1, 1, 1, 1, 1, None, None, None, None, 0,
                         _C.ptr(saved) if saved_bytes else None, saved_bytes)
    fws = L.tops_gla_chunk_fwd_workspace_size(ctypes.byref(fa))
    ws_f = torch.empty(max(fws, 1), dtype=torch.uint8, device="cuda")
    o = torch.full((B, T, H, V), float("nan"), dtype=dtype, device="cuda")
    ht = torch.full((B, H, K, V), float("nan"), device="cuda")
    desc = _C.XlaDesc(B, T, H, K, V, C, dt, scale, 1, 1, 1, 1, 1, 0, saved_bytes, fws)
    # fwd buffers: q, k, v, g, h0 | o, ht, saved, workspace
    st = _call(L, "tops_gla_xla_chunk_fwd", stream,
               [_C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(o), _C.ptr(ht),
                _C.ptr(saved) if saved_bytes else None, _C.ptr(ws_f)], desc)
    st.check("tops_gla_xla_chunk_fwd")
    qn, kn, vn, gn, h0n, don, dhtn = (_np(x) for x in (q, k, v, g, h0, do, dht))
    o_r, ht_r = O.chunk_gla(qn, kn, vn, gn, scale=scale, initial_state=h0n, output_final_state=True, chunk_size=C)
    dq_r, dk_r, dv_r, dg_r, dh0_r = O.chunk_gla_bwd(qn, kn, vn, gn, None, scale, h0n, None, None, don, dhtn, None, C)

    ba = _C.ChunkBwdArgs(sh, *([1] * 4), 1, 1, 1, None, None, None, 1, 1, 1, 1, 1, None, 0,
                         _C.ptr(saved) if saved_bytes else None, saved_bytes)
    bws = L.tops_gla_chunk_bwd_workspace_size(ctypes.byref(ba))
    assert bws > 0, L.tops_gla_last_error()
    ws_b = torch.empty(bws, dtype=torch.uint8, device="cuda")
    dq, dk = (torch.full((B, T, H, K), float("nan"), dtype=dtype, device="cuda") for _ in range(2))
    dv = torch.full((B, T, H, V), float("nan"), dtype=dtype, device="cuda")
    dg = torch.full((B, T, H, K), float("nan"), device="cuda")
    dh0 = torch.full((B, H, K, V), float("nan"), device="cuda")
    desc_b = _C.XlaDesc(B, T, H, K, V, C, dt, scale, 1, 1, 1, 1, 1, 0, saved_bytes, bws)
    # bwd buffers: q, k, v, g, h0, do, dht, saved | dq, dk, dv, dg, dh0, workspace
    st = _call(L, "tops_gla_xla_chunk_bwd", stream,
               [_C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(do), _C.ptr(dht),
                _C.ptr(saved) if saved_bytes else None,
                _C.ptr(dq), _C.ptr(dk), _C.ptr(dv), _C.ptr(dg), _C.ptr(dh0), _C.ptr(ws_b)], desc_b)
    st.check("tops_gla_xla_chunk_bwd")
    got = {"o": (o, o_r), "ht": (ht, ht_r), "dq": (dq, dq_r), "dk": (dk, dk_r), "dv": (dv, dv_r),
           "dg": (dg, dg_r), "dh0": (dh0, dh0_r)}
    for nm, (t, r) in got.items():
        if dtype == torch.float32:
            assert_close(nm, t, r, **FP32)
        else:
            assert_rel_l2(nm, t, r, BF16_L2)


def test_xla_recurrent_fwd(xla):
    _C, L, _ = xla
    B, T, H, K, V = 8, 1, 4, 128, 128  # a decode step (BASELINE config 2 distributions, reduced batch)
    scale = K ** -0.5
    q, k, v, g, h0, _, _ = _inputs(12, B, T, H, K, V, torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    ra = _C.RecArgs(B, T, H, K, V, B, _C.BF16, scale, 0, None, 1, 1, 1, 1, None, 1, 1, 1, None, 0)
    ws_n = L.tops_gla_recurrent_fwd_workspace_size(ctypes.byref(ra))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device="cuda")
    o = torch.full((B, T, H, V), float("nan"), device="cuda")
    ht = torch.full((B, H, K, V), float("nan"), device="cuda")
    desc = _C.XlaDesc(B, T, H, K, V, 64, _C.BF16, scale, 1, 1, 1, 0, 0, 0, 0, ws_n)
    # buffers: q, k, v, gk, h0 | o, ht, workspace
    st = _call(L, "tops_gla_xla_recurrent_fwd", stream,
               [_C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(o), _C.ptr(ht), _C.ptr(ws)], desc)
    st.check("tops_gla_xla_recurrent_fwd")
    o_r, ht_r = O.fused_recurrent_gla(_np(q), _np(k), _np(v), _np(g), None, scale, _np(h0), True)
    assert_rel_l2("o", o, o_r, BF16_L2)
    assert_rel_l2("ht", ht, ht_r, BF16_L2)

