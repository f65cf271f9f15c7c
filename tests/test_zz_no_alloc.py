"""The allocation-free chunk forward (tops_gla_chunk_fwd_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory or pass a workspace (a host
framework that hands an operator only its inputs and outputs, or a serving loop
that must not call the allocator).  Its scratch is a fixed array inside the
library.  This test checks that two calls in a row give the same results as the
regular entry point (tops_gla_chunk_fwd with a caller workspace) within the fp32
tolerance used by the other parity tests, and that a problem too large for the
fixed array is rejected with a clear error.  The file sorts last so that a run
stopping at the first failure has already run every other test.

Cases: the CUDA-core path (fp32 and bf16 at K=64, V=96); the tensor-core path (bf16,
K = V = 128), where the forward's saved block -- the chunk states and the gated q / k
copies the tcgen05 kernels read back through TMA -- lives in the fixed array, checked for
bit equality with the workspace entry point and against the oracle; and an ungated call
(g = None) right after a gated one, which must not read the gated call's leftovers.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _util import assert_close, assert_rel_l2
from oracle import gla_oracle as O

pytestmark = pytest.mark.gpu

FP32 = dict(atol=1e-4, rtol=1e-4)


def _args(_C, p, q, k, v, g, h0, o, ht, ws=None):
    return _C.ChunkFwdArgs(p.shape(), _C.ptr(q), _C.ptr(k), _C.ptr(v), _C.ptr(g), _C.ptr(h0), _C.ptr(o), _C.ptr(ht),
                           None, None, None, _C.ptr(ws), 0 if ws is None else ws.numel())


def _run_both(L, _C, p, q, k, v, g, h0, dtype, stream):
    """The workspace entry point, then the allocation-free one on NaN-filled outputs."""
    B, T, H, V = q.shape[0], q.shape[1], q.shape[2], v.shape[3]
    K = q.shape[3]
    o_ref = torch.empty(B, T, H, V, dtype=dtype, device="cuda")
    ht_ref = torch.empty(B, H, K, V, device="cuda")
    a = _args(_C, p, q, k, v, g, h0, o_ref, ht_ref)
    need = L.tops_gla_chunk_fwd_workspace_size(ctypes.byref(a))
    assert 0 < need <= 16 * 1024 * 1024
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    a = _args(_C, p, q, k, v, g, h0, o_ref, ht_ref, ws)
    assert L.tops_gla_chunk_fwd(ctypes.byref(a), stream) == 0, L.tops_gla_last_error()
    o = torch.full((B, T, H, V), float("nan"), dtype=dtype, device="cuda")
    ht = torch.full((B, H, K, V), float("nan"), device="cuda")
    b = _args(_C, p, q, k, v, g, h0, o, ht)
    rc = L.tops_gla_chunk_fwd_noalloc(ctypes.byref(b), stream)
    assert rc == 0, L.tops_gla_last_error()
    torch.cuda.synchronize()
    return o, ht, o_ref, ht_ref


def _inputs(seed, B, T, H, K, V, dtype):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q, k = (torch.randn(B, T, H, K, device="cuda", generator=gen).to(dtype) for _ in range(2))
    v = torch.randn(B, T, H, V, device="cuda", generator=gen).to(dtype)
    g = (torch.nn.functional.logsigmoid(torch.randn(B, T, H, K, device="cuda", generator=gen)) / 16).contiguous()
    h0 = torch.randn(B, H, K, V, device="cuda", generator=gen)
    return q, k, v, g, h0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_noalloc_matches_workspace_entry_point(dtype):
    from tops import _C
    from tops.ops.gla import _core
    L = _C.lib()
    B, T, H, K, V, C = 2, 200, 4, 64, 96, 64
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((1, 2)):  # two calls in a row, different inputs
        q, k, v, g, h0 = _inputs(seed, B, T, H, K, V, dtype)
        p = _core.make_plan(q, V, C, None, K ** -0.5)
        o_ref = torch.empty(B, T, H, V, dtype=dtype, device="cuda")
        ht_ref = torch.empty(B, H, K, V, device="cuda")
        a = _args(_C, p, q, k, v, g, h0, o_ref, ht_ref)
        need = L.tops_gla_chunk_fwd_workspace_size(ctypes.byref(a))
        assert 0 < need <= 16 * 1024 * 1024
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        a = _args(_C, p, q, k, v, g, h0, o_ref, ht_ref, ws)
        assert L.tops_gla_chunk_fwd(ctypes.byref(a), stream) == 0, L.tops_gla_last_error()
        o = torch.full((B, T, H, V), float("nan"), dtype=dtype, device="cuda")
        ht = torch.full((B, H, K, V), float("nan"), device="cuda")
        b = _args(_C, p, q, k, v, g, h0, o, ht)
        rc = L.tops_gla_chunk_fwd_noalloc(ctypes.byref(b), stream)
        assert rc == 0, L.tops_gla_last_error()
        torch.cuda.synchronize()
        assert_close(f"o (call {call})", o, o_ref, **FP32)
        assert_close(f"ht (call {call})", ht, ht_ref, **FP32)


def test_noalloc_tensor_core_path_bit_equal():
    """bf16 with K = V = 128 runs the tcgen05 kernels; their saved block sits in the fixed array."""
    from tops import _C
    from tops.ops.gla import _core
    L = _C.lib()
    if not L.tops_gla_has_tcgen05():
        pytest.skip("needs an sm_100 device for the tensor-core path")
    B, T, H, K, V, C = 2, 256, 2, 128, 128, 64
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((3, 4)):  # two calls in a row, different inputs
        q, k, v, g, h0 = _inputs(seed, B, T, H, K, V, torch.bfloat16)
        h0 = h0 * 0.1
        p = _core.make_plan(q, V, C, None, K ** -0.5)
        assert L.tops_gla_chunk_saved_size(ctypes.byref(p.shape())) > 0, "shape must take the tensor-core path"
        o, ht, o_ref, ht_ref = _run_both(L, _C, p, q, k, v, g, h0, torch.bfloat16, stream)
        # same kernels on the same inputs: bit for bit
        assert torch.equal(o, o_ref), f"o (call {call}) differs from the workspace entry point"
        assert torch.equal(ht, ht_ref), f"ht (call {call}) differs from the workspace entry point"
        qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
        o_r, ht_r = O.chunk_gla(qn, kn, vn, g.cpu().numpy(), initial_state=h0.cpu().numpy(),
                                output_final_state=True, chunk_size=C)
        assert_rel_l2(f"o vs oracle (call {call})", o, o_r, 2e-2)
        assert_rel_l2(f"ht vs oracle (call {call})", ht, ht_r, 2e-2)


def test_noalloc_ungated_after_gated_call():
    """A call with g = None right after a gated call sees none of the gated call's scratch."""
    from tops import _C
    from tops.ops.gla import _core
    L = _C.lib()
    B, T, H, K, V, C = 2, 200, 4, 64, 96, 64
    stream = torch.cuda.current_stream().cuda_stream
    q, k, v, g, h0 = _inputs(5, B, T, H, K, V, torch.float32)
    p = _core.make_plan(q, V, C, None, K ** -0.5)
    _run_both(L, _C, p, q, k, v, g, h0, torch.float32, stream)  # fills the array with gated sums
    q, k, v, _, h0 = _inputs(6, B, T, H, K, V, torch.float32)
    o, ht, o_ref, ht_ref = _run_both(L, _C, p, q, k, v, None, h0, torch.float32, stream)
    assert torch.equal(o, o_ref) and torch.equal(ht, ht_ref), "ungated call differs from the workspace entry point"
    o_r, ht_r = O.chunk_gla(*(x.cpu().numpy() for x in (q, k, v)), None, initial_state=h0.cpu().numpy(),
                            output_final_state=True, chunk_size=C)
    assert_close("o vs oracle (ungated)", o, o_r, **FP32)
    assert_close("ht vs oracle (ungated)", ht, ht_r, **FP32)


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    from tops import _C
    from tops.ops.gla import _core
    L = _C.lib()
    q = torch.empty(8, 4096, 4, 256, dtype=torch.bfloat16, device="cuda")
    p = _core.make_plan(q, 512, 64, None, None)
    a = _C.ChunkFwdArgs(p.shape(), 1, 1, 1, None, None, 1, None, None, None, None, None, 0)
    assert L.tops_gla_chunk_fwd_workspace_size(ctypes.byref(a)) > 16 * 1024 * 1024
    rc = L.tops_gla_chunk_fwd_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == -4  # TOPS_ERR_WORKSPACE, before anything is launched
    assert b"more than the fixed" in L.tops_gla_last_error()
