"""CPU checks of the C-ABI library: it builds, loads without a GPU, exports every
symbol declared in include/tops_gla.h, its struct layouts match the ctypes mirror,
and argument validation rejects bad calls before touching the device."""
from __future__ import annotations

import ctypes
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tops_gla.h"


@pytest.fixture(scope="module")
def lib():
    sys.path.insert(0, str(ROOT / "pallas-kernel_b200"))
    import build as B  # pallas-kernel_b200/build.py (incremental)
    B.build()
    from tops import _C
    return _C


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TOPS_API\s+[\w\s\*]+?\b(tops_gla_\w+)\s*\(", text)))


def test_header_declares_the_reference_ops():
    syms = declared_symbols()
    for need in ("tops_gla_chunk_fwd", "tops_gla_chunk_bwd", "tops_gla_recurrent_fwd", "tops_gla_recurrent_bwd",
                 "tops_gla_chunk_fwd_h", "tops_gla_chunk_bwd_dh", "tops_gla_state_combine"):
        assert need in syms


def test_library_exports_every_declared_symbol(lib):
    so = ctypes.CDLL(str(lib.LIB_PATH))
    missing = [s for s in declared_symbols() if not hasattr(so, s)]
    assert not missing, f"not exported: {missing}"
    assert set(declared_symbols()) == set(lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_struct_layouts_match_ctypes(lib, tmp_path):
    """Compile a C probe against the header and compare sizeof/offsetof with ctypes."""
    structs = {"tops_gla_shape": lib.Shape, "tops_gla_chunk_fwd_args": lib.ChunkFwdArgs,
               "tops_gla_xla_desc": lib.XlaDesc, "tops_gla_exchange_args": lib.ExchangeArgs,
               "tops_gla_chunk_bwd_args": lib.ChunkBwdArgs, "tops_gla_recurrent_args": lib.RecArgs,
               "tops_gla_recurrent_bwd_args": lib.RecBwdArgs, "tops_gla_p2p_args": lib.P2PArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(void){"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-o", str(exe), str(src)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for line in out:
        if line.strip():
            c, f, n = line.split()
            got[(c, f)] = int(n)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


def test_num_chunks_matches_host_plan(lib):
    L = lib.lib()
    assert L.tops_gla_num_chunks(3, 37, 16, None, 3, None) == 9
    cu = (ctypes.c_int32 * 4)(0, 13, 37, 50)
    offs = (ctypes.c_int32 * 4)()
    assert L.tops_gla_num_chunks(1, 50, 16, ctypes.cast(cu, ctypes.c_void_p), 3, ctypes.cast(offs, ctypes.c_void_p)) == 4
    assert list(offs) == [0, 1, 3, 4]
    bad = (ctypes.c_int32 * 3)(0, 10, 5)
    assert L.tops_gla_num_chunks(1, 10, 16, ctypes.cast(bad, ctypes.c_void_p), 2, None) == -1


def test_validation_rejects_bad_calls_without_a_device(lib):
    L = lib.lib()
    s = lib.Shape(2, 32, 4, 32, 64, 2, 4, 16, lib.BF16, 0.1, None, None)
    a = lib.ChunkFwdArgs(s, None, None, None, None, None, None, None, None, None, None, None, 0)
    assert L.tops_gla_chunk_fwd(ctypes.byref(a), None) == -1  # q/k/v/o missing
    assert b"required" in L.tops_gla_last_error()
    s2 = lib.Shape(2, 32, 4, 32, 64, 2, 4, 12, lib.BF16, 0.1, None, None)  # chunk 12 not a power of 2
    assert L.tops_gla_chunk_local_cumsum(ctypes.byref(s2), 1, 1, 0, 1.0, None) == -1
    s3 = lib.Shape(2, 32, 4, 32, 64, 2, 5, 16, lib.BF16, 0.1, None, None)  # wrong NT
    assert L.tops_gla_chunk_fwd_h(ctypes.byref(s3), 1, 1, 1, None, 1, None, None) == -1
    r = lib.RecArgs(2, 1, 4, 32, 64, 3, lib.BF16, 0.1, 0, None, 1, 1, 1, None, None, None, 1, None, None, 0)
    assert L.tops_gla_recurrent_fwd(ctypes.byref(r), None) == -1  # N != B without cu_seqlens
    assert L.tops_gla_abi_version() == 1


def test_workspace_queries_are_pure(lib):
    L = lib.lib()
    s = lib.Shape(8, 4096, 4, 256, 512, 8, 8 * 64, 64, lib.BF16, 0.0625, None, None)
    a = lib.ChunkFwdArgs(s, None, None, None, None, None, None, None, None, None, None, None, 0)
    n = L.tops_gla_chunk_fwd_workspace_size(ctypes.byref(a))
    assert n >= 8 * 4096 * 4 * (256 + 64) * 4  # g_cumsum + A (fp32) at least
    b = lib.ChunkBwdArgs(s, *([None] * 15), None, 0)
    assert L.tops_gla_chunk_bwd_workspace_size(ctypes.byref(b)) > n


def test_jax_frontend_imports_where_jax_exists():
    """The JAX custom-call frontend needs jax (absent on this image and the B200 box)."""
    pytest.importorskip("jax")
    import tops.jax as TJ  # noqa: F401
    assert callable(TJ.chunk_gla)


def test_noalloc_lookup_path_without_a_device(lib):
    """The allocation-free forward looks up its array's address per call; without a usable
    device that lookup fails with a CUDA status and a message, it neither crashes nor uses a
    host-side stand-in address.  Oversized problems are rejected before any lookup."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("checks the no-device path")
    L = lib.lib()
    s = lib.Shape(2, 32, 4, 32, 64, 2, 4, 16, lib.F32, 0.1, None, None)
    a = lib.ChunkFwdArgs(s, 1, 1, 1, None, None, 1, None, None, None, None, None, 0)
    rc = L.tops_gla_chunk_fwd_noalloc(ctypes.byref(a), None)
    assert rc == -3, rc  # TOPS_ERR_CUDA
    assert b"chunk_fwd_noalloc" in L.tops_gla_last_error()
    big = lib.Shape(8, 4096, 4, 256, 512, 8, 8 * 64, 64, lib.F32, 0.0625, None, None)
    b = lib.ChunkFwdArgs(big, 1, 1, 1, None, None, 1, None, None, None, None, None, 0)
    assert L.tops_gla_chunk_fwd_noalloc(ctypes.byref(b), None) == -4  # TOPS_ERR_WORKSPACE
    assert b"more than the fixed" in L.tops_gla_last_error()


def test_xla_custom_call_failure_reaches_the_status(lib, tmp_path):
    """A malformed descriptor given to an XLA custom-call target is reported through
    XlaCustomCallStatusSetFailure (resolved from the host process at run time; here a C
    stand-in loaded globally) before anything touches the device."""
    src, so = tmp_path / "status.c", tmp_path / "libxla_status_standin.so"
    src.write_text("#include <stddef.h>\n#include <string.h>\n"
                   "void XlaCustomCallStatusSetFailure(void* st, const char* m, size_t n) {"
                   " char* s = (char*)st; size_t k = n < 254 ? n : 254; s[0] = 1; memcpy(s + 1, m, k); s[1 + k] = 0; }\n")
    subprocess.run(["gcc", "-shared", "-fPIC", str(src), "-o", str(so)], check=True)
    ctypes.CDLL(str(so), mode=ctypes.RTLD_GLOBAL)
    L = lib.lib()
    for name in ("tops_gla_xla_chunk_fwd", "tops_gla_xla_chunk_bwd", "tops_gla_xla_recurrent_fwd"):
        st = ctypes.create_string_buffer(256)
        arr = (ctypes.c_void_p * 1)(None)
        getattr(L, name)(None, ctypes.cast(arr, ctypes.c_void_p), b"\x00" * 7, 7, ctypes.cast(st, ctypes.c_void_p))
        assert st.raw[0] == 1, name
        assert b"bad descriptor" in st.raw, st.raw[:80]


def test_nccl_failure_entry_points_validate_without_a_device(lib):
    """Abort of a NULL communicator is a no-op; the check and the bounded wait reject a NULL
    communicator or a non-positive timeout before touching NCCL or the device."""
    L = lib.lib()
    assert L.tops_gla_nccl_comm_abort(None) == 0
    assert L.tops_gla_nccl_comm_check(None) == -1
    assert b"comm is NULL" in L.tops_gla_last_error()
    assert L.tops_gla_state_exchange_wait(None, None, 100) == -1
    assert L.tops_gla_state_exchange_wait(1, None, 0) == -1
    assert b"positive timeout" in L.tops_gla_last_error()


def test_p2p_exchange_entry_points_validate_without_a_device(lib):
    """The peer-memory exchange sizes its region from the shape alone and rejects bad ranks,
    missing buffers and a non-positive timeout before launching anything; freeing or closing a
    NULL region is a no-op."""
    import ctypes
    L = lib.lib()
    a = lib.P2PArgs(0, 2, 1, 16, 128, 128, 0, None, None, None, None, None, None, None, 1000)
    per = 16 * 128 * 128 + 16 * 128
    assert L.tops_gla_p2p_region_size(ctypes.byref(a)) == 4096 + 2 * 2 * per * 4
    assert L.tops_gla_p2p_exchange(ctypes.byref(a), None) == -1  # no buffers
    a.local_state = a.decay = a.out = a.regions = a.own_region = 16
    a.rank = 2
    assert L.tops_gla_p2p_exchange(ctypes.byref(a), None) == -1
    assert b"rank / world" in L.tops_gla_last_error()
    a.rank, a.world = 0, 65
    assert L.tops_gla_p2p_region_size(ctypes.byref(a)) == 0
    a.world, a.timeout_ms = 2, 0
    assert L.tops_gla_p2p_exchange(ctypes.byref(a), None) == -1
    assert b"timeout_ms" in L.tops_gla_last_error()
    assert L.tops_gla_p2p_free(None) == 0 and L.tops_gla_ipc_close(None) == 0
    assert L.tops_gla_ipc_handle(None, None) == -1
