"""ctypes binding of libtops_gla.so (the C ABI declared in include/tops_gla.h).

The library is the product: there is no fallback.  If it has not been built the
first call raises ``ImportError`` naming the build command, and every non-zero
status of the C ABI is raised as :class:`TopsError` with the library's message.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtops_gla.so"

F32, BF16, F16 = 0, 1, 2
_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


class TopsError(RuntimeError):
    """A libtops_gla call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed with status {status}: {msg}")
        self.status = status


class Shape(C.Structure):
    _fields_ = [("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("K", C.c_int32), ("V", C.c_int32),
                ("N", C.c_int32), ("NT", C.c_int32), ("chunk_size", C.c_int32), ("dtype", C.c_int32),
                ("scale", C.c_float), ("cu_seqlens", C.c_void_p), ("chunk_offsets", C.c_void_p)]


class ChunkFwdArgs(C.Structure):
    _fields_ = [("s", Shape), ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("g", C.c_void_p),
                ("h0", C.c_void_p), ("o", C.c_void_p), ("ht", C.c_void_p), ("g_cumsum", C.c_void_p),
                ("A", C.c_void_p), ("h", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
                ("saved", C.c_void_p), ("saved_bytes", C.c_size_t)]


class ChunkBwdArgs(C.Structure):
    _fields_ = [("s", Shape), ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("g", C.c_void_p),
                ("h0", C.c_void_p), ("do_", C.c_void_p), ("dht", C.c_void_p), ("g_cumsum", C.c_void_p),
                ("A", C.c_void_p), ("h", C.c_void_p), ("dq", C.c_void_p), ("dk", C.c_void_p), ("dv", C.c_void_p),
                ("dg", C.c_void_p), ("dh0", C.c_void_p), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_size_t), ("saved", C.c_void_p), ("saved_bytes", C.c_size_t)]


class RecArgs(C.Structure):
    _fields_ = [("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("K", C.c_int32), ("V", C.c_int32),
                ("N", C.c_int32), ("dtype", C.c_int32), ("scale", C.c_float), ("reverse", C.c_int32),
                ("cu_seqlens", C.c_void_p), ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p),
                ("gk", C.c_void_p), ("gv", C.c_void_p), ("h0", C.c_void_p), ("o", C.c_void_p), ("ht", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class RecBwdArgs(C.Structure):
    _fields_ = [("f", RecArgs), ("o", C.c_void_p), ("do_", C.c_void_p), ("dht", C.c_void_p), ("dq", C.c_void_p),
                ("dk", C.c_void_p), ("dv", C.c_void_p), ("dgk", C.c_void_p), ("dgv", C.c_void_p),
                ("dh0", C.c_void_p)]


class XlaDesc(C.Structure):
    _fields_ = [("B", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("K", C.c_int32), ("V", C.c_int32),
                ("chunk_size", C.c_int32), ("dtype", C.c_int32), ("scale", C.c_float), ("has_g", C.c_int32),
                ("has_h0", C.c_int32), ("out_final", C.c_int32), ("has_dht", C.c_int32), ("want_dh0", C.c_int32),
                ("reverse", C.c_int32), ("saved_bytes", C.c_uint64), ("workspace_bytes", C.c_uint64)]


class ExchangeArgs(C.Structure):
    _fields_ = [("comm", C.c_void_p), ("rank", C.c_int32), ("world", C.c_int32), ("N", C.c_int32), ("H", C.c_int32),
                ("K", C.c_int32), ("V", C.c_int32), ("backward", C.c_int32), ("local_state", C.c_void_p),
                ("decay", C.c_void_p), ("boundary", C.c_void_p), ("out", C.c_void_p), ("total", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class P2PArgs(C.Structure):
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("N", C.c_int32), ("H", C.c_int32), ("K", C.c_int32),
                ("V", C.c_int32), ("backward", C.c_int32), ("local_state", C.c_void_p), ("decay", C.c_void_p),
                ("boundary", C.c_void_p), ("out", C.c_void_p), ("total", C.c_void_p), ("regions", C.c_void_p),
                ("own_region", C.c_void_p), ("timeout_ms", C.c_int32)]


IPC_HANDLE_BYTES = 64
VP, I32, F32C = C.c_void_p, C.c_int32, C.c_float
SIGNATURES = {
    "tops_gla_last_error": (C.c_char_p, []),
    "tops_gla_abi_version": (I32, []),
    "tops_gla_launch_count": (C.c_uint64, []),
    "tops_gla_timing_enable": (None, [I32]),
    "tops_gla_timing_collect": (I32, [C.c_char_p, I32, C.POINTER(C.c_float), I32]),
    "tops_gla_has_tcgen05": (I32, []),
    "tops_gla_device_error": (I32, []),
    "tops_gla_selftest_wait_timeout": (C.c_int, [VP]),
    "tops_gla_num_chunks": (I32, [I32, I32, I32, VP, I32, VP]),
    "tops_gla_chunk_fwd": (C.c_int, [C.POINTER(ChunkFwdArgs), VP]),
    "tops_gla_chunk_fwd_workspace_size": (C.c_size_t, [C.POINTER(ChunkFwdArgs)]),
    "tops_gla_chunk_saved_size": (C.c_size_t, [C.POINTER(Shape)]),
    "tops_gla_chunk_bwd": (C.c_int, [C.POINTER(ChunkBwdArgs), VP]),
    "tops_gla_chunk_fwd_noalloc": (C.c_int, [C.POINTER(ChunkFwdArgs), VP]),
    "tops_gla_chunk_bwd_workspace_size": (C.c_size_t, [C.POINTER(ChunkBwdArgs)]),
    "tops_gla_recurrent_fwd": (C.c_int, [C.POINTER(RecArgs), VP]),
    "tops_gla_recurrent_fwd_workspace_size": (C.c_size_t, [C.POINTER(RecArgs)]),
    "tops_gla_recurrent_bwd": (C.c_int, [C.POINTER(RecBwdArgs), VP]),
    "tops_gla_recurrent_bwd_workspace_size": (C.c_size_t, [C.POINTER(RecBwdArgs)]),
    "tops_gla_chunk_local_cumsum": (C.c_int, [C.POINTER(Shape), VP, VP, I32, F32C, VP]),
    "tops_gla_chunk_fwd_h": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP, VP, VP, VP]),
    "tops_gla_chunk_bwd_dh": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP, VP, VP, VP]),
    "tops_gla_chunk_fwd_intra": (C.c_int, [C.POINTER(Shape), VP, VP, VP, I32, VP, VP]),
    "tops_gla_chunk_fwd_o": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP, VP, VP, VP]),
    "tops_gla_chunk_bwd_dA": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP]),
    "tops_gla_chunk_bwd_dv": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP, VP, VP, VP]),
    "tops_gla_chunk_bwd_dqk_intra": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP, VP, VP, VP]),
    "tops_gla_chunk_bwd_dqkg": (C.c_int, [C.POINTER(Shape), VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, VP, I32, VP,
                                          VP]),
    "tops_gla_chunk_span_saved_size": (C.c_size_t, [C.POINTER(Shape)]),
    "tops_gla_chunk_fwd_span_begin": (C.c_int, [C.POINTER(ChunkFwdArgs), VP, VP, VP]),
    "tops_gla_chunk_fwd_span_finish": (C.c_int, [C.POINTER(ChunkFwdArgs), VP]),
    "tops_gla_chunk_bwd_span_workspace_size": (C.c_size_t, [C.POINTER(ChunkBwdArgs)]),
    "tops_gla_chunk_bwd_span_begin": (C.c_int, [C.POINTER(ChunkBwdArgs), VP, VP]),
    "tops_gla_chunk_bwd_span_finish": (C.c_int, [C.POINTER(ChunkBwdArgs), VP]),
    "tops_gla_span_decay": (C.c_int, [C.POINTER(Shape), VP, VP, VP]),
    "tops_gla_state_combine": (C.c_int, [I32, I32, I32, I32, VP, VP, VP, VP, VP]),
    "tops_gla_norm_gate_fwd": (C.c_int, [C.c_int64, I32, I32, F32C, VP, VP, VP, VP, VP, VP]),
    "tops_gla_norm_gate_bwd_workspace_size": (C.c_size_t, [C.c_int64, I32]),
    "tops_gla_norm_gate_bwd": (C.c_int, [C.c_int64, I32, I32, VP, VP, VP, VP, VP, VP, VP, VP, VP, C.c_size_t,
                                         VP]),
    "tops_gla_gate_logsigmoid_fwd": (C.c_int, [C.c_int64, I32, F32C, F32C, I32, VP, VP, VP]),
    "tops_gla_gate_logsigmoid_bwd": (C.c_int, [C.c_int64, I32, F32C, F32C, I32, VP, VP, VP, VP]),
    "tops_gla_state_exchange_workspace_size": (C.c_size_t, [C.POINTER(ExchangeArgs)]),
    "tops_gla_state_exchange": (C.c_int, [C.POINTER(ExchangeArgs), VP]),
    "tops_gla_nccl_get_unique_id": (C.c_int, [VP]),
    "tops_gla_nccl_comm_init": (C.c_int, [C.POINTER(C.c_void_p), I32, VP, I32]),
    "tops_gla_nccl_comm_destroy": (C.c_int, [VP]),
    "tops_gla_nccl_comm_abort": (C.c_int, [VP]),
    "tops_gla_nccl_comm_check": (C.c_int, [VP]),
    "tops_gla_state_exchange_wait": (C.c_int, [VP, VP, I32]),
    "tops_gla_p2p_region_size": (C.c_size_t, [C.POINTER(P2PArgs)]),
    "tops_gla_p2p_alloc": (C.c_int, [C.c_size_t, C.POINTER(VP)]),
    "tops_gla_p2p_free": (C.c_int, [VP]),
    "tops_gla_ipc_handle": (C.c_int, [VP, VP]),
    "tops_gla_ipc_open": (C.c_int, [VP, C.POINTER(VP)]),
    "tops_gla_ipc_close": (C.c_int, [VP]),
    "tops_gla_p2p_exchange": (C.c_int, [C.POINTER(P2PArgs), VP]),
    "tops_gla_p2p_combine": (C.c_int, [C.POINTER(P2PArgs), VP]),
    "tops_gla_chunk_fwd_span_begin_p2p": (C.c_int, [C.POINTER(ChunkFwdArgs), VP, C.POINTER(P2PArgs), VP]),
    "tops_gla_chunk_bwd_span_begin_p2p": (C.c_int, [C.POINTER(ChunkBwdArgs), VP, C.POINTER(P2PArgs), VP]),
    "tops_gla_xla_chunk_fwd": (None, [VP, VP, C.c_char_p, C.c_size_t, VP]),
    "tops_gla_xla_chunk_bwd": (None, [VP, VP, C.c_char_p, C.c_size_t, VP]),
    "tops_gla_xla_recurrent_fwd": (None, [VP, VP, C.c_char_p, C.c_size_t, VP]),
}

_lib = None
_lock = threading.Lock()


def lib() -> C.CDLL:
    """Load libtops_gla.so once (raises ImportError when it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise ImportError(f"{LIB_PATH} is missing: build it with `python pallas-kernel_b200/build.py` "
                                      "(or __graft_entry__.build()); the GLA ops have no other implementation")
                l = C.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(l, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = l
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise TopsError(name, rc, lib().tops_gla_last_error().decode())


def ptr(t) -> int | None:
    """Device pointer of a tensor (None for None)."""
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected float32, bfloat16 or float16") from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def launch_count() -> int:
    return int(lib().tops_gla_launch_count())


def timing_enable(on: bool) -> None:
    lib().tops_gla_timing_enable(1 if on else 0)


def timing_collect(max_entries: int = 4096) -> list[tuple[str, float]]:
    """(kernel name, milliseconds) of every launch since timing was enabled (clears the record)."""
    stride = 64
    names = C.create_string_buffer(stride * max_entries)
    ms = (C.c_float * max_entries)()
    n = lib().tops_gla_timing_collect(names, stride, ms, max_entries)
    out = []
    for i in range(min(n, max_entries)):
        raw = names.raw[i * stride:(i + 1) * stride]
        out.append((raw.split(b"\0", 1)[0].decode(), float(ms[i])))
    return out


def has_tcgen05() -> bool:
    return bool(lib().tops_gla_has_tcgen05())
