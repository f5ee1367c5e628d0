"""ctypes binding of libtq_b200.so (the C ABI declared in include/tq_b200.h).

There is no CPU fallback: importing this module succeeds without a GPU, but
every call that launches work needs the built library and a CUDA device and
raises when either is missing.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libtq_b200.so")

TQ_OK = 0
TQ_ERR_INVALID = -1
TQ_ERR_CUDA = -2
TQ_ERR_WORKSPACE = -3
TQ_ERR_DEVICE = -4
TQ_F32, TQ_F16, TQ_BF16 = 0, 1, 2
DEV_WAIT_TIMEOUT, DEV_BAD_BLOCK = 1, 2
PAGE_TOKENS = 64
PHASE_QPREP, PHASE_DECODE, PHASE_MERGE = 1, 2, 4

# every symbol include/tq_b200.h declares
EXPORTED = (
    "tq_last_error", "tq_version", "tq_page_bytes", "tq_quantize_rotated",
    "tq_append", "tq_dequantize", "tq_decode_workspace_bytes", "tq_decode_attn",
    "tq_decode_step", "tq_decode_attn_noalloc", "tq_noalloc_status", "tq_workspace_status", "tq_device_status",
    "tq_append_tensor_core", "tq_prefill_attn", "tq_prefill_workspace_bytes",
    "tq_prefill_tensor_core",
    "tq_shared_alloc", "tq_shared_open", "tq_shared_close", "tq_shared_free",
    "tq_tables_bytes", "tq_init_tables",
)
MAX_PEERS = 8
SHARED_HANDLE_BYTES = 64


class TqError(RuntimeError):
    """A libtq_b200 call returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with status {status}: {message}")
        self.status = status


class Geom(ctypes.Structure):
    _fields_ = [("head_dim", ctypes.c_int32), ("key_bits", ctypes.c_int32),
                ("value_bits", ctypes.c_int32), ("qjl", ctypes.c_int32)]


class Tables(ctypes.Structure):
    _fields_ = [("k_centroids", ctypes.c_void_p), ("k_boundaries", ctypes.c_void_p),
                ("v_centroids", ctypes.c_void_p), ("v_boundaries", ctypes.c_void_p),
                ("rot", ctypes.c_void_p), ("qjl", ctypes.c_void_p),
                ("rot_t", ctypes.c_void_p), ("qjl_t", ctypes.c_void_p),
                ("rot_bf16x3", ctypes.c_void_p), ("rot_f16", ctypes.c_void_p),
                ("qjl_bf16", ctypes.c_void_p)]


class Cache(ctypes.Structure):
    _fields_ = [("pages", ctypes.c_void_p), ("streams", ctypes.c_int64),
                ("pages_per_stream", ctypes.c_int64), ("block_table", ctypes.c_void_p),
                ("block_table_stride", ctypes.c_int64), ("num_blocks", ctypes.c_int64)]


class Tensor4(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 4), ("stride", ctypes.c_int64 * 4)]


class Gather(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("peer_out", ctypes.c_void_p * MAX_PEERS),
                ("peer_flag", ctypes.c_void_p * MAX_PEERS)]


class DecodeArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.POINTER(Tensor4)), ("out", ctypes.POINTER(Tensor4)),
                ("window_k", ctypes.POINTER(Tensor4)), ("window_v", ctypes.POINTER(Tensor4)),
                ("n_tokens", ctypes.c_int64), ("num_q_heads", ctypes.c_int64),
                ("scale", ctypes.c_float), ("num_ctas", ctypes.c_int32),
                ("phases", ctypes.c_int32), ("gather", ctypes.POINTER(Gather)),
                ("seq_lens", ctypes.c_void_p), ("kv_start", ctypes.c_void_p)]


class PrefillArgs(ctypes.Structure):
    _fields_ = [("q", ctypes.POINTER(Tensor4)), ("out", ctypes.POINTER(Tensor4)),
                ("n_tokens", ctypes.c_int64), ("scale", ctypes.c_float),
                ("causal", ctypes.c_int32), ("engine", ctypes.c_int32),
                ("kv_start", ctypes.c_void_p),
                ("window_k", ctypes.POINTER(Tensor4)), ("window_v", ctypes.POINTER(Tensor4)),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t)]


_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and return the library; raises if it has not been built."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"libtq_b200.so not found at {path}; build it with "
                "`python -m bhaskera_col_b200.csrc.build` (there is no CPU fallback)")
        lib = ctypes.CDLL(path)
        P, I32, I64, SZ, VP = (ctypes.POINTER, ctypes.c_int32, ctypes.c_int64,
                               ctypes.c_size_t, ctypes.c_void_p)
        sig = {
            "tq_last_error": (ctypes.c_char_p, []),
            "tq_version": (I32, []),
            "tq_page_bytes": (I64, [P(Geom)]),
            "tq_quantize_rotated": (I32, [VP, I64, VP, I32, VP, VP]),
            "tq_append": (I32, [P(Geom), P(Tables), P(Cache), P(Tensor4), P(Tensor4), I64, VP]),
            "tq_dequantize": (I32, [P(Geom), P(Tables), P(Cache), I64, I64, P(Tensor4),
                                    P(Tensor4), VP]),
            "tq_decode_workspace_bytes": (SZ, [P(Geom), P(Cache), P(DecodeArgs)]),
            "tq_decode_attn": (I32, [P(Geom), P(Tables), P(Cache), P(DecodeArgs), VP, SZ, VP]),
            "tq_decode_step": (I32, [P(Geom), P(Tables), P(Cache), P(Tensor4), P(Tensor4), I64,
                                     P(DecodeArgs), VP, SZ, VP]),
            "tq_decode_attn_noalloc": (I32, [P(Geom), P(Tables), P(Cache), P(DecodeArgs), VP]),
            "tq_noalloc_status": (I32, [P(ctypes.c_uint32), VP]),
            "tq_workspace_status": (I32, [VP, P(ctypes.c_uint32), VP]),
            "tq_device_status": (I32, [P(ctypes.c_uint32), VP]),
            "tq_append_tensor_core": (I32, [P(Geom), P(Tables), P(Tensor4), P(Tensor4)]),
            "tq_prefill_attn": (I32, [P(Geom), P(Tables), P(Cache), P(PrefillArgs), VP]),
            "tq_prefill_workspace_bytes": (SZ, [P(Geom), P(Cache), P(PrefillArgs)]),
            "tq_prefill_tensor_core": (I32, [P(Geom)]),
            "tq_shared_alloc": (I32, [SZ, P(ctypes.c_void_p), VP]),
            "tq_shared_open": (I32, [VP, P(ctypes.c_void_p)]),
            "tq_shared_close": (I32, [VP]),
            "tq_shared_free": (I32, [VP]),
            "tq_tables_bytes": (SZ, [P(Geom)]),
            "tq_init_tables": (I32, [P(Geom), VP, VP, VP, VP, VP, VP, VP, SZ, P(Tables), VP]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def last_error() -> str:
    return load().tq_last_error().decode(errors="replace")


def check(fn: str, status: int) -> None:
    if status != TQ_OK:
        raise TqError(fn, status, last_error())
