"""ctypes binding of libafterimage_b200.so (the C ABI in
include/afterimage_b200.h).

The library is built in-tree (afterimage_b200/lib/) by
afterimage_b200.csrc.build; if it is missing, it is built on first use with
nvcc. There is no fallback: if the library cannot be loaded every decode
entry point raises.
"""
from __future__ import annotations

import ctypes
import pathlib
import threading

from .csrc import build as _build

_lock = threading.Lock()
_lib = None

AIB_OK = 0
AIB_EINVAL = 1
AIB_ECUDA = 2
AIB_EIO = 3
AIB_ESHORT = 4
AIB_MAX_BATCH = 16
AIB_GEMV_SCRATCH_FLOATS = 1 << 20

STATUS_BAD_CHUNK_RANGE = 1
STATUS_LUT_NOT_PREFIX = 2
STATUS_LUT_RANGE = 4
STATUS_WAIT_TIMEOUT = 8
STATUS_PEER_TIMEOUT = 16
WAIT_LIMIT_POLLS = 1 << 22  # AIB_WAIT_LIMIT_POLLS

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int32
CI = ctypes.c_int


class StreamDesc(ctypes.Structure):
    """aib_stream_desc (include/afterimage_b200.h)."""
    _fields_ = [
        ("packed", P),
        ("packed_capacity", I64),
        ("packed_nbytes", I64),
        ("offset_base", I64),
        ("chunk_offsets", P),
        ("chunk_nbytes", P),
        ("chunk_base", I64),
        ("tables", P),
        ("sym_lut", P),
        ("len_lut", P),
        ("max_bits", I32),
        ("chunk_size", I32),
        ("n_symbols", I64),
        ("elem_begin", I64),
        ("elem_end", I64),
        ("sign_mantissa", P),
        ("out", P),
        ("stripe_base", P),
    ]


class GemvDesc(ctypes.Structure):
    """aib_gemv_desc (include/afterimage_b200.h)."""
    _fields_ = [
        ("stream", StreamDesc),
        ("cols", I64),
        ("x", P),
        ("partial", P),
        ("y", P),
    ]


AR_MAX_RANKS = 8      # AIB_AR_MAX_RANKS
AR_MAX_CTAS = 64      # AIB_AR_MAX_CTAS
AR_HANDLE_BYTES = 64  # AIB_AR_HANDLE_BYTES


class ArGroup(ctypes.Structure):
    """aib_ar_group (include/afterimage_b200.h)."""
    _fields_ = [
        ("buffers", P * AR_MAX_RANKS),
        ("rank", I32),
        ("world", I32),
        ("max_floats", I64),
    ]


# (name, restype, argtypes) of every exported entry point; tests check that
# the header declares exactly these.
SIGNATURES = [
    ("aib_last_error", ctypes.c_char_p, []),
    ("aib_abi_version", CI, []),
    ("aib_split_bf16", CI, [P, I64, P, P]),
    ("aib_histogram", CI, [P, I64, P]),
    ("aib_build_code", CI, [P, CI, P, P, P]),
    ("aib_build_decode_lut", CI, [P, P, CI, P, P]),
    ("aib_chunk_nbytes", CI, [P, I64, I64, P, P, P]),
    ("aib_pack_chunks", CI, [P, I64, I64, P, P, P, P, P, I64]),
    ("aib_host_threads", CI, []),
    ("aib_pread_batch", CI, [CI, P, P, P, P, I64, CI, P]),
    ("aib_tables_bytes", ctypes.c_size_t, []),
    ("aib_build_tables", CI, [P, P, CI, P, P]),
    ("aib_tables_flags", CI, [P, P, P]),
    ("aib_decode_bf16", CI, [ctypes.POINTER(StreamDesc), P, P]),
    ("aib_decode_exponents_u8", CI, [ctypes.POINTER(StreamDesc), P, P]),
    ("aib_decode_exponents_i32", CI, [ctypes.POINTER(StreamDesc), P, P]),
    ("aib_decode_bf16_batch", CI, [ctypes.POINTER(StreamDesc), CI, P, P]),
    ("aib_decode_bf16_batch_ctas", CI, [ctypes.POINTER(StreamDesc), CI, CI, P, P]),
    ("aib_decode_gemv_bf16_batch", CI, [ctypes.POINTER(GemvDesc), CI, P, P]),
    ("aib_decode_gemv_bf16_batch_noalloc", CI, [ctypes.POINTER(GemvDesc), CI, P, P]),
    ("aib_recombine", CI, [P, P, I64, P, P]),
    ("aib_stripe_layout", CI, [P, I64, P, P]),
    ("aib_stripe_stream", CI, [P, I64, I64, P, P, I64, I64, P, P, I64, P, P]),
    ("aib_stripe_stream_host", CI, [P, I64, I64, P, P, I64, P, P, I64]),
    ("aib_ar_buffer_bytes", ctypes.c_size_t, [I64]),
    ("aib_ar_alloc", CI, [I64, P]),
    ("aib_ar_free", CI, [P]),
    ("aib_ar_ipc_handle", CI, [P, P]),
    ("aib_ar_ipc_open", CI, [P, P]),
    ("aib_ar_ipc_close", CI, [P]),
    ("aib_ar_ctas", CI, [I64]),
    ("aib_allreduce_oneshot_f32", CI, [P, P, P, I64, ctypes.c_uint, P, P]),
    ("aib_selftest_wait_timeout", CI, [ctypes.c_uint, P, P]),
    ("aib_add_rmsnorm_bf16", CI, [P, P, P, P, I64, I64, ctypes.c_float, P]),
    ("aib_qk_rope_cache_bf16", CI, [P, CI, CI, CI, CI, P, P, ctypes.c_float, P, P, P, P, P, I64, P]),
    ("aib_decode_attention_bf16", CI, [P, P, P, CI, CI, CI, I64, P, ctypes.c_float, P, P]),
    ("aib_silu_mul_bf16", CI, [P, P, I64, I64, P]),
    ("aib_gemv_bf16", CI, [P, I64, P, I64, P, I64, I64, I64, CI, CI, P]),
    ("aib_gemm_bf16_tc", CI, [P, I64, P, I64, P, I64, I64, I64, I64, P, I64, P, P]),
    ("aib_gemm_bf16_tc_workspace_floats", I64, [I64, I64, I64]),
]


class AibError(RuntimeError):
    pass


def lib_path() -> pathlib.Path:
    return _build.LIB


def load():
    """Load (building if needed) the library; raises if that fails."""
    global _lib
    with _lock:
        if _lib is None:
            path = _build.build()
            L = ctypes.CDLL(str(path))
            for name, res, args in SIGNATURES:
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            if L.aib_abi_version() != 2:
                raise AibError("libafterimage_b200.so ABI version mismatch")
            _lib = L
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc == AIB_OK:
        return
    msg = load().aib_last_error().decode(errors="replace")
    if rc in (AIB_EINVAL, AIB_ESHORT):
        raise ValueError(f"{what}: {msg}" if what else msg)
    if rc == AIB_EIO:
        raise OSError(f"{what}: {msg}" if what else msg)
    raise AibError(f"{what}: {msg}" if what else msg)
