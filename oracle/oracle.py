"""CPU ORACLE -- test infrastructure only, never part of the product path.

Python face of the C restatement in oracle.c (see its header for the
function-by-function map onto the reference), plus a pure-Python restatement
of the reference's bit reader for small cases. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module.

Pinned against the reference: tests/test_oracle_golden.py compares both the
C and the pure-Python decoders with golden vectors that the reference's own
code produced (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess
import threading

import numpy as np

_HERE = pathlib.Path(__file__).resolve().parent
_BUILD = _HERE / "_build"
_SO = _BUILD / "liboracle.so"
_lock = threading.Lock()
_lib = None


def build(force: bool = False) -> pathlib.Path:
    """Compile oracle.c into oracle/_build/liboracle.so (gcc, OpenMP)."""
    src = _HERE / "oracle.c"
    if _SO.exists() and not force and _SO.stat().st_mtime >= src.stat().st_mtime:
        return _SO
    _BUILD.mkdir(exist_ok=True)
    tmp = _SO.with_suffix(".so.tmp%d" % os.getpid())
    subprocess.run(["gcc", "-O2", "-fopenmp", "-shared", "-fPIC", "-std=c11",
                    str(src), "-o", str(tmp)], check=True)
    os.replace(tmp, _SO)
    return _SO


def lib():
    global _lib
    with _lock:
        if _lib is None:
            path = build()
            L = ctypes.CDLL(str(path))
            P = ctypes.c_void_p
            I64 = ctypes.c_int64
            CI = ctypes.c_int
            L.orc_decode_chunk.argtypes = [P, I64, P, P, CI, I64, P]
            L.orc_decode_chunk.restype = None
            L.orc_decode_chunks.argtypes = [P, P, P, P, P, CI, I64, I64, I64, CI, P]
            L.orc_decode_chunks.restype = None
            L.orc_recombine.argtypes = [P, P, I64, P]
            L.orc_recombine.restype = None
            L.orc_decompress_range.argtypes = [P, P, P, P, P, CI, I64, I64, P, I64, I64, CI, P]
            L.orc_decompress_range.restype = None
            L.orc_max_threads.argtypes = []
            L.orc_max_threads.restype = CI
            _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _arrays(enc):
    packed = np.ascontiguousarray(enc.packed, dtype=np.uint8)
    offs = np.ascontiguousarray(enc.chunk_offsets, dtype=np.int32)
    nb = np.ascontiguousarray(enc.chunk_nbytes, dtype=np.int32)
    sym = np.ascontiguousarray(enc.sym_lut, dtype=np.int32)
    ln = np.ascontiguousarray(enc.len_lut, dtype=np.int8)
    return packed, offs, nb, sym, ln


def max_threads() -> int:
    return int(lib().orc_max_threads())


def decode_chunks(enc, chunk_lo: int = 0, chunk_hi: int | None = None,
                  n_threads: int = 0) -> np.ndarray:
    """Restates decode_chunks_numba (cpu_decode.py:97-113): full chunk_size
    symbols per chunk, flat uint8; callers truncate to n_symbols."""
    chunk_hi = int(enc.n_chunks if chunk_hi is None else chunk_hi)
    n = max(0, chunk_hi - chunk_lo)
    out = np.zeros(n * int(enc.chunk_size), dtype=np.uint8)
    if n == 0:
        return out
    packed, offs, nb, sym, ln = _arrays(enc)
    lib().orc_decode_chunks(_ptr(packed), _ptr(offs), _ptr(nb), _ptr(sym), _ptr(ln),
                            int(enc.max_bits), int(enc.chunk_size), int(chunk_lo),
                            int(chunk_hi), int(n_threads), _ptr(out))
    return out


def decode_chunked(enc, n_threads: int = 0) -> np.ndarray:
    """Restates decode_chunked_cpu_reference (huffman_chunked.py:256-267)."""
    return decode_chunks(enc, 0, None, n_threads)[: int(enc.n_symbols)]


def recombine(exponent: np.ndarray, sign_mantissa: np.ndarray) -> np.ndarray:
    """Restates _recombine (compressed_store.py:94-114); returns uint16 bits."""
    e = np.ascontiguousarray(exponent, dtype=np.uint8)
    sm = np.ascontiguousarray(sign_mantissa, dtype=np.uint8)
    out = np.empty(e.shape[0], dtype=np.uint16)
    lib().orc_recombine(_ptr(e), _ptr(sm), int(e.shape[0]), _ptr(out))
    return out


def decompress_range(enc, sign_mantissa: np.ndarray, e0: int, e1: int,
                     n_threads: int = 0) -> np.ndarray:
    """Elements [e0, e1) as uint16 bf16 bit patterns (decompress_layer_gpu on
    device="cpu" / decompress_rows_gpu, compressed_store.py:186-303)."""
    n = int(enc.n_symbols)
    e1 = min(int(e1), n)
    e0 = max(0, int(e0))
    out = np.zeros(max(0, e1 - e0), dtype=np.uint16)
    if e1 <= e0:
        return out
    packed, offs, nb, sym, ln = _arrays(enc)
    sm = np.ascontiguousarray(sign_mantissa, dtype=np.uint8)
    lib().orc_decompress_range(_ptr(packed), _ptr(offs), _ptr(nb), _ptr(sym), _ptr(ln),
                               int(enc.max_bits), int(enc.chunk_size), n, _ptr(sm),
                               e0, e1, int(n_threads), _ptr(out))
    return out


def decompress(enc, sign_mantissa: np.ndarray, n_threads: int = 0) -> np.ndarray:
    return decompress_range(enc, sign_mantissa, 0, int(enc.n_symbols), n_threads)


# --- pure-Python restatement (small cases only) --------------------------------

def py_decode_chunk(chunk_bytes, sym_lut, len_lut, max_bits: int, n_out: int) -> list:
    """ChunkedBitReader (huffman_chunked.py:210-253), written out in Python."""
    buf = 0
    nbits = 0
    pos = 0
    out = []
    nbytes = len(chunk_bytes)
    for _ in range(n_out):
        while nbits < max_bits and pos < nbytes:
            buf |= int(chunk_bytes[pos]) << (24 - nbits)
            pos += 1
            nbits += 8
        window = (buf >> (32 - max_bits)) & ((1 << max_bits) - 1) if max_bits else 0
        out.append(int(sym_lut[window]))
        consumed = int(len_lut[window])
        buf = (buf << consumed) & 0xFFFFFFFF
        nbits -= consumed
    return out


def py_decode_chunked(enc) -> np.ndarray:
    out = []
    cs = int(enc.chunk_size)
    for c in range(int(enc.n_chunks)):
        s = int(enc.chunk_offsets[c])
        e = s + int(enc.chunk_nbytes[c])
        out.extend(py_decode_chunk(enc.packed[s:e], enc.sym_lut, enc.len_lut,
                                   int(enc.max_bits), cs))
    return np.asarray(out[: int(enc.n_symbols)], dtype=np.int64)


def py_recombine(exponent, sign_mantissa) -> np.ndarray:
    e = np.asarray(exponent, dtype=np.uint16)
    sm = np.asarray(sign_mantissa, dtype=np.uint16)
    return ((e << 7) | (sm & 0x7F) | ((sm & 0x80) << 8)).astype(np.uint16)
