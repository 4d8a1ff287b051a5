"""Canonical Huffman code construction for the exponent field -- the
encoder-side helpers of the reference's afterimage/runtime/huffman.py
(build_lengths :99-103, canonical_codes :106-125, build_decode_lut
:128-150), computed by the library's C++ encoder (aib_build_code,
aib_build_decode_lut) so the product encoder and these helpers agree byte
for byte with the reference.

Symbols are exponent bytes: every symbol must be in [0, 255].
"""
from __future__ import annotations

import ctypes
import dataclasses

import numpy as np

from .. import _lib


@dataclasses.dataclass
class HuffmanTable:
    """Same fields as the reference's HuffmanTable (huffman.py:30-38)."""
    symbols: list[int]
    lengths: list[int]
    max_bits: int

    @property
    def n_symbols(self) -> int:
        return len(self.symbols)


def _counts_from_freqs(freqs: dict[int, int]) -> np.ndarray:
    counts = np.zeros(256, dtype=np.int64)
    for s, f in freqs.items():
        if f > 0:
            if not 0 <= int(s) <= 255:
                raise ValueError(f"symbol {s} outside the exponent alphabet [0, 255]")
            counts[int(s)] = int(f)
    return counts


def code_from_counts(counts: np.ndarray, max_bits: int = 16) -> tuple[np.ndarray, np.ndarray, int]:
    """(lengths int32[256], codes uint32[256], max_bits) for a symbol histogram."""
    L = _lib.load()
    counts = np.ascontiguousarray(counts, dtype=np.int64)
    if counts.shape != (256,):
        raise ValueError("counts must have 256 entries")
    lengths = np.zeros(256, dtype=np.int32)
    codes = np.zeros(256, dtype=np.uint32)
    mb = ctypes.c_int32(0)
    _lib.check(L.aib_build_code(counts.ctypes.data, int(max_bits), lengths.ctypes.data,
                                codes.ctypes.data, ctypes.addressof(mb)), "build_code")
    return lengths, codes, int(mb.value)


def build_lengths(freqs: dict[int, int], max_bits: int = 16) -> dict[int, int]:
    """Code length per symbol: natural Huffman, length-limited by
    package-merge when deeper than max_bits (reference huffman.py:41-103)."""
    lengths, _, _ = code_from_counts(_counts_from_freqs(freqs), max_bits)
    return {int(s): int(lengths[s]) for s in range(256) if lengths[s] > 0}


def canonical_codes(lengths: dict[int, int]) -> tuple[HuffmanTable, dict[int, int]]:
    """Canonical code assignment by (length, symbol) (reference huffman.py:106-125)."""
    order = sorted(lengths.items(), key=lambda kv: (kv[1], kv[0]))
    symbols = [int(s) for s, _ in order]
    lens = [int(n) for _, n in order]
    code = 0
    prev = lens[0] if lens else 0
    codes: dict[int, int] = {}
    for s, n in zip(symbols, lens):
        code <<= (n - prev)
        codes[s] = code
        code += 1
        prev = n
    return HuffmanTable(symbols=symbols, lengths=lens, max_bits=max(lens) if lens else 0), codes


def build_decode_lut(table: HuffmanTable, codes: dict[int, int]) -> tuple[np.ndarray, np.ndarray]:
    """Flat 2^max_bits LUT (reference huffman.py:128-150)."""
    L = _lib.load()
    lengths = np.zeros(256, dtype=np.int32)
    cd = np.zeros(256, dtype=np.uint32)
    for s, n in zip(table.symbols, table.lengths):
        lengths[s] = n
        cd[s] = codes[s]
    size = 1 << table.max_bits
    sym_lut = np.zeros(size, dtype=np.int32)
    len_lut = np.zeros(size, dtype=np.int8)
    _lib.check(L.aib_build_decode_lut(lengths.ctypes.data, cd.ctypes.data, int(table.max_bits),
                                      sym_lut.ctypes.data, len_lut.ctypes.data), "build_decode_lut")
    return sym_lut, len_lut


def pack_bits(symbol_stream: np.ndarray, codes: dict[int, int], lengths: dict[int, int]) -> bytes:
    """MSB-first concatenation of every symbol's code, zero-padded to a whole
    byte (reference huffman.py:153-192), packed by the library's C++ packer
    with the whole stream as one chunk. Every symbol must have a code (a
    symbol without one raises ValueError); at most 2^30 symbols per call."""
    flat = np.asarray(symbol_stream).reshape(-1)
    n = int(flat.shape[0])
    if n == 0:
        return b""
    if int(flat.min()) < 0 or int(flat.max()) > 255:
        raise ValueError("symbols must be in [0, 255]")
    if n > 1 << 30:
        raise ValueError("pack_bits packs at most 2^30 symbols per call")
    flat = np.ascontiguousarray(flat, dtype=np.uint8)
    ln = np.zeros(256, dtype=np.int32)
    cd = np.zeros(256, dtype=np.uint32)
    for s, c in codes.items():
        if 0 <= int(s) <= 255:
            ln[int(s)] = int(lengths[s])
            cd[int(s)] = int(c)
    L = _lib.load()
    nbytes = np.zeros(1, dtype=np.int32)
    offsets = np.zeros(1, dtype=np.int32)
    total = ctypes.c_int64(0)
    rc = L.aib_chunk_nbytes(flat.ctypes.data, n, n, ln.ctypes.data, nbytes.ctypes.data, ctypes.addressof(total))
    if rc != _lib.AIB_OK:
        raise ValueError("pack_bits: " + L.aib_last_error().decode())
    out = np.empty(int(total.value) + 8, dtype=np.uint8)
    _lib.check(L.aib_pack_chunks(flat.ctypes.data, n, n, ln.ctypes.data, cd.ctypes.data, nbytes.ctypes.data,
                                 offsets.ctypes.data, out.ctypes.data, int(out.shape[0])), "pack_bits")
    return out[:int(total.value)].tobytes()


@dataclasses.dataclass
class EncodedTensor:
    """The unchunked encoding (reference huffman.py:243-250)."""
    packed: bytes
    table: HuffmanTable
    codes: dict[int, int]
    sym_lut: np.ndarray
    len_lut: np.ndarray
    n_symbols: int
    shape: tuple[int, ...]


def encode_exponents(exponents, max_bits: int = 16) -> EncodedTensor:
    """Code from the tensor's own symbol histogram, one packed stream and
    its decode LUT (reference huffman.py:253-272). The chunked format
    (huffman_chunked.encode_chunked) is what the decoders read."""
    import torch
    flat = (exponents.detach().flatten().cpu().numpy() if isinstance(exponents, torch.Tensor)
            else np.asarray(exponents).reshape(-1)).astype(np.int64)
    counts = np.bincount(flat) if flat.size else np.zeros(0, dtype=np.int64)
    freqs = {int(s): int(c) for s, c in enumerate(counts) if c > 0}
    lengths = build_lengths(freqs, max_bits=max_bits)
    table, codes = canonical_codes(lengths)
    sym_lut, len_lut = build_decode_lut(table, codes)
    return EncodedTensor(packed=pack_bits(flat, codes, lengths), table=table, codes=codes, sym_lut=sym_lut,
                         len_lut=len_lut, n_symbols=int(flat.shape[0]), shape=tuple(exponents.shape))
