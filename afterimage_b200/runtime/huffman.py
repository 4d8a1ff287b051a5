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
