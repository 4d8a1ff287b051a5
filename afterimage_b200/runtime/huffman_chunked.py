"""Chunked canonical-Huffman format for parallel decode (reference:
afterimage/runtime/huffman_chunked.py).

`ChunkedEncoded` is the reference's format type field for field
(huffman_chunked.py:135-148). `encode_chunked` produces byte-identical
output to the reference's encode_chunked (huffman_chunked.py:151-207) --
packed stream, chunk offsets and byte counts, LUTs and max_bits -- using the
library's C++ encoder (histogram, code construction, two-pass parallel
packing). Decoding lives on the GPU (gpu_decode_v2 / compressed_store); this
package has no CPU decoder.
"""
from __future__ import annotations

import ctypes
import dataclasses

import numpy as np
import torch

from .. import _lib
from .huffman import code_from_counts


@dataclasses.dataclass
class ChunkedEncoded:
    packed: np.ndarray          # uint8, all chunks concatenated, + 8 zero tail bytes
    chunk_offsets: np.ndarray   # int32, byte offset of each chunk's start
    chunk_nbytes: np.ndarray    # int32, byte length of each chunk
    sym_lut: np.ndarray         # int32[2^max_bits]
    len_lut: np.ndarray         # int8[2^max_bits]
    max_bits: int               # the table's ACTUAL width (longest code)
    chunk_size: int             # symbols per chunk
    n_symbols: int
    shape: tuple[int, ...]

    @property
    def n_chunks(self) -> int:
        return len(self.chunk_offsets)


def _symbols_u8(exponents) -> np.ndarray:
    if isinstance(exponents, torch.Tensor):
        flat = exponents.detach().flatten().cpu()
        if flat.dtype != torch.uint8:
            if flat.numel() and (int(flat.min()) < 0 or int(flat.max()) > 255):
                raise ValueError("exponent symbols must be in [0, 255]")
            flat = flat.to(torch.uint8)
        return flat.numpy()
    a = np.asarray(exponents).reshape(-1)
    if a.dtype != np.uint8:
        if a.size and (int(a.min()) < 0 or int(a.max()) > 255):
            raise ValueError("exponent symbols must be in [0, 255]")
        a = a.astype(np.uint8)
    return np.ascontiguousarray(a)


def encode_symbols(flat: np.ndarray, chunk_size: int, max_bits: int, shape: tuple) -> ChunkedEncoded:
    """Encodes a flat uint8 symbol array (the body of encode_chunked)."""
    if chunk_size < 1:
        raise ValueError("chunk_size must be >= 1")
    L = _lib.load()
    flat = np.ascontiguousarray(flat, dtype=np.uint8)
    n = int(flat.shape[0])
    counts = np.zeros(256, dtype=np.int64)
    _lib.check(L.aib_histogram(flat.ctypes.data, n, counts.ctypes.data), "histogram")
    lengths, codes, mb = code_from_counts(counts, max_bits)
    size = 1 << mb
    sym_lut = np.zeros(size, dtype=np.int32)
    len_lut = np.zeros(size, dtype=np.int8)
    _lib.check(L.aib_build_decode_lut(lengths.ctypes.data, codes.ctypes.data, mb,
                                      sym_lut.ctypes.data, len_lut.ctypes.data), "build_decode_lut")
    n_chunks = (n + chunk_size - 1) // chunk_size
    chunk_nbytes = np.zeros(n_chunks, dtype=np.int32)
    chunk_offsets = np.zeros(n_chunks, dtype=np.int32)
    total = ctypes.c_int64(0)
    _lib.check(L.aib_chunk_nbytes(flat.ctypes.data, n, int(chunk_size), lengths.ctypes.data,
                                  chunk_nbytes.ctypes.data, ctypes.addressof(total)), "chunk_nbytes")
    packed = np.empty(int(total.value) + 8, dtype=np.uint8)
    _lib.check(L.aib_pack_chunks(flat.ctypes.data, n, int(chunk_size), lengths.ctypes.data,
                                 codes.ctypes.data, chunk_nbytes.ctypes.data,
                                 chunk_offsets.ctypes.data, packed.ctypes.data,
                                 int(packed.shape[0])), "pack_chunks")
    return ChunkedEncoded(packed=packed, chunk_offsets=chunk_offsets, chunk_nbytes=chunk_nbytes,
                          sym_lut=sym_lut, len_lut=len_lut, max_bits=mb,
                          chunk_size=int(chunk_size), n_symbols=n, shape=tuple(shape))


def encode_chunked(exponents, chunk_size: int = 512, max_bits: int = 16) -> ChunkedEncoded:
    """Reference signature (huffman_chunked.py:151). Accepts a torch tensor
    or numpy array of exponent symbols (any integer dtype, values 0..255)."""
    shape = tuple(exponents.shape)
    return encode_symbols(_symbols_u8(exponents), int(chunk_size), int(max_bits), shape)
