"""The product encoder (C++ behind afterimage_b200.runtime.huffman_chunked)
must be byte-identical to the reference encoder: packed stream, offsets,
byte counts, LUTs and max_bits, on every golden case the reference produced."""
import numpy as np
import pytest

import golden_cases as G
from afterimage_b200.runtime import huffman as H
from afterimage_b200.runtime.huffman_chunked import encode_chunked

EXP = [c["name"] for c in G.cases("exponents")]


def _same(enc, name):
    c = G.case(name)
    assert enc.max_bits == c["max_bits"]
    assert enc.chunk_size == c["chunk_size"]
    assert enc.n_symbols == c["n_symbols"]
    assert enc.n_chunks == c["n_chunks"]
    assert np.array_equal(enc.packed, G.arr(name, "packed"))
    assert np.array_equal(enc.chunk_offsets, G.arr(name, "chunk_offsets"))
    assert np.array_equal(enc.chunk_nbytes, G.arr(name, "chunk_nbytes"))
    assert np.array_equal(enc.sym_lut, G.arr(name, "sym_lut"))
    assert np.array_equal(enc.len_lut, G.arr(name, "len_lut"))
    assert enc.packed.dtype == np.uint8 and enc.chunk_offsets.dtype == np.int32
    assert enc.sym_lut.dtype == np.int32 and enc.len_lut.dtype == np.int8


@pytest.mark.parametrize("name", EXP)
def test_encode_chunked_byte_identical_to_reference(name):
    c = G.case(name)
    enc = encode_chunked(G.arr(name, "symbols"), chunk_size=c["chunk_size_arg"],
                         max_bits=c["max_bits_arg"])
    _same(enc, name)


def test_package_merge_limit_respected_and_identical():
    # Fibonacci alphabet: natural depth > 16, limited by package-merge
    enc = encode_chunked(G.arr("fibonacci_limit6", "symbols"), chunk_size=512, max_bits=6)
    assert enc.max_bits <= 6
    _same(enc, "fibonacci_limit6")


def test_build_lengths_and_canonical_codes_match_lut():
    name = "dirichlet_3"
    syms = G.arr(name, "symbols")
    freqs = {int(s): int(c) for s, c in enumerate(np.bincount(syms, minlength=256)) if c > 0}
    lengths = H.build_lengths(freqs, max_bits=16)
    table, codes = H.canonical_codes(lengths)
    sym_lut, len_lut = H.build_decode_lut(table, codes)
    assert np.array_equal(sym_lut, G.arr(name, "sym_lut"))
    assert np.array_equal(len_lut, G.arr(name, "len_lut"))


def test_symbols_outside_byte_range_rejected():
    with pytest.raises(ValueError):
        encode_chunked(np.array([0, 256, 3]), chunk_size=4)
