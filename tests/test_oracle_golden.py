"""Pins the CPU oracle (oracle/) to the reference: every decoder in the
oracle must reproduce the golden vectors that the reference's own code
produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest

import golden_cases as G
from oracle import oracle as O

EXP = [c["name"] for c in G.cases("exponents")]
BF16 = [c["name"] for c in G.cases("bf16")]


@pytest.mark.parametrize("name", EXP)
def test_c_oracle_matches_reference_decoder(name):
    e = G.enc(name)
    got = O.decode_chunked(e)
    assert np.array_equal(got, G.arr(name, "decoded"))
    assert np.array_equal(got, G.arr(name, "symbols"))


@pytest.mark.parametrize("name", [n for n in EXP if G.has(n, "numba_full")])
def test_c_oracle_padding_symbols_match_numba(name):
    """Full chunk_size output per chunk, including the padding symbols the
    last chunk decodes past n_symbols (cpu_decode.py:67-113 semantics)."""
    e = G.enc(name)
    assert np.array_equal(O.decode_chunks(e), G.arr(name, "numba_full"))


@pytest.mark.parametrize("threads", [1, 2, 5])
def test_c_oracle_thread_count_invariant(threads):
    e = G.enc("real_bf16_128x4096")
    assert np.array_equal(O.decode_chunked(e, n_threads=threads), G.arr("real_bf16_128x4096", "decoded"))


@pytest.mark.parametrize("name", [n for n in EXP if G.case(n)["n_symbols"] <= 20000])
def test_python_restatement_matches_reference(name):
    e = G.enc(name)
    assert np.array_equal(O.py_decode_chunked(e), G.arr(name, "decoded").astype(np.int64))


@pytest.mark.parametrize("name", BF16)
def test_oracle_decompress_matches_reference_recon(name):
    e = G.enc(name)
    sm = G.arr(name, "sign_mantissa")
    got = O.decompress(e, sm)
    assert np.array_equal(got.view(np.int16), G.arr(name, "recon_bits"))
    assert np.array_equal(got.view(np.int16), G.arr(name, "weight_bits"))
    exps = O.decode_chunked(e)
    assert np.array_equal(O.recombine(exps, sm), got)
    assert np.array_equal(O.py_recombine(exps, sm), got)


@pytest.mark.parametrize("name", [n for n in BF16 if G.has(n, "rows_bits")])
def test_oracle_rows_match_reference_rows(name):
    c = G.case(name)
    e = G.enc(name)
    r0, r1 = c["rows"]
    cols = c["shape"][1]
    got = O.decompress_range(e, G.arr(name, "sign_mantissa"), r0 * cols, r1 * cols)
    assert np.array_equal(got.view(np.int16), G.arr(name, "rows_bits"))


def test_oracle_empty_range_and_empty_tensor():
    e = G.enc("empty")
    assert O.decode_chunked(e).shape == (0,)
    e = G.enc("store_128x512")
    assert O.decompress_range(e, G.arr("store_128x512", "sign_mantissa"), 10, 10).shape == (0,)
