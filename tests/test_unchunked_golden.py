"""The unchunked encoder helpers (huffman.pack_bits, encode_exponents)
against the reference's own outputs (tests/golden/unchunked_cases.npz,
written by make_unchunked_golden.py from the reference's huffman.py): the
same packed bytes, canonical table, codes and LUTs."""
import json
import pathlib

import numpy as np
import pytest
import torch

from afterimage_b200.runtime.huffman import encode_exponents, pack_bits

DATA = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "unchunked_cases.npz")
META = json.loads(bytes(DATA["meta"]).decode())


@pytest.mark.parametrize("name", sorted(META))
def test_encode_exponents_matches_reference(name):
    m = META[name]
    x = torch.from_numpy(DATA[name + "/symbols"].copy())
    e = encode_exponents(x, max_bits=m["max_bits_arg"])
    assert e.packed == DATA[name + "/packed"].tobytes()
    assert e.table.symbols == m["table_symbols"] and e.table.lengths == m["table_lengths"]
    assert e.table.max_bits == m["table_max_bits"]
    assert e.codes == {int(k): v for k, v in m["codes"].items()}
    assert np.array_equal(e.sym_lut, DATA[name + "/sym_lut"]) and np.array_equal(e.len_lut, DATA[name + "/len_lut"])
    assert e.n_symbols == m["n_symbols"] and list(e.shape) == m["shape"]


@pytest.mark.parametrize("name", sorted(META))
def test_pack_bits_matches_reference(name):
    m = META[name]
    codes = {int(k): v for k, v in m["codes"].items()}
    lengths = dict(zip(m["table_symbols"], m["table_lengths"]))
    assert pack_bits(DATA[name + "/symbols"], codes, lengths) == DATA[name + "/packed"].tobytes()


def test_pack_bits_rejects_symbols_without_a_code():
    with pytest.raises(ValueError):
        pack_bits(np.array([1, 2, 9], dtype=np.uint8), {1: 0, 2: 1}, {1: 1, 2: 1})
