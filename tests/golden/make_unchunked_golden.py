"""Generates tests/golden/unchunked_cases.npz by running the REFERENCE's
unchunked encoder (afterimage/runtime/huffman.py encode_exponents, which
builds the code and calls pack_bits and build_decode_lut) on seeded symbol
streams: one repeated symbol, a single symbol, a skewed alphabet, all 256
symbols, real BF16 exponents, a Fibonacci-weighted stream whose code is
length-limited to 12 bits, and an empty stream.

Usage: python tests/golden/make_unchunked_golden.py <path to an Afterimage checkout>
       (or set AFTERIMAGE_REF)

Stored per case: the input symbols, max_bits, the packed bytes, the
canonical table (symbols, lengths, max_bits), the codes and both LUTs.
"""
from __future__ import annotations

import importlib.util
import json
import os
import pathlib
import sys

sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "unchunked_cases.npz"


def load_reference(root: pathlib.Path):
    spec = importlib.util.spec_from_file_location("afterimage_ref_huffman", root / "afterimage" / "runtime" / "huffman.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # its dataclasses look their module up by name
    spec.loader.exec_module(mod)
    return mod


def inputs() -> dict:
    g = torch.Generator().manual_seed(0)
    fib, a, b = [], 1, 1
    for s in range(24):
        fib += [s] * a
        a, b = b, a + b
    return {
        "repeated": (torch.full((1000,), 7, dtype=torch.uint8), 16),
        "single": (torch.tensor([3], dtype=torch.uint8), 16),
        "skewed": (torch.randint(0, 4, (5000,), generator=g).to(torch.uint8)
                   * torch.randint(0, 2, (5000,), generator=g).to(torch.uint8), 16),
        "uniform256": (torch.randint(0, 256, (20000,), generator=g).to(torch.uint8), 16),
        "bf16_exponents": ((((torch.randn(100000, generator=g) * 0.02).to(torch.bfloat16).view(torch.int16) >> 7)
                            & 0xFF).to(torch.uint8), 16),
        "fibonacci_limit12": (torch.tensor(fib, dtype=torch.uint8), 12),
        "empty": (torch.zeros(0, dtype=torch.uint8), 16),
    }


def main() -> None:
    root = pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["AFTERIMAGE_REF"])
    ref = load_reference(root)
    arrays, meta = {}, {}
    for name, (x, mb) in inputs().items():
        e = ref.encode_exponents(x, max_bits=mb)
        arrays[name + "/symbols"] = x.numpy()
        arrays[name + "/packed"] = np.frombuffer(e.packed, dtype=np.uint8)
        arrays[name + "/sym_lut"] = e.sym_lut
        arrays[name + "/len_lut"] = e.len_lut
        meta[name] = {"max_bits_arg": mb, "table_symbols": e.table.symbols, "table_lengths": e.table.lengths,
                      "table_max_bits": e.table.max_bits, "codes": {str(k): v for k, v in e.codes.items()},
                      "n_symbols": e.n_symbols, "shape": list(e.shape)}
    np.savez_compressed(OUT, meta=np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8), **arrays)
    print("wrote", OUT, sorted(meta))


if __name__ == "__main__":
    main()
