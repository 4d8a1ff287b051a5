"""Generates tests/golden/binstore_extents.json by running the REFERENCE's
BinaryWeightReader.read_many (afterimage/runtime/binstore.py) on seeded
blob layouts: adjacent, gapped and overlapping blobs in shuffled request
order, under several max_gap_bytes / max_extent_bytes bounds. Recorded per
case: the requests, the bounds, the reference's read-call and byte counts
and a crc32 of each returned array.

Usage: python tests/golden/make_binstore_golden.py <path to an Afterimage checkout>
       (or set AFTERIMAGE_REF)

The file read is a deterministic byte pattern (byte i = (i * 131 + 7) mod
251), so a test can rebuild it without the fixture carrying it.
"""
from __future__ import annotations

import importlib.util
import json
import os
import pathlib
import random
import sys
import tempfile
import zlib

sys.dont_write_bytecode = True

import numpy as np  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "binstore_extents.json"
FILE_BYTES = 1 << 16


def pattern(n: int) -> bytes:
    return bytes(((np.arange(n, dtype=np.int64) * 131 + 7) % 251).astype(np.uint8))


def load_reference(root: pathlib.Path):
    path = root / "afterimage" / "runtime" / "binstore.py"
    spec = importlib.util.spec_from_file_location("afterimage_ref_binstore", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # its dataclasses look their module up by name
    spec.loader.exec_module(mod)
    return mod


def layout(rng: random.Random, kind: str) -> list[dict]:
    refs, pos = [], rng.randrange(0, 64)
    for _ in range(rng.randrange(1, 12)):
        dtype = rng.choice(["uint8", "int16", "int32"])
        item = np.dtype(dtype).itemsize
        count = rng.randrange(0, 300)
        nbytes = count * item
        if kind == "gapped":
            pos += rng.randrange(0, 200)
        elif kind == "overlapping" and refs and rng.random() < 0.4:
            pos = max(0, pos - rng.randrange(1, 100))
        if pos + nbytes > FILE_BYTES:
            break
        refs.append({"offset": pos, "nbytes": nbytes, "dtype": dtype, "shape": [count]})
        pos += nbytes
    rng.shuffle(refs)
    return refs


def main() -> None:
    root = pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["AFTERIMAGE_REF"])
    ref = load_reference(root)
    rng = random.Random(20)
    cases = []
    with tempfile.TemporaryDirectory() as tmp:
        path = pathlib.Path(tmp) / "weights.bin"
        path.write_bytes(pattern(FILE_BYTES))
        reader = ref.BinaryWeightReader(path)
        try:
            for kind in ("adjacent", "gapped", "overlapping"):
                for _ in range(12):
                    refs = layout(rng, kind)
                    for gap, extent in ((0, 1 << 28), (64, 1 << 28), (256, 512), (1 << 20, 1)):
                        arrays, calls, nbytes = reader.read_many(refs, max_gap_bytes=gap, max_extent_bytes=extent)
                        cases.append({"kind": kind, "refs": refs, "max_gap_bytes": gap, "max_extent_bytes": extent,
                                      "calls": calls, "bytes": nbytes,
                                      "crc32": [zlib.crc32(np.ascontiguousarray(a).tobytes()) for a in arrays]})
        finally:
            reader.close()
    OUT.write_text(json.dumps({"file_bytes": FILE_BYTES, "cases": cases}))
    print("wrote %s: %d cases" % (OUT, len(cases)))


if __name__ == "__main__":
    main()
