"""read_many's extent coalescing against the reference's own results
(tests/golden/binstore_extents.json, written by make_binstore_golden.py with
the reference's BinaryWeightReader.read_many): the same number of read calls
and bytes read, and the same array contents in the caller's order, for
adjacent, gapped and overlapping blobs under several gap / extent bounds, in
every read mode of this package's reader."""
import json
import pathlib
import zlib

import numpy as np
import pytest

from afterimage_b200.runtime.binstore import BinaryWeightReader, PinnedBuffer

GOLDEN = json.loads((pathlib.Path(__file__).resolve().parent / "golden" / "binstore_extents.json").read_text())


@pytest.fixture(scope="module")
def weights(tmp_path_factory):
    n = GOLDEN["file_bytes"]
    path = tmp_path_factory.mktemp("extents") / "weights.bin"
    path.write_bytes(((np.arange(n, dtype=np.int64) * 131 + 7) % 251).astype(np.uint8).tobytes())
    return path


@pytest.mark.parametrize("mode", ["plain", "pinned", "pinned_parallel"])
def test_read_many_matches_reference_extents(weights, mode):
    threads = 4 if mode == "pinned_parallel" else 1
    buf = PinnedBuffer() if mode != "plain" else False
    with BinaryWeightReader(weights, threads=threads) as reader:
        for c in GOLDEN["cases"]:
            arrays, calls, nbytes = reader.read_many(c["refs"], max_gap_bytes=c["max_gap_bytes"],
                                                     max_extent_bytes=c["max_extent_bytes"], pinned=buf)
            assert (calls, nbytes) == (c["calls"], c["bytes"]), c["kind"]
            got = [zlib.crc32(np.ascontiguousarray(a).tobytes()) for a in arrays]
            assert got == c["crc32"], c["kind"]
            for a, r in zip(arrays, c["refs"]):
                assert a.dtype == np.dtype(r["dtype"]) and list(a.shape) == r["shape"]


def test_fixture_exercises_merging_and_bounds():
    kinds = {c["kind"] for c in GOLDEN["cases"]}
    assert kinds == {"adjacent", "gapped", "overlapping"}
    assert any(c["calls"] < len(c["refs"]) for c in GOLDEN["cases"])    # merged extents
    assert any(c["calls"] == len(c["refs"]) > 1 for c in GOLDEN["cases"])  # nothing merged
