"""Compressed-store I/O: the reference's binstore tests (afterimage
tests/test_binstore.py) restated, plus the pinned and O_DIRECT read paths."""
import json
import zlib

import numpy as np
import pytest
import torch

from afterimage_b200.runtime.binstore import (
    BinaryWeightReader, BinaryWeightWriter, PinnedBuffer, blobref_to_dict, verify_store,
)


def _store(path, arrays):
    with BinaryWeightWriter(path) as w:
        return [blobref_to_dict(w.write(a)) for a in arrays]


def test_write_then_read_roundtrip_exact(tmp_path):
    arrays = [np.random.randint(0, 256, size=1000, dtype=np.uint8), np.random.randn(50, 30).astype(np.float32),
              np.array([1, 2, 3], dtype=np.int32)]
    refs = _store(tmp_path / "w.bin", arrays)
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        for a, ref in zip(arrays, refs):
            got = r.read(ref)
            assert np.array_equal(got, a) and got.dtype == a.dtype and got.shape == a.shape
            assert ref["crc32"] == zlib.crc32(a.tobytes())


def test_offsets_are_sequential_and_non_overlapping(tmp_path):
    with BinaryWeightWriter(tmp_path / "w.bin") as w:
        r1, r2, r3 = (w.write(np.zeros(n, dtype=np.uint8)) for n in (100, 50, 200))
    assert (r1.offset, r2.offset, r3.offset) == (0, 100, 150)
    assert (tmp_path / "w.bin").stat().st_size == 350


@pytest.mark.parametrize("pinned", [False, True])
@pytest.mark.parametrize("direct", [False, True])
def test_read_many_coalesces_bit_exact_in_any_mode(tmp_path, pinned, direct):
    arrays = [np.arange(64, dtype=np.uint8), np.arange(20, dtype=np.float32).reshape(4, 5),
              np.arange(11, dtype=np.int32), np.random.randint(0, 255, 10000, dtype=np.uint8)]
    refs = _store(tmp_path / "w.bin", arrays)
    with BinaryWeightReader(tmp_path / "w.bin", direct=direct) as r:
        got, calls, nbytes = r.read_many(refs, max_extent_bytes=1 << 20, pinned=pinned)
    assert calls == 1 and nbytes == (tmp_path / "w.bin").stat().st_size
    assert all(np.array_equal(a, b) for a, b in zip(got, arrays))


@pytest.mark.parametrize("direct", [False, True])
@pytest.mark.parametrize("threads,piece", [(4, 4096), (3, 12288), (8, 1 << 20)])
def test_parallel_pinned_reads_are_bit_exact(tmp_path, direct, threads, piece):
    """Extents split into pieces read concurrently land exactly where a
    single sequential read puts them (ragged last piece, unaligned blob
    starts inside extents, several extents)."""
    rng = np.random.default_rng(threads + piece)
    arrays = [rng.integers(0, 256, n, dtype=np.uint8) for n in (5, 70001, 4096, 123457, 3, 65536 * 3 + 17)]
    refs = _store(tmp_path / "w.bin", arrays)
    with BinaryWeightReader(tmp_path / "w.bin", direct=direct, threads=threads, piece_bytes=piece) as r:
        for extent in (1 << 30, 100000):
            got, calls, nbytes = r.read_many(refs, max_extent_bytes=extent, pinned=True)
            assert all(np.array_equal(a, b) for a, b in zip(got, arrays))
            assert nbytes == sum(a.nbytes for a in arrays)


def test_parallel_short_read_raises(tmp_path):
    refs = _store(tmp_path / "w.bin", [np.zeros(50000, np.uint8)])
    bad = dict(refs[0], nbytes=90000, shape=[90000])
    with BinaryWeightReader(tmp_path / "w.bin", threads=4, piece_bytes=4096) as r:
        with pytest.raises(ValueError, match="short read"):
            r.read_many([bad], pinned=True)


def test_read_many_respects_extent_bound_and_original_order(tmp_path):
    arrays = [np.full(32, v, dtype=np.uint8) for v in range(3)]
    refs = _store(tmp_path / "w.bin", arrays)
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        got, calls, nbytes = r.read_many([refs[2], refs[0], refs[1]], max_extent_bytes=48)
    assert calls == 3 and nbytes == 96 and [int(a[0]) for a in got] == [2, 0, 1]


@pytest.mark.parametrize("pinned", [False, True])
def test_read_many_groups_merge_only_within_a_label(tmp_path, pinned):
    """Per-tensor extents in one call: adjacent blobs of different labels
    stay separate reads; the arrays are the same either way."""
    arrays = [np.full(40, v, dtype=np.uint8) for v in range(6)]
    refs = _store(tmp_path / "w.bin", arrays)
    order = [4, 0, 5, 2, 1, 3]
    labels = ["a", "a", "b", "b", "c", "c"]
    with BinaryWeightReader(tmp_path / "w.bin", threads=2) as r:
        merged, calls_all, _ = r.read_many([refs[i] for i in order], pinned=pinned)
        merged = [a.copy() for a in merged]
        grouped, calls_grp, nbytes = r.read_many([refs[i] for i in order], pinned=pinned,
                                                 groups=[labels[i] for i in order])
    assert calls_all == 1 and calls_grp == 3 and nbytes == 240
    assert all(np.array_equal(a, b) for a, b in zip(merged, grouped))
    assert [int(a[0]) for a in grouped] == order
    with BinaryWeightReader(tmp_path / "w.bin") as r, pytest.raises(ValueError, match="one label per ref"):
        r.read_many(refs, groups=["a"])


def test_read_many_unaligned_views_are_writable_and_torch_consumable(tmp_path):
    arrays = [np.arange(7, dtype=np.uint8), np.arange(5, dtype=np.uint32), np.arange(3, dtype=np.float32),
              np.arange(9, dtype=np.uint16).reshape(3, 3)]
    refs = _store(tmp_path / "w.bin", arrays)
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        got, calls, _ = r.read_many(refs, verify=True)
    assert calls == 1
    for a, g in zip(arrays, got):
        assert np.array_equal(a, g) and g.flags.writeable and not g.flags.owndata
        torch.from_numpy(g)


def test_pinned_buffer_is_reused_and_grows(tmp_path):
    arrays = [np.random.randint(0, 255, 5000, dtype=np.uint8) for _ in range(4)]
    refs = _store(tmp_path / "w.bin", arrays)
    buf = PinnedBuffer()
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        a, _, _ = r.read_many(refs[:1], pinned=buf)
        cap = buf.array.shape[0]
        assert np.array_equal(a[0], arrays[0])
        b, _, _ = r.read_many(refs, pinned=buf)
        assert all(np.array_equal(x, y) for x, y in zip(b, arrays))
        assert buf.array.shape[0] >= cap


def test_empty_array_and_read_many_empty(tmp_path):
    refs = _store(tmp_path / "w.bin", [np.array([], dtype=np.uint8)])
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        assert r.read(refs[0]).shape == (0,)
        assert r.read_many([]) == ([], 0, 0)
    with pytest.raises(ValueError):
        BinaryWeightReader(tmp_path / "w.bin").read_many(refs, max_gap_bytes=-1)


def test_read_row_and_rows_match_full_read(tmp_path):
    table = np.random.randint(-30000, 30000, size=(37, 24), dtype=np.int16)
    with BinaryWeightWriter(tmp_path / "w.bin") as w:
        ref = w.write(table)
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        full = r.read(blobref_to_dict(ref))
        for i in range(37):
            assert np.array_equal(r.read_row(ref.offset, i, 48, "int16"), full[i])
        idx = [5, 0, 36, 5]
        assert np.array_equal(r.read_rows(ref.offset, idx, 48, "int16"), full[idx])


def test_checksums_detect_corruption_only_when_asked(tmp_path):
    arr = np.random.randint(0, 256, size=500, dtype=np.uint8)
    refs = _store(tmp_path / "w.bin", [arr])
    with open(tmp_path / "w.bin", "r+b") as f:
        f.seek(250)
        f.write(bytes([arr[250] ^ 0xFF]))
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        with pytest.raises(ValueError, match="checksum mismatch"):
            r.read(refs[0], verify=True)
        with pytest.raises(ValueError, match="checksum mismatch"):
            r.read_many(refs, verify=True)
        assert not np.array_equal(r.read(refs[0]), arr)


def test_short_read_raises(tmp_path):
    refs = _store(tmp_path / "w.bin", [np.zeros(100, np.uint8)])
    bad = dict(refs[0], nbytes=200, shape=[200])
    with BinaryWeightReader(tmp_path / "w.bin") as r:
        with pytest.raises(ValueError, match="short read"):
            r.read_many([bad])


def test_verify_store_flags_corrupted_tensors_by_key(tmp_path):
    store = tmp_path / "store"
    store.mkdir()
    with BinaryWeightWriter(store / "weights.bin") as w:
        ra = blobref_to_dict(w.write(np.arange(50, dtype=np.int32)))
        rb = blobref_to_dict(w.write(np.arange(30, dtype=np.float32)))
    (store / "manifest.json").write_text(json.dumps({"tensors": {"a": {"blobs": {"x": ra}},
                                                                 "b": {"blobs": {"x": rb}}}}))
    assert verify_store(store) == (True, [])
    with open(store / "weights.bin", "r+b") as f:
        f.seek(rb["offset"] + 3)
        f.write(b"\xff")
    assert verify_store(store) == (False, ["b"])
