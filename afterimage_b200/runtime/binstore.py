"""Compressed-store file I/O -- drop-in for the reference's
afterimage/runtime/binstore.py: one flat `weights.bin` holding every blob
back to back, each described in the manifest by
{offset, nbytes, dtype, shape, crc32}.

Kept semantics (reference file:line): BinaryWeightWriter.write :58-66
(CRC32 at write time), BinaryWeightReader.read :88-107 (optional CRC check,
returns an owning writable copy), read_many :109-192 (coalesces adjacent
blobs into bounded extents, returns arrays in the caller's order plus the
read-call and byte counts; the arrays are non-owning, possibly unaligned
views), read_row :194-205, blobref_to_dict :217-219, verify_store :222-247.

Added for the B200 path: `read_many(..., pinned=True)` reads the extents
straight into page-locked host memory (`PinnedBuffer`), so the arrays it
returns can be uploaded with asynchronous DMA copies and no intermediate
pageable copy; `direct=True` additionally bypasses the page cache with
O_DIRECT (aligned supersets of each extent), falling back to buffered reads
where the filesystem refuses O_DIRECT.
"""
from __future__ import annotations

import dataclasses
import json
import os
import pathlib
import zlib

import numpy as np

_DIRECT_ALIGN = 4096


@dataclasses.dataclass
class BlobRef:
    offset: int
    nbytes: int
    dtype: str
    shape: tuple
    crc32: int = 0


class BinaryWeightWriter:
    """Appends arrays to one file, recording where each one landed."""

    def __init__(self, path):
        self.path = pathlib.Path(path)
        self._fh = open(self.path, "wb")
        self._pos = 0

    def write(self, arr: np.ndarray) -> BlobRef:
        arr = np.ascontiguousarray(arr)
        data = arr.tobytes()
        ref = BlobRef(offset=self._pos, nbytes=len(data), dtype=str(arr.dtype), shape=tuple(arr.shape),
                      crc32=zlib.crc32(data))
        self._fh.write(data)
        self._pos += len(data)
        return ref

    def close(self) -> None:
        self._fh.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _checksum_error(ref: dict, got: int) -> ValueError:
    return ValueError("checksum mismatch at offset %d (%d bytes): store is corrupted -- got crc32=%d, "
                      "manifest says %d" % (ref["offset"], ref["nbytes"], got, ref.get("crc32", 0)))


class PinnedBuffer:
    """Growable page-locked host buffer (torch pinned memory) exposed as a
    numpy uint8 array. Reused across reads; grows by doubling."""

    def __init__(self, nbytes: int = 0):
        self._t = None
        self.array = np.zeros(0, dtype=np.uint8)
        if nbytes:
            self.reserve(nbytes)

    def reserve(self, nbytes: int) -> np.ndarray:
        if nbytes > self.array.shape[0]:
            import torch
            cap = max(nbytes, 2 * self.array.shape[0], _DIRECT_ALIGN)
            cap = (cap + _DIRECT_ALIGN - 1) // _DIRECT_ALIGN * _DIRECT_ALIGN
            self._t = torch.empty(cap, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
            self.array = self._t.numpy()
        return self.array

    @property
    def tensor(self):
        return self._t


class BinaryWeightReader:
    """One open file handle for the store's lifetime.

    `threads` > 1 reads the pinned extents of `read_many` in pieces of
    `piece_bytes` with the library's native thread pool (aib_pread_batch),
    outside the interpreter lock: one thread's page-cache copy rate is a
    few GB/s, and Python reader threads stall on the lock held by the
    forward pass."""

    def __init__(self, path, direct: bool = False, threads: int = 1, piece_bytes: int = 8 << 20):
        self.path = pathlib.Path(path)
        self._fh = open(self.path, "rb")
        self._fd = self._fh.fileno()
        self.threads = max(1, int(threads))
        self.piece_bytes = max(_DIRECT_ALIGN, int(piece_bytes) // _DIRECT_ALIGN * _DIRECT_ALIGN)
        self._direct_fd = None
        if direct and hasattr(os, "O_DIRECT"):
            try:
                self._direct_fd = os.open(self.path, os.O_RDONLY | os.O_DIRECT)
            except OSError:
                self._direct_fd = None

    @property
    def direct(self) -> bool:
        return self._direct_fd is not None

    def read(self, ref: dict, verify: bool = False) -> np.ndarray:
        self._fh.seek(ref["offset"])
        data = self._fh.read(ref["nbytes"])
        if verify:
            got = zlib.crc32(data)
            if got != ref.get("crc32", 0):
                raise _checksum_error(ref, got)
        return np.frombuffer(data, dtype=ref["dtype"]).copy().reshape(ref["shape"])

    def _pread_full(self, fd: int, start: int, view: memoryview) -> int:
        got = 0
        n = len(view)
        while got < n:
            k = os.preadv(fd, [view[got:]], start + got)
            if k <= 0:
                break
            got += k
        return got

    def _native_reads(self, fd: int, spans: list[tuple[int, int, int, int]]) -> None:
        """spans: (file offset, bytes to read, bytes needed, destination
        address). Cut into pieces of piece_bytes and read by the library's
        thread pool in one call (outside the interpreter lock)."""
        import ctypes
        from .. import _lib
        offs, sizes, need, dests = [], [], [], []
        for start, size, needed, addr in spans:
            for o in range(0, size, self.piece_bytes):
                m = min(self.piece_bytes, size - o)
                offs.append(start + o)
                sizes.append(m)
                need.append(max(0, min(m, needed - o)))
                dests.append(addr + o)
        n = len(offs)
        if n == 0:
            return
        A = ctypes.c_int64 * n
        D = ctypes.c_void_p * n
        got = ctypes.c_int64(0)
        L = _lib.load()
        _lib.check(L.aib_pread_batch(fd, A(*offs), A(*sizes), A(*need), D(*dests), n, self.threads,
                                     ctypes.byref(got)), "read_many")

    def _readinto(self, start: int, view: memoryview) -> int:
        """Fill `view` with file bytes [start, start + len(view)). O_DIRECT
        when enabled and the destination/offset/length are sector aligned
        (retrying buffered on EINVAL); buffered otherwise."""
        n = len(view)
        if self._direct_fd is not None and n and start % _DIRECT_ALIGN == 0:
            addr = np.frombuffer(view, dtype=np.uint8).ctypes.data
            if addr % _DIRECT_ALIGN == 0:
                try:
                    return self._pread_full(self._direct_fd, start, view)
                except OSError:
                    os.close(self._direct_fd)
                    self._direct_fd = None
        self._fh.seek(start)
        return self._fh.readinto(view)

    def read_many(self, refs: list[dict], *, max_gap_bytes: int = 0, max_extent_bytes: int = 1 << 28,
                  verify: bool = False, pinned: PinnedBuffer | bool = False, groups: list | None = None
                  ) -> tuple[list[np.ndarray], int, int]:
        """Reads blobs through bounded contiguous extents (reference
        binstore.py:109-192). Returns (arrays in the caller's order, number
        of read calls, bytes read). With `pinned`, every extent lands in one
        page-locked buffer (a PinnedBuffer to reuse, or True for a fresh
        one); the arrays view that buffer and stay valid until it is reused.
        With `groups` (one label per ref), blobs merge only with neighbours
        of the same label: per-tensor extents in one call."""
        if max_gap_bytes < 0:
            raise ValueError("max_gap_bytes must be non-negative")
        if max_extent_bytes < 1:
            raise ValueError("max_extent_bytes must be positive")
        if groups is not None and len(groups) != len(refs):
            raise ValueError("groups needs one label per ref")
        if not refs:
            return [], 0, 0
        ordered = sorted(enumerate(refs), key=lambda item: int(item[1]["offset"]))
        extents: list[dict] = []
        for idx, ref in ordered:
            start = int(ref["offset"])
            end = start + int(ref["nbytes"])
            if end < start:
                raise ValueError("blob extent overflows its offset")
            if extents:
                prev = extents[-1]
                gap = start - prev["end"]
                merged_end = max(prev["end"], end)
                same = groups is None or groups[idx] == groups[prev["items"][-1][0]]
                if same and 0 <= gap <= max_gap_bytes and merged_end - prev["start"] <= max_extent_bytes:
                    prev["end"] = merged_end
                    prev["items"].append((idx, ref))
                    continue
            extents.append({"start": start, "end": end, "items": [(idx, ref)]})

        buf = None
        if pinned:
            buf = pinned if isinstance(pinned, PinnedBuffer) else PinnedBuffer()
            # each extent at a sector-aligned position so O_DIRECT can land in place
            pos = 0
            for e in extents:
                lead = e["start"] % _DIRECT_ALIGN
                e["slot"] = pos + lead
                span = lead + (e["end"] - e["start"])
                pos += (span + _DIRECT_ALIGN - 1) // _DIRECT_ALIGN * _DIRECT_ALIGN
            arena = buf.reserve(pos)

        out: list = [None] * len(refs)
        bytes_read = 0
        if buf is not None and self.threads > 1:
            # every extent of the call in one native batch of parallel positional reads
            base = arena.ctypes.data
            if self.direct:
                spans = []
                for e in extents:
                    lead = e["start"] % _DIRECT_ALIGN
                    span = (lead + e["end"] - e["start"] + _DIRECT_ALIGN - 1) // _DIRECT_ALIGN * _DIRECT_ALIGN
                    spans.append((e["start"] - lead, span, lead + e["end"] - e["start"], base + e["slot"] - lead))
                try:
                    self._native_reads(self._direct_fd, spans)
                except OSError:
                    os.close(self._direct_fd)
                    self._direct_fd = None
            if not self.direct:
                self._native_reads(self._fd, [(e["start"], e["end"] - e["start"], e["end"] - e["start"],
                                              base + e["slot"]) for e in extents])
            for e in extents:
                e["done"] = True
        for e in extents:
            start, nbytes = e["start"], e["end"] - e["start"]
            if buf is not None:
                lead = start % _DIRECT_ALIGN
                a0 = e["slot"] - lead
                span = (lead + nbytes + _DIRECT_ALIGN - 1) // _DIRECT_ALIGN * _DIRECT_ALIGN
                if e.get("done"):
                    got = nbytes
                elif self.direct:
                    got = self._readinto(start - lead, memoryview(arena[a0:a0 + span]))
                    got = min(max(0, got - lead), nbytes)
                else:
                    got = self._readinto(start, memoryview(arena[e["slot"]:e["slot"] + nbytes]))
                data = memoryview(arena[e["slot"]:e["slot"] + nbytes])
            else:
                storage = bytearray(nbytes)
                got = self._readinto(start, memoryview(storage))
                data = memoryview(storage)
            if got != nbytes:
                raise ValueError("short read at offset %d: wanted %d bytes, got %d" % (start, nbytes, got))
            bytes_read += nbytes
            for idx, ref in e["items"]:
                rel = int(ref["offset"]) - start
                blob = data[rel:rel + int(ref["nbytes"])]
                if verify:
                    got_crc = zlib.crc32(blob)
                    if got_crc != ref.get("crc32", 0):
                        raise _checksum_error(ref, got_crc)
                out[idx] = np.frombuffer(blob, dtype=ref["dtype"]).reshape(ref["shape"])
        return out, len(extents), bytes_read

    def read_row(self, base_offset: int, row_index: int, row_nbytes: int, dtype: str) -> np.ndarray:
        """Exactly one row of a row-major 2-D blob (reference :194-205)."""
        self._fh.seek(base_offset + row_index * row_nbytes)
        return np.frombuffer(self._fh.read(row_nbytes), dtype=dtype).copy()

    def read_rows(self, base_offset: int, rows, row_nbytes: int, dtype: str) -> np.ndarray:
        """Several rows (token ids of an embedding gather) in one call."""
        rows = [int(r) for r in rows]
        out = np.empty((len(rows), row_nbytes), dtype=np.uint8)
        for i, r in enumerate(rows):
            self._fh.seek(base_offset + r * row_nbytes)
            if self._fh.readinto(memoryview(out[i])) != row_nbytes:
                raise ValueError("short row read")
        return out.view(dtype).reshape(len(rows), -1)

    def close(self) -> None:
        self._fh.close()
        if self._direct_fd is not None:
            os.close(self._direct_fd)
            self._direct_fd = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def blobref_to_dict(ref: BlobRef) -> dict:
    return {"offset": ref.offset, "nbytes": ref.nbytes, "dtype": ref.dtype, "shape": list(ref.shape),
            "crc32": ref.crc32}


def verify_store(store_dir) -> tuple[bool, list[str]]:
    """Reads every blob once and checks its CRC32 against the manifest;
    returns (ok, keys of the tensors that failed) (reference :222-247)."""
    store_dir = pathlib.Path(store_dir)
    manifest = json.loads((store_dir / "manifest.json").read_text())
    bad = []
    with BinaryWeightReader(store_dir / "weights.bin") as reader:
        for key, meta in manifest["tensors"].items():
            for ref in meta.get("blobs", {}).values():
                if "crc32" not in ref:
                    continue
                try:
                    reader.read(ref, verify=True)
                except ValueError:
                    bad.append(key)
                    break
    return (len(bad) == 0, bad)
