"""Device plumbing shared by the decode entry points: device resolution
(CUDA only -- there is no CPU fallback), host->device uploads of a
ChunkedEncoded stream, the per-device status word, and descriptor
construction for the C ABI."""
from __future__ import annotations

import ctypes
import dataclasses
import threading

import numpy as np
import torch

from .. import _lib

_status_lock = threading.Lock()
_status: dict[int, torch.Tensor] = {}


def cuda_device(device) -> torch.device:
    """The CUDA device a call targets; raises for anything else. The product
    path has no CPU decoder (the reference's CPU decoders are the test
    oracle in oracle/)."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError(
            f"afterimage_b200 decodes on CUDA devices only (got device={device!r}); "
            "there is no CPU fallback")
    if not torch.cuda.is_available():
        raise RuntimeError("afterimage_b200: CUDA is not available")
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    _lib.load()  # fail loudly if the CUDA library is missing
    return dev


def stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def status_word(dev: torch.device) -> torch.Tensor:
    """Per-device int32 the kernels OR AIB_STATUS_* bits into."""
    with _status_lock:
        t = _status.get(dev.index)
        if t is None:
            t = torch.zeros(1, dtype=torch.int32, device=dev)
            _status[dev.index] = t
        return t


def check_status(dev: torch.device) -> None:
    """Reads (and clears) the device status word; raises on corrupt input.
    Synchronises the current stream. A CPU device (the host-only tensor-parallel
    tests) has no decode kernels and nothing to check."""
    if torch.device(dev).type != "cuda":
        return
    t = status_word(dev)
    v = int(t.item())
    if v:
        t.zero_()
        bits = []
        if v & _lib.STATUS_BAD_CHUNK_RANGE:
            bits.append("a chunk's byte range lies outside the packed stream (corrupt offsets)")
        if v & _lib.STATUS_WAIT_TIMEOUT:
            bits.append("a bounded shared-memory copy wait timed out")
        if v & _lib.STATUS_PEER_TIMEOUT:
            bits.append("a one-shot all-reduce gave up waiting for a peer rank")
        if v & ~(_lib.STATUS_BAD_CHUNK_RANGE | _lib.STATUS_WAIT_TIMEOUT | _lib.STATUS_PEER_TIMEOUT):
            bits.append(f"status bits 0x{v:x}")
        raise RuntimeError("afterimage_b200 decode failed: " + "; ".join(bits))


def upload(arr: np.ndarray, dev: torch.device, dtype=None) -> torch.Tensor:
    a = np.ascontiguousarray(arr if dtype is None else np.asarray(arr, dtype=dtype))
    if not a.flags.writeable:
        a = a.copy()
    return torch.from_numpy(a).to(device=dev)


def upload_padded_u8(arr: np.ndarray, dev: torch.device) -> tuple[torch.Tensor, int, int]:
    """uint8 bytes into a 16-byte aligned device buffer whose size is a
    multiple of 16 (>= 16); returns (tensor, nbytes, capacity)."""
    a = np.ascontiguousarray(arr, dtype=np.uint8).reshape(-1)
    n = int(a.shape[0])
    cap = max(16, (n + 15) // 16 * 16)
    t = torch.empty(cap, dtype=torch.uint8, device=dev)
    if n:
        src = a if a.flags.writeable else a.copy()
        t[:n].copy_(torch.from_numpy(src))
    return t, n, cap


@dataclasses.dataclass
class DeviceStream:
    """A chunk range [c0, c1) of one tensor's compressed stream on a device."""
    packed: torch.Tensor
    nbytes: int
    capacity: int
    offset_base: int
    offsets: torch.Tensor
    chunk_nbytes: torch.Tensor
    chunk_base: int
    # striped layout (aib_stripe_stream): each group's first 16-byte block;
    # None for the reference layout
    stripe_base: torch.Tensor | None = None

    @property
    def striped(self) -> bool:
        return self.stripe_base is not None


def upload_stream(enc, dev: torch.device, c0: int = 0, c1: int | None = None) -> DeviceStream:
    """Uploads chunks [c0, c1): the byte span they occupy (+ the 8-byte
    slack the reference keeps after a slice, compressed_store.py:141-146)
    and their offset / byte-count entries."""
    c1 = int(enc.n_chunks if c1 is None else c1)
    c0 = int(c0)
    if c1 <= c0:
        packed, n, cap = upload_padded_u8(np.zeros(0, np.uint8), dev)
        empty = torch.zeros(1, dtype=torch.int32, device=dev)
        return DeviceStream(packed, n, cap, 0, empty, empty, c0)
    offs = np.asarray(enc.chunk_offsets)
    nbs = np.asarray(enc.chunk_nbytes)
    byte_start = int(offs[c0]) if c0 > 0 else 0
    if c0 == 0 and c1 == enc.n_chunks:
        byte_end = int(np.asarray(enc.packed).shape[0])
    else:
        byte_end = min(int(offs[c1 - 1]) + int(nbs[c1 - 1]) + 8, int(np.asarray(enc.packed).shape[0]))
    packed, n, cap = upload_padded_u8(np.asarray(enc.packed)[byte_start:byte_end], dev)
    return DeviceStream(packed=packed, nbytes=n, capacity=cap, offset_base=byte_start,
                        offsets=upload(offs[c0:c1], dev, np.int32),
                        chunk_nbytes=upload(nbs[c0:c1], dev, np.int32), chunk_base=c0)


def stripe_layout(chunk_nbytes: np.ndarray) -> np.ndarray:
    """int64[ceil(n / 32) + 1]: each chunk group's first block in the striped
    layout, then the total (aib_stripe_layout)."""
    nbs = np.ascontiguousarray(chunk_nbytes, dtype=np.int32)
    n = int(nbs.shape[0])
    base = np.zeros((n + 31) // 32 + 1, dtype=np.int64)
    total = ctypes.c_int64(0)
    _lib.check(_lib.load().aib_stripe_layout(nbs.ctypes.data if n else None, n, base.ctypes.data,
                                             ctypes.byref(total)), "stripe_layout")
    return base


def stripe_host(packed: np.ndarray, chunk_offsets: np.ndarray, chunk_nbytes: np.ndarray,
                offset_base: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(striped bytes, group_base) of a reference-layout stream, made on the
    host (aib_stripe_stream_host) for images that are built on the host."""
    src = np.ascontiguousarray(packed, dtype=np.uint8)
    offs = np.ascontiguousarray(chunk_offsets, dtype=np.int32)
    nbs = np.ascontiguousarray(chunk_nbytes, dtype=np.int32)
    base = stripe_layout(nbs)
    out = np.zeros(max(16, int(base[-1]) * 16), dtype=np.uint8)
    if nbs.shape[0]:
        _lib.check(_lib.load().aib_stripe_stream_host(
            src.ctypes.data, src.shape[0], int(offset_base), offs.ctypes.data, nbs.ctypes.data, nbs.shape[0],
            base.ctypes.data, out.ctypes.data, out.shape[0]), "stripe_stream_host")
    return out[:int(base[-1]) * 16], base


def stripe_stream(ds: DeviceStream, chunk_nbytes: np.ndarray, dev: torch.device) -> DeviceStream:
    """The striped copy of a reference-layout device stream (chunk_base a
    multiple of 32). `chunk_nbytes` is the host copy of ds.chunk_nbytes'
    entries. Stream-ordered on the current stream; ds.packed can be dropped
    once this is enqueued (the caching allocator reuses it in stream order)."""
    if ds.striped:
        return ds
    if ds.chunk_base % 32:
        raise ValueError(f"striping needs a chunk range starting at a multiple of 32, got {ds.chunk_base}")
    nbs = np.ascontiguousarray(chunk_nbytes, dtype=np.int32)
    n = int(nbs.shape[0])
    base = stripe_layout(nbs)
    total = int(base[-1]) * 16
    cap = max(16, total)
    # the kernel writes every block of every group region; a stream with no
    # blocks keeps its one (never read) block zeroed
    dst = torch.empty(cap, dtype=torch.uint8, device=dev) if total else torch.zeros(cap, dtype=torch.uint8,
                                                                                     device=dev)
    d_base = torch.from_numpy(base).to(dev)
    if n:
        _lib.check(_lib.load().aib_stripe_stream(
            ds.packed.data_ptr(), ds.nbytes, ds.offset_base, ds.offsets.data_ptr(), ds.chunk_nbytes.data_ptr(),
            ds.chunk_base, n, d_base.data_ptr(), dst.data_ptr(), cap, status_word(dev).data_ptr(),
            stream_ptr(dev)), "stripe_stream")
    return DeviceStream(packed=dst, nbytes=total, capacity=cap, offset_base=0, offsets=ds.offsets,
                        chunk_nbytes=ds.chunk_nbytes, chunk_base=ds.chunk_base, stripe_base=d_base)


def make_desc(ds: DeviceStream, tables, enc, e0: int, e1: int, out: torch.Tensor,
              sign_mantissa: torch.Tensor | None = None) -> _lib.StreamDesc:
    d = _lib.StreamDesc()
    d.packed = ds.packed.data_ptr()
    d.packed_capacity = ds.capacity
    d.packed_nbytes = ds.nbytes
    d.offset_base = ds.offset_base
    d.chunk_offsets = ds.offsets.data_ptr()
    d.chunk_nbytes = ds.chunk_nbytes.data_ptr()
    d.chunk_base = ds.chunk_base
    d.tables = tables.block.data_ptr()
    d.sym_lut = tables.sym_lut.data_ptr()
    d.len_lut = tables.len_lut.data_ptr()
    d.max_bits = int(enc.max_bits)
    d.chunk_size = int(enc.chunk_size)
    d.n_symbols = int(enc.n_symbols)
    d.elem_begin = int(e0)
    d.elem_end = int(e1)
    d.sign_mantissa = sign_mantissa.data_ptr() if sign_mantissa is not None else None
    d.out = out.data_ptr()
    d.stripe_base = ds.stripe_base.data_ptr() if ds.stripe_base is not None else None
    return d


def call(fn_name: str, desc: _lib.StreamDesc, dev: torch.device) -> None:
    L = _lib.load()
    fn = getattr(L, fn_name)
    _lib.check(fn(ctypes.byref(desc), status_word(dev).data_ptr(), stream_ptr(dev)), fn_name)
