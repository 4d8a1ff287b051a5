"""Whole-layer decode: every compressed tensor of one decoder layer in ONE
kernel launch (aib_decode_bf16_batch).

This is the decode step of the layer streamer. The reference decodes a
layer tensor by tensor, each with its own host->device copies, Triton
launch and synchronisation (streaming_engine.py:1834-1842 -> _decode_tensor
:1074-1138 -> decompress_layer_gpu). Here a layer's tensors are uploaded on
the current stream (asynchronously when their host arrays live in pinned
memory, see `pin_layer`) and decoded by a single batched launch into BF16
outputs allocated through PyTorch's caching allocator.

`ResidentLayer` keeps a layer's compressed form on the device (stream,
sign/mantissa bytes, decode tables) so that it can be decoded repeatedly
with no host traffic -- the VRAM-resident compressed tier.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from .. import _lib
from . import _device
from . import gpu_decode_v2 as _gd
from .compressed_store import CompressedLayer
from .huffman_chunked import ChunkedEncoded


def _pinned_copy(a: np.ndarray) -> tuple[np.ndarray, torch.Tensor]:
    a = np.ascontiguousarray(a)
    t = torch.empty(a.shape, dtype=torch.from_numpy(a[:0].copy()).dtype, pin_memory=True)
    arr = t.numpy()
    arr[...] = a
    return arr, t


def pin_layer(layer: CompressedLayer) -> CompressedLayer:
    """A copy of `layer` whose arrays live in page-locked host memory, so
    that uploads are asynchronous DMA copies. The pinned tensors are kept
    alive by the returned object (attribute `_pinned`)."""
    enc = layer.encoded
    keep = []
    fields = {}
    for name in ("packed", "chunk_offsets", "chunk_nbytes", "sym_lut", "len_lut"):
        arr, t = _pinned_copy(np.asarray(getattr(enc, name)))
        fields[name] = arr
        keep.append(t)
    sm = torch.empty(layer.sign_mantissa.numel(), dtype=torch.uint8, pin_memory=True)
    sm.copy_(layer.sign_mantissa.reshape(-1))
    keep.append(sm)
    new_enc = ChunkedEncoded(max_bits=enc.max_bits, chunk_size=enc.chunk_size,
                             n_symbols=enc.n_symbols, shape=enc.shape, **fields)
    out = CompressedLayer(sign_mantissa=sm, encoded=new_enc, shape=layer.shape)
    out._pinned = keep  # type: ignore[attr-defined]
    return out


def _h2d(a, dev: torch.device, dtype=None) -> torch.Tensor:
    t = a if isinstance(a, torch.Tensor) else torch.from_numpy(
        np.ascontiguousarray(a if dtype is None else np.asarray(a, dtype=dtype)))
    return t.to(device=dev, non_blocking=t.is_pinned())


@dataclasses.dataclass
class ResidentLayer:
    """One tensor's compressed form resident on a device."""
    stream: _device.DeviceStream
    sign_mantissa: torch.Tensor
    tables: _gd.DecodeTables
    encoded: ChunkedEncoded
    shape: tuple

    @property
    def n(self) -> int:
        return int(self.encoded.n_symbols)


def upload_layer(layer: CompressedLayer, device, striped: bool = False) -> ResidentLayer:
    """Host -> device copy of one compressed tensor plus its decode tables
    (stream-ordered; asynchronous for pinned host arrays). `striped` keeps the
    stream in the striped device layout (aib_stripe_stream), which the decode
    kernel reads with one coalesced 512-byte copy per warp step instead of 32
    scattered 16-byte ones; the decoded output is the same."""
    dev = _device.cuda_device(device)
    enc = layer.encoded
    with torch.cuda.device(dev):
        packed_np = np.asarray(enc.packed)
        n = int(packed_np.shape[0])
        cap = max(16, (n + 15) // 16 * 16)
        packed = torch.empty(cap, dtype=torch.uint8, device=dev)
        if n:
            src = torch.from_numpy(packed_np) if packed_np.flags.writeable else torch.from_numpy(packed_np.copy())
            packed[:n].copy_(src, non_blocking=src.is_pinned())
        ds = _device.DeviceStream(packed=packed, nbytes=n, capacity=cap, offset_base=0,
                                  offsets=_h2d(enc.chunk_offsets, dev, np.int32) if enc.n_chunks else
                                  torch.zeros(1, dtype=torch.int32, device=dev),
                                  chunk_nbytes=_h2d(enc.chunk_nbytes, dev, np.int32) if enc.n_chunks else
                                  torch.zeros(1, dtype=torch.int32, device=dev),
                                  chunk_base=0)
        if striped:
            ds = _device.stripe_stream(ds, np.asarray(enc.chunk_nbytes), dev)
        sm = _h2d(layer.sign_mantissa.reshape(-1), dev)
        sym = _h2d(enc.sym_lut, dev, np.int32)
        ln = _h2d(enc.len_lut, dev, np.int8)
        if int(np.asarray(enc.sym_lut).max(initial=0)) > 255:
            raise AssertionError("decoder output is uint8; symbol alphabet must fit in a byte")
        if not 0 <= int(enc.max_bits) <= 16:
            raise ValueError(f"max_bits must be in [0, 16] for the CUDA decoder, got {enc.max_bits}")
        L = _lib.load()
        block = torch.empty(int(L.aib_tables_bytes()), dtype=torch.uint8, device=dev)
        _lib.check(L.aib_build_tables(sym.data_ptr(), ln.data_ptr(), int(enc.max_bits), block.data_ptr(),
                                      _device.stream_ptr(dev)), "build_tables")
        tables = _gd.DecodeTables(sym, ln, block, int(enc.max_bits))
    return ResidentLayer(stream=ds, sign_mantissa=sm, tables=tables, encoded=enc, shape=tuple(layer.shape))


class LayerDecoder:
    """Decodes lists of resident (or host) compressed tensors, up to
    AIB_MAX_BATCH per kernel launch, on torch.cuda.current_stream(device)."""

    def __init__(self, device="cuda", max_ctas: int = 0):
        self.device = _device.cuda_device(device)
        self.launches = 0
        # > 0: each launch uses at most this many CTAs (one per SM), leaving
        # the other SMs to kernels on other streams (aib_decode_bf16_batch_ctas)
        self.max_ctas = int(max_ctas)

    def descriptors(self, tensors: list[ResidentLayer], outs: list[torch.Tensor]):
        descs = (_lib.StreamDesc * len(tensors))()
        for i, (r, o) in enumerate(zip(tensors, outs)):
            descs[i] = _device.make_desc(r.stream, r.tables, r.encoded, 0, r.n, o, r.sign_mantissa)
        return descs

    def launch(self, descs, count: int, max_ctas: int | None = None) -> None:
        """One batched decode launch over prepared descriptors (at most
        `max_ctas` CTAs when given, else self.max_ctas; 0 = no cap)."""
        L = _lib.load()
        cap = self.max_ctas if max_ctas is None else int(max_ctas)
        with torch.cuda.device(self.device):
            for s in range(0, count, _lib.AIB_MAX_BATCH):
                k = min(_lib.AIB_MAX_BATCH, count - s)
                base = _lib.ctypes.addressof(descs) + s * _lib.ctypes.sizeof(_lib.StreamDesc)
                ptr = _lib.ctypes.cast(base, _lib.ctypes.POINTER(_lib.StreamDesc))
                status = _device.status_word(self.device).data_ptr()
                if cap > 0:
                    _lib.check(L.aib_decode_bf16_batch_ctas(ptr, k, cap, status,
                                                            _device.stream_ptr(self.device)), "decode_bf16_batch_ctas")
                else:
                    _lib.check(L.aib_decode_bf16_batch(ptr, k, status, _device.stream_ptr(self.device)),
                               "decode_bf16_batch")
                self.launches += 1

    def decode(self, tensors: list[ResidentLayer], outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
        if outs is None:
            outs = [torch.empty(r.shape, dtype=torch.bfloat16, device=self.device) for r in tensors]
        live = [(r, o) for r, o in zip(tensors, outs) if r.n > 0]
        if live:
            descs = self.descriptors([r for r, _ in live], [o for _, o in live])
            self.launch(descs, len(live))
        return outs

    def decode_host(self, layers: list[CompressedLayer]) -> list[torch.Tensor]:
        """Upload (pinned -> async) and decode a layer's tensors; the device
        copies are released to the caching allocator once the decode is
        enqueued (stream-ordered reuse)."""
        resident = [upload_layer(layer, self.device) for layer in layers]
        return self.decode(resident)
