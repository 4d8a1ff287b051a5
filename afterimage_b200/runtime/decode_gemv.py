"""Fused decode -> GEMV for single-token projections: y = W x with W read
only in its compressed form (aib_decode_gemv_bf16_batch).

In the reference a layer's weights are decoded to BF16 and then consumed by
transformers' nn.Linear (streaming_engine.py:1871-1915 hooks around the
decoder layer) or by the chunked head's F.linear (:2330). For one token
(M = 1) that is a decode writing 2 bytes per weight followed by a GEMV
reading them back; here one kernel decodes each chunk and multiplies it
into the input vector as it goes, so the weights never reach HBM in BF16.
Each chunk's fp32 partial sum lands in a small scratch buffer and a second
kernel sums every row's partials in column order (deterministic), rounding
to BF16 like F.linear's output.

Requirements (checked by the library): the element range is whole rows,
the row length is a multiple of chunk_size, chunk_size is a multiple of 4
and the sign/mantissa bytes are 4-byte aligned.
"""
from __future__ import annotations

import torch

from .. import _lib
from . import _device


def gemv_supported(enc, cols: int, e0: int = 0) -> bool:
    cs = int(enc.chunk_size)
    return cs >= 4 and cs % 4 == 0 and cols % cs == 0 and e0 % cols == 0


def gemv_desc(ds: _device.DeviceStream, tables, enc, e0: int, e1: int, sign_mantissa: torch.Tensor, cols: int,
              x: torch.Tensor, partial: torch.Tensor, y: torch.Tensor) -> _lib.GemvDesc:
    """Descriptor for rows [e0 / cols, e1 / cols) of a compressed [*, cols]
    tensor; `sign_mantissa` starts at element e0, `partial` holds
    (e1 - e0) / chunk_size floats, `y` (e1 - e0) / cols BF16 values."""
    g = _lib.GemvDesc()
    g.stream = _device.make_desc(ds, tables, enc, e0, e1, y, sign_mantissa)
    g.cols = int(cols)
    g.x = x.data_ptr()
    g.partial = partial.data_ptr()
    g.y = y.data_ptr()
    return g


class GemvBatch:
    """A prepared launch: up to AIB_MAX_BATCH descriptors whose pointers stay
    fixed (static x / y / scratch buffers), so a forward issues one library
    call per batch (and a CUDA graph can capture it)."""

    def __init__(self, descs: list, device):
        if not 1 <= len(descs) <= _lib.AIB_MAX_BATCH:
            raise ValueError("a GEMV batch holds 1..%d descriptors" % _lib.AIB_MAX_BATCH)
        self.n = len(descs)
        self.descs = (_lib.GemvDesc * self.n)(*descs)
        self.device = _device.cuda_device(device)

    def launch(self) -> None:
        L = _lib.load()
        with torch.cuda.device(self.device):
            _lib.check(L.aib_decode_gemv_bf16_batch(self.descs, self.n,
                                                    _device.status_word(self.device).data_ptr(),
                                                    _device.stream_ptr(self.device)), "decode_gemv")


def decode_gemv(resident, x: torch.Tensor, rows: tuple[int, int] | None = None,
                synchronize: bool = True) -> torch.Tensor:
    """y = W x for a compressed tensor resident on the device
    (layer_decode.ResidentLayer of shape [R, C]) and x: bf16[C]; `rows`
    restricts to rows [r0, r1). Returns bf16[r1 - r0]."""
    R, C = resident.shape
    r0, r1 = rows if rows is not None else (0, R)
    if not 0 <= r0 <= r1 <= R:
        raise ValueError("row range [%d, %d) outside [0, %d)" % (r0, r1, R))
    dev = resident.sign_mantissa.device
    if x.dtype != torch.bfloat16 or x.numel() != C or x.device != dev:
        raise ValueError("x must be a bf16 vector of %d elements on %s" % (C, dev))
    x = x.contiguous().reshape(-1)
    enc = resident.encoded
    cs = int(enc.chunk_size)
    y = torch.empty(r1 - r0, dtype=torch.bfloat16, device=dev)
    partial = torch.empty(max(1, (r1 - r0) * C // cs), dtype=torch.float32, device=dev)
    e0, e1 = r0 * C, r1 * C
    g = gemv_desc(resident.stream, resident.tables, enc, e0, e1, resident.sign_mantissa[e0:], C, x, partial, y)
    GemvBatch([g], dev).launch()
    if synchronize:
        _device.check_status(dev)
    return y
