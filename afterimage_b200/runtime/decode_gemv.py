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


def _compare(spec, chunks: dict, device="cuda", reps: int = 50) -> dict:
    """Times one layer's single-token projections: one batched decode
    launch followed by F.linear per tensor, against the fused kernel (per
    dependent launch group, and all tensors in one launch)."""
    import torch.nn.functional as F
    from .compressed_store import compress_layer
    from .layer_decode import LayerDecoder, upload_layer
    dev = _device.cuda_device(device)
    g = torch.Generator(device=dev).manual_seed(7)
    res = []
    for name, r, c in spec:
        W = (torch.randn(r, c, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        res.append(upload_layer(compress_layer(W.cpu(), chunk_size=chunks.get(name, 1024)), dev))
    outs = [torch.empty(r, c, dtype=torch.bfloat16, device=dev) for _, r, c in spec]
    dec = LayerDecoder(dev)
    descs = dec.descriptors(res, outs)
    xs = [torch.randn(c, device=dev, generator=g).to(torch.bfloat16) for _, _, c in spec]
    ys = [torch.empty(r, dtype=torch.bfloat16, device=dev) for _, r, _ in spec]
    parts = [torch.empty(r * c // int(rr.encoded.chunk_size), dtype=torch.float32, device=dev)
             for rr, (_, r, c) in zip(res, spec)]
    gd = [gemv_desc(rr.stream, rr.tables, rr.encoded, 0, r * c, rr.sign_mantissa, c, x, p, y)
          for rr, (_, r, c), x, p, y in zip(res, spec, xs, parts, ys)]
    names = [n for n, _, _ in spec]
    groups = [[names.index(n) for n in grp if n in names]
              for grp in (("q_proj", "k_proj", "v_proj"), ("o_proj",), ("gate_proj", "up_proj"), ("down_proj",))]
    batches = [GemvBatch([gd[i] for i in grp], dev) for grp in groups if grp]
    one = GemvBatch(gd, dev)

    def timed(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / reps

    t_dec = timed(lambda: dec.launch(descs, len(spec)))
    t_lin = timed(lambda: [F.linear(x[None], o) for x, o in zip(xs, outs)])
    t_groups = timed(lambda: [bt.launch() for bt in batches])
    t_one = timed(one.launch)
    _device.check_status(dev)
    return {"weights": sum(r * c for _, r, c in spec), "decode_ms": round(t_dec, 4), "linear_ms": round(t_lin, 4),
            "unfused_ms": round(t_dec + t_lin, 4), "fused_4_launches_ms": round(t_groups, 4),
            "fused_one_launch_ms": round(t_one, 4)}


def main() -> None:
    """python -m afterimage_b200.runtime.decode_gemv: fused vs unfused
    single-token projections of a Qwen3-14B-shaped layer (whole, TP-ready
    chunking, and one rank of TP 8); one JSON line per case."""
    import json
    layer = [("q_proj", 5120, 5120), ("k_proj", 1024, 5120), ("v_proj", 1024, 5120), ("o_proj", 5120, 5120),
             ("gate_proj", 17408, 5120), ("up_proj", 17408, 5120), ("down_proj", 5120, 17408)]
    rank8 = [("q_proj", 640, 5120), ("k_proj", 128, 5120), ("v_proj", 128, 5120), ("o_proj", 5120, 640),
             ("gate_proj", 2176, 5120), ("up_proj", 2176, 5120), ("down_proj", 5120, 1088)]
    tp = {"o_proj": 640, "down_proj": 1088}
    for name, spec, chunks in (("qwen3-14b-layer", layer, {}), ("qwen3-14b-layer-tp8-chunks", layer, tp),
                               ("qwen3-14b-rank-of-tp8", rank8, tp)):
        print(json.dumps({"case": name, **_compare(spec, chunks)}), flush=True)


if __name__ == "__main__":
    main()
