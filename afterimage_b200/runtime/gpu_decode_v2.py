"""Exponent-stream decode on the GPU -- drop-in for the reference's
afterimage/runtime/gpu_decode_v2.py (prepare_decode_tables :71-76,
decode_gpu_v2 :79-117), backed by the sm_100a kernels of
libafterimage_b200.so instead of the Triton kernel.

Semantics kept from the reference:
  * `block_chunks` must be a power of two; anything else raises
    ValueError("... power of 2 ...") before anything is allocated
    (gpu_decode_v2.py:94-95). The CUDA kernel's grouping is fixed (32 chunks
    per warp), so the value is otherwise only validated.
  * `tables=None` prepares tensor-local tables and the call synchronises by
    default; passing prepared tables keeps the call stream-ordered.
  * the result is a uint8 tensor of n_symbols decoded exponents, bit-identical
    to the reference decoder's.
Work is enqueued on torch.cuda.current_stream(device).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _lib
from . import _device


class DecodeTables(tuple):
    """Tensor-local decode tables on the device. It unpacks like the
    reference's (sym_lut, len_lut) pair; `block` is the library's table
    block (a multi-symbol first-level table staged into shared memory by the
    kernel, plus validation flags). The reference LUTs stay resident for
    codes longer than the first level."""

    def __new__(cls, sym_lut: torch.Tensor, len_lut: torch.Tensor, block: torch.Tensor, max_bits: int):
        self = super().__new__(cls, (sym_lut, len_lut))
        self.block = block
        self.max_bits = int(max_bits)
        return self

    @property
    def sym_lut(self) -> torch.Tensor:
        return self[0]

    @property
    def len_lut(self) -> torch.Tensor:
        return self[1]


def _lut(x, dev, np_dtype, torch_dtype) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device=dev, dtype=torch_dtype).contiguous()
    return _device.upload(x, dev, np_dtype)


def _build(sym_lut, len_lut, max_bits: int, dev) -> DecodeTables:
    """Device LUTs (int32 symbols, int8 lengths) plus their table block."""
    mb = int(max_bits)
    if not 0 <= mb <= 16:
        raise ValueError(f"max_bits must be in [0, 16] for the CUDA decoder, got {mb}")
    with torch.cuda.device(dev):
        sym = _lut(sym_lut, dev, np.int32, torch.int32)
        ln = _lut(len_lut, dev, np.int8, torch.int8)
        L = _lib.load()
        block = torch.empty(int(L.aib_tables_bytes()), dtype=torch.uint8, device=dev)
        _lib.check(L.aib_build_tables(sym.data_ptr(), ln.data_ptr(), mb, block.data_ptr(),
                                      _device.stream_ptr(dev)), "prepare_decode_tables")
    return DecodeTables(sym, ln, block, mb)


def prepare_decode_tables(enc, device: str = "cuda") -> DecodeTables:
    """One tensor-local codebook; never cache across unrelated tensors
    (reference gpu_decode_v2.py:71-76). Stream-ordered, no synchronisation."""
    assert np.asarray(enc.sym_lut).max() <= 255, (
        "decoder output is uint8; symbol alphabet must fit in a byte")
    return _build(enc.sym_lut, enc.len_lut, enc.max_bits, _device.cuda_device(device))


def _as_tables(tables, enc, dev) -> DecodeTables:
    """Tables from prepare_decode_tables as they are; a plain (sym_lut,
    len_lut) pair, as the reference's prepare_decode_tables returns, gets
    its table block built here."""
    if isinstance(tables, DecodeTables):
        return tables
    if isinstance(tables, (tuple, list)) and len(tables) == 2:
        return _build(tables[0], tables[1], enc.max_bits, dev)
    raise TypeError("tables must be prepare_decode_tables' result or a (sym_lut, len_lut) pair")


def decode_gpu_v2(enc, block_chunks: int = 32, device: str = "cuda", *,
                  tables: tuple | None = None, synchronize: bool = True) -> torch.Tensor:
    if block_chunks < 1 or block_chunks & (block_chunks - 1) != 0:
        raise ValueError(f"block_chunks must be a power of 2, got {block_chunks}")
    dev = _device.cuda_device(device)
    with torch.cuda.device(dev):
        t = prepare_decode_tables(enc, dev) if tables is None else _as_tables(tables, enc, dev)
        n = int(enc.n_symbols)
        out = torch.empty(n, dtype=torch.uint8, device=dev)
        if n == 0:
            return out
        ds = _device.upload_stream(enc, dev)
        desc = _device.make_desc(ds, t, enc, 0, n, out)
        _device.call("aib_decode_exponents_u8", desc, dev)
        if synchronize:
            torch.cuda.synchronize(dev)
            _device.check_status(dev)
    return out
