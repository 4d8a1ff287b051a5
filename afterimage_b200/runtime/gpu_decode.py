"""int32 exponent decode -- drop-in for the reference's
afterimage/runtime/gpu_decode.py (decode_gpu :61-75): same result (an int32
tensor of n_symbols exponents), same always-synchronise behaviour, computed
by the library's sm_100a decode kernel in its int32-output form."""
from __future__ import annotations

import torch

from . import _device
from .gpu_decode_v2 import prepare_decode_tables


def decode_gpu(enc, device: str = "cuda") -> torch.Tensor:
    dev = _device.cuda_device(device)
    with torch.cuda.device(dev):
        n = int(enc.n_symbols)
        out = torch.empty(n, dtype=torch.int32, device=dev)
        if n == 0:
            return out
        t = prepare_decode_tables(enc, dev)
        ds = _device.upload_stream(enc, dev)
        desc = _device.make_desc(ds, t, enc, 0, n, out)
        _device.call("aib_decode_exponents_i32", desc, dev)
        torch.cuda.synchronize(dev)
        _device.check_status(dev)
    return out
