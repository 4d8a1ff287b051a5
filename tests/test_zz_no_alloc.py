"""aib_decode_gemv_bf16_batch_noalloc: the fused decode -> GEMV with the
partial sums in the library's own scratch array (for callers that hold only
device pointers handed to them). Same results, bit for bit, as the entry
point with a caller buffer; oversized batches are refused on the host."""
import ctypes

import pytest
import torch

from afterimage_b200 import _lib


def test_noalloc_refuses_batches_larger_than_the_scratch_without_a_gpu():
    L = _lib.load()
    g = _lib.GemvDesc()
    g.stream.chunk_size = 16
    g.stream.n_symbols = g.stream.elem_end = 16 * (_lib.AIB_GEMV_SCRATCH_FLOATS + 1)
    assert L.aib_decode_gemv_bf16_batch_noalloc(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"scratch" in L.aib_last_error()
    assert L.aib_decode_gemv_bf16_batch_noalloc(ctypes.byref(g), 0, None, None) == _lib.AIB_EINVAL


@pytest.mark.gpu
def test_noalloc_matches_caller_scratch_bit_for_bit():
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.decode_gemv import gemv_desc
    from afterimage_b200.runtime.layer_decode import upload_layer
    dev = torch.device("cuda", 0)
    shapes = [((1024, 5120), 1024), ((512, 640), 640), ((128, 2176), 1088)]
    descs, ys, ys2, keep = [], [], [], []
    for i, ((R, C), cs) in enumerate(shapes):
        g = torch.Generator().manual_seed(40 + i)
        W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(C, generator=g).to(torch.bfloat16).to(dev)
        res = upload_layer(compress_layer(W, chunk_size=cs), dev)
        y = torch.empty(R, dtype=torch.bfloat16, device=dev)
        y2 = torch.empty_like(y)
        part = torch.empty(R * C // cs, dtype=torch.float32, device=dev)
        descs.append(gemv_desc(res.stream, res.tables, res.encoded, 0, R * C, res.sign_mantissa, C, x, part, y))
        d2 = gemv_desc(res.stream, res.tables, res.encoded, 0, R * C, res.sign_mantissa, C, x, part, y2)
        d2.partial = None
        ys.append(y), ys2.append((y2, d2)), keep.append((res, x, part))
    L = _lib.load()
    st = _device.status_word(dev)
    arr = (_lib.GemvDesc * len(descs))(*descs)
    _lib.check(L.aib_decode_gemv_bf16_batch(arr, len(descs), st.data_ptr(), torch.cuda.current_stream().cuda_stream))
    arr2 = (_lib.GemvDesc * len(descs))(*[d for _, d in ys2])
    _lib.check(L.aib_decode_gemv_bf16_batch_noalloc(arr2, len(descs), st.data_ptr(),
                                                    torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for y, (y2, _) in zip(ys, ys2):
        assert torch.equal(y.view(torch.int16), y2.view(torch.int16))
