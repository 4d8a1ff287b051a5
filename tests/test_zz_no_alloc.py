"""aib_decode_gemv_bf16_batch_noalloc: the fused decode -> GEMV for callers
that cannot allocate device memory (they hold only device pointers handed to
them, or run under an allocator that must account for every byte). The
partial sums live in the library's own fixed array instead of a caller
buffer. Results must equal the entry point that takes a caller buffer, on
consecutive calls that reuse the shared array; oversized batches are refused
on the host. This file is collected last."""
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


def test_noalloc_counts_the_aligned_areas_and_rejects_bogus_ranges_without_a_gpu():
    """Each descriptor's area starts 256-byte aligned: two descriptors whose
    partial counts sum to exactly the array's size do not fit once the first
    is padded to 64 floats. Ranges past n_symbols are refused before any
    sum is formed (no overflow from bogus sizes)."""
    L = _lib.load()
    gs = (_lib.GemvDesc * 2)()
    for g, chunks in zip(gs, (1, _lib.AIB_GEMV_SCRATCH_FLOATS - 1)):
        g.stream.chunk_size = 16
        g.stream.n_symbols = g.stream.elem_end = 16 * chunks
    assert L.aib_decode_gemv_bf16_batch_noalloc(gs, 2, None, None) == _lib.AIB_EINVAL
    assert b"scratch" in L.aib_last_error()
    g = _lib.GemvDesc()
    g.stream.chunk_size = 1
    g.stream.n_symbols = 16
    g.stream.elem_end = 2 ** 62   # past n_symbols
    assert L.aib_decode_gemv_bf16_batch_noalloc(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"element range" in L.aib_last_error()
    g.stream.n_symbols = g.stream.elem_end = 2 ** 62   # consistent but far too large
    assert L.aib_decode_gemv_bf16_batch_noalloc(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"scratch" in L.aib_last_error()


@pytest.mark.gpu
def test_noalloc_matches_caller_scratch_on_two_calls_in_a_row():
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.decode_gemv import gemv_desc
    from afterimage_b200.runtime.layer_decode import upload_layer
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = _lib.load()
    st = _device.status_word(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # partial counts 5120, 512, 256 and 3: the last is no multiple of 64, so
    # the next descriptor's area would start after 61 floats of padding
    shapes = [((1024, 5120), 1024), ((512, 640), 640), ((128, 2176), 1088), ((3, 1024), 1024),
              ((64, 512), 512)]
    layers = []
    for i, ((R, C), cs) in enumerate(shapes):
        g = torch.Generator().manual_seed(40 + i)
        W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
        layers.append((R, C, cs, upload_layer(compress_layer(W, chunk_size=cs), dev)))

    def run(entry, xs, with_partial):
        ys, keep, descs = [], [], []
        for (R, C, cs, res), x in zip(layers, xs):
            y = torch.full((R,), float("nan"), dtype=torch.bfloat16, device=dev)
            part = torch.empty(R * C // cs, dtype=torch.float32, device=dev) if with_partial else None
            d = gemv_desc(res.stream, res.tables, res.encoded, 0, R * C, res.sign_mantissa, C, x,
                          part if part is not None else y, y)
            if not with_partial:
                d.partial = None  # the entry point supplies its own scratch
            descs.append(d)
            ys.append(y)
            keep.append(part)
        arr = (_lib.GemvDesc * len(descs))(*descs)
        _lib.check(entry(arr, len(descs), st.data_ptr(), stream))
        torch.cuda.synchronize(dev)
        assert int(st.item()) == 0
        return ys

    for call in range(2):  # the second call finds the first call's partial sums in the array
        g = torch.Generator().manual_seed(100 + call)
        xs = [torch.randn(C, generator=g).to(torch.bfloat16).to(dev) for _, C, _, _ in layers]
        want = run(L.aib_decode_gemv_bf16_batch, xs, True)
        got = run(L.aib_decode_gemv_bf16_batch_noalloc, xs, False)
        for y, w in zip(got, want):
            # same kernels in the same order: bit-identical (tighter than the BF16 tolerance elsewhere)
            assert torch.equal(y.view(torch.int16), w.view(torch.int16)), call
