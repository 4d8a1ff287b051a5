"""Fused decode -> GEMV (aib_decode_gemv_bf16_batch) on the GPU: y = W x
from the compressed stream against a float64 product of the bit-exact
weights (the decoded W is the reference encoder's input), within BF16
output rounding plus fp32 accumulation error; deterministic; batches,
row ranges, every chunk-size path, corrupt offsets."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _resident(W, cs):
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.layer_decode import upload_layer
    return upload_layer(compress_layer(W, chunk_size=cs), "cuda")


def _ref(W, x, r0=0, r1=None):
    Wd = W[r0:r1].double()
    xd = x.double().cpu()
    ref = Wd @ xd
    mag = Wd.abs() @ xd.abs()
    return ref, mag


def _close(y, ref, mag):
    y = y.double().cpu()
    # BF16 output rounding (half an ulp: 2^-9 relative) + fp32 accumulation
    tol = ref.abs() * 2.0 ** -8 + mag * 1e-5 + 1e-30
    bad = (y - ref).abs() > tol
    assert not bool(bad.any()), (int(bad.sum()), float((y - ref).abs().max()))


@pytest.mark.parametrize("shape,cs", [((1024, 4096), 1024), ((512, 5120), 1024), ((640, 1280), 640),
                                      ((256, 2176), 1088), ((300, 256), 64), ((33, 96), 4), ((64, 1024), 1024), ((40, 32768), 1024)])
def test_gemv_matches_float64_reference(shape, cs):
    g = torch.Generator().manual_seed(shape[0] + cs)
    W = (torch.randn(*shape, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(shape[1], generator=g).to(torch.bfloat16)
    from afterimage_b200.runtime.decode_gemv import decode_gemv
    res = _resident(W, cs)
    y = decode_gemv(res, x.cuda())
    assert y.shape == (shape[0],) and y.dtype == torch.bfloat16
    _close(y, *_ref(W, x))
    # deterministic: the same bits again
    assert torch.equal(decode_gemv(res, x.cuda()).view(torch.int16), y.view(torch.int16))


def test_gemv_agrees_with_linear_on_decoded_weights():
    from afterimage_b200.runtime.decode_gemv import decode_gemv
    g = torch.Generator().manual_seed(1)
    W = (torch.randn(5120, 5120, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(5120, generator=g).to(torch.bfloat16)
    y = decode_gemv(_resident(W, 1024), x.cuda()).double().cpu()
    lin = torch.nn.functional.linear(x.cuda()[None], W.cuda())[0].double().cpu()
    ref, mag = _ref(W, x)
    # both round a float sum to BF16 in their own order: within two BF16 ulps
    # (plus accumulation error) of each other, and the fused one is the
    # closer to the float64 product on average
    tol = torch.maximum(lin.abs(), y.abs()) * 2.0 ** -6 + mag * 1e-5
    assert bool(((y - lin).abs() <= tol).all()), float((y - lin).abs().max())
    assert float((y - ref).abs().mean()) <= float((lin - ref).abs().mean()) * 1.05


def test_gemv_row_ranges_and_wide_values():
    from afterimage_b200.runtime.decode_gemv import decode_gemv
    g = torch.Generator().manual_seed(2)
    W = torch.randn(700, 2048, generator=g) * torch.logspace(-4, 3, 2048)[None, :]
    W = W.to(torch.bfloat16)
    x = torch.randn(2048, generator=g).to(torch.bfloat16)
    res = _resident(W, 512)
    for r0, r1 in ((0, 700), (0, 1), (17, 450), (699, 700), (300, 300)):
        y = decode_gemv(res, x.cuda(), rows=(r0, r1))
        assert y.shape == (r1 - r0,)
        if r1 > r0:
            _close(y, *_ref(W, x, r0, r1))


def test_gemv_batch_mixed_chunk_sizes_in_one_launch():
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.decode_gemv import GemvBatch, gemv_desc
    shapes = [((1024, 5120), 1024), ((256, 5120), 1024), ((512, 640), 640), ((128, 2176), 1088), ((96, 512), 64)]
    Ws, xs, ys, keep, descs = [], [], [], [], []
    for i, ((R, C), cs) in enumerate(shapes):
        g = torch.Generator().manual_seed(10 + i)
        W = (torch.randn(R, C, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(C, generator=g).to(torch.bfloat16).cuda()
        res = _resident(W, cs)
        y = torch.empty(R, dtype=torch.bfloat16, device="cuda")
        part = torch.empty(R * C // cs, dtype=torch.float32, device="cuda")
        descs.append(gemv_desc(res.stream, res.tables, res.encoded, 0, R * C, res.sign_mantissa, C, x, part, y))
        Ws.append(W), xs.append(x), ys.append(y), keep.append((res, part))
    GemvBatch(descs, "cuda").launch()
    _device.check_status(torch.device("cuda", torch.cuda.current_device()))
    for W, x, y in zip(Ws, xs, ys):
        _close(y, *_ref(W, x.cpu()))


def test_gemv_infinities_propagate():
    from afterimage_b200.runtime.decode_gemv import decode_gemv
    W = (torch.randn(64, 256) * 0.02).to(torch.bfloat16)
    W[3, 7] = float("inf")
    W[5, 9] = float("-inf")
    x = torch.ones(256).to(torch.bfloat16)
    y = decode_gemv(_resident(W, 64), x.cuda()).float().cpu()
    assert y[3] == float("inf") and y[5] == float("-inf")
    mask = torch.ones(64, dtype=torch.bool)
    mask[[3, 5]] = False
    assert bool(torch.isfinite(y[mask]).all())


def test_gemv_corrupt_offsets_raise_and_context_survives():
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.decode_gemv import decode_gemv
    from afterimage_b200.runtime.layer_decode import upload_layer
    W = (torch.randn(64, 1024) * 0.02).to(torch.bfloat16)
    layer = compress_layer(W, chunk_size=256)
    offs = np.asarray(layer.encoded.chunk_offsets).copy()
    offs[5] = 10 ** 9
    layer.encoded.chunk_offsets = offs
    res = upload_layer(layer, "cuda")
    with pytest.raises(RuntimeError, match="corrupt offsets"):
        decode_gemv(res, torch.ones(1024, dtype=torch.bfloat16, device="cuda"))
    # the context is still usable
    assert float(torch.ones(4, device="cuda").sum()) == 4.0


def test_gemv_rejects_unsupported_layouts():
    from afterimage_b200.runtime.decode_gemv import decode_gemv
    W = (torch.randn(10, 100) * 0.02).to(torch.bfloat16)
    res = _resident(W, 64)  # a row of 100 is not whole chunks of 64
    with pytest.raises(ValueError, match="cols"):
        decode_gemv(res, torch.ones(100, dtype=torch.bfloat16, device="cuda"))
