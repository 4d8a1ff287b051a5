"""csrc/gemv.cu: Y = X W^T for 1..8 tokens (the single-token step and the
speculative verification of the tensor-parallel decoder) against a float64
product of the same BF16 inputs: every output within one BF16 rounding step
of the exact value plus the fp32 summation error (the kernel sums in fp32 and
rounds once); the fp32 output within that summation error. (cuBLAS is not
the yardstick: PyTorch lets its split-K BF16 GEMMs reduce in BF16.)"""
import pytest
import torch

from bf16tol import bf16_ulp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k,m", [(7168, 5120, 1), (5120, 17408, 1), (896, 5120, 1), (5120, 640, 1),
                                   (4352, 5120, 1), (5120, 5120, 5), (640, 5120, 8), (100, 24, 3), (1, 8, 8),
                                   (3, 2056, 2), (1031, 4104, 7)])
def test_gemv_matches_float64_within_one_bf16_step(n, k, m):
    from afterimage_b200.runtime import tp_ops
    g = torch.Generator(device="cuda").manual_seed(n * 31 + k + m)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    exact = x.double() @ w.double().t()
    got = tp_ops.gemv(x, w)
    assert got.shape == (m, n) and got.dtype == torch.bfloat16
    # one BF16 rounding of an fp32 sum: one step of the exact value, plus the fp32 summation
    # error, which dominates near zero (k * 2^-24 * sum |x w|)
    slack = k * 2.0 ** -24 * (x.abs().double() @ w.abs().double().t())
    d = (got.double() - exact).abs()
    assert bool((d <= bf16_ulp(exact).double() + slack).all()), float((d - slack).max())
    f32 = tp_ops.gemv(x, w, out_dtype=torch.float32)
    assert f32.dtype == torch.float32
    assert bool(((f32.double() - exact).abs() <= slack + 1e-7 * exact.abs()).all())


def test_gemv_strided_operands_and_rejects_bad_shapes():
    from afterimage_b200.runtime import tp_ops
    g = torch.Generator(device="cuda").manual_seed(5)
    wbig = (torch.randn(300, 1024, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w = wbig[:, :512]               # row stride 1024, k 512
    xbig = torch.randn(4, 768, device="cuda", generator=g).to(torch.bfloat16)
    x = xbig[:, 256:768]            # row stride 768, 16-byte aligned start
    out = torch.full((4, 400), -7.0, device="cuda", dtype=torch.bfloat16)
    tp_ops.gemv(x, w, out=out[:, :300])
    assert bool((out[:, 300:] == -7.0).all())
    exact = x.double() @ w.double().t()
    assert bool(((out[:, :300].double() - exact).abs() <= bf16_ulp(exact).double()).all())
    with pytest.raises(ValueError):
        tp_ops.gemv(torch.randn(9, 64, device="cuda").to(torch.bfloat16), w[:, :64])   # m > 8
    with pytest.raises(ValueError):
        tp_ops.gemv(x[:, :12], w[:, :12])                                               # k not a multiple of 8
