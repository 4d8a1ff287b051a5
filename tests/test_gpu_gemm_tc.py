"""csrc/gemm_tc.cu: the tcgen05 tensor-core GEMM for a prompt's projections,
Y = X W^T with BF16 operands and fp32 accumulation, against a float64
product of the same BF16 inputs: every output within one BF16 rounding step
of the exact value plus the fp32 summation error; the device status word
stays clear. Shapes cover the Qwen3-14B layer at 64 prompt tokens (with and
without a K split), ragged row and token tiles, and one token."""
import pytest
import torch

from bf16tol import bf16_ulp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(64, 7168, 5120), (64, 5120, 17408), (64, 34816, 5120), (256, 1024, 1024),
                                   (17, 300, 128), (1, 128, 64), (200, 5120, 640), (9, 896, 5120),
                                   (128, 4352, 5120), (33, 130, 2176)])
def test_tensor_core_gemm_matches_float64(m, n, k):
    from afterimage_b200.runtime import _device, tp_ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, device="cuda", generator=g).to(torch.bfloat16)
    got = tp_ops.gemm_tc(x, w)
    torch.cuda.synchronize()
    _device.check_status(dev)
    exact = x.double() @ w.double().t()
    slack = k * 2.0 ** -24 * (x.abs().double() @ w.abs().double().t())
    d = (got.double() - exact).abs()
    bad = d > bf16_ulp(exact).double() + slack
    assert not bool(bad.any()), (int(bad.sum()), float((d - slack).max()))


def test_tensor_core_gemm_strided_output_and_bad_shapes():
    from afterimage_b200.runtime import tp_ops
    g = torch.Generator(device="cuda").manual_seed(1)
    w = (torch.randn(256, 512, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(40, 512, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.full((40, 300), 3.0, device="cuda", dtype=torch.bfloat16)
    tp_ops.gemm_tc(x, w, out=out[:, :256])
    assert bool((out[:, 256:] == 3.0).all())
    exact = x.double() @ w.double().t()
    slack = 512 * 2.0 ** -24 * (x.abs().double() @ w.abs().double().t())
    assert bool(((out[:, :256].double() - exact).abs() <= bf16_ulp(exact).double() + slack).all())
    with pytest.raises(ValueError):
        tp_ops.gemm_tc(x[:, :100], w[:, :100])          # k not a multiple of 64
    with pytest.raises(ValueError):
        tp_ops.gemm_tc(torch.zeros(257, 512, device="cuda", dtype=torch.bfloat16), w)   # m > 256
