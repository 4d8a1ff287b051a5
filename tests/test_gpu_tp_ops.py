"""The fused single-token layer kernels (csrc/tp_ops.cu) against plain
PyTorch references of the same ops: transformers' BF16 rounding points for
the norms, rotary embedding and SiLU (equal up to one BF16 ulp from fp32
reduction order), an fp32 reference for the attention (BF16 output
tolerance)."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rms(x, w, eps):
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w * h.to(torch.bfloat16)


def _ulp_close(a, b, frac_exact=0.99):
    a, b = a.float(), b.float()
    ulp = torch.maximum(a.abs(), b.abs()) * 2.0 ** -7 + 1e-30
    assert bool(((a - b).abs() <= ulp).all()), float((a - b).abs().max())
    assert float((a == b).float().mean()) >= frac_exact


@pytest.mark.parametrize("rows,cols", [(1, 5120), (3, 320), (64, 1024), (1, 17408)])
@pytest.mark.parametrize("with_delta", [False, True])
def test_add_rmsnorm(rows, cols, with_delta):
    from afterimage_b200.runtime.tp_ops import add_rmsnorm
    g = torch.Generator(device="cuda").manual_seed(rows * cols)
    x = torch.randn(rows, cols, device="cuda", generator=g).to(torch.bfloat16)
    d = torch.randn(rows, cols, device="cuda", generator=g).to(torch.bfloat16) if with_delta else None
    w = (1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).to(torch.bfloat16)
    ref_x = x + d if with_delta else x.clone()
    ref = _rms(ref_x, w, 1e-6)
    out = add_rmsnorm(x, d, w, 1e-6)
    assert torch.equal(x, ref_x)
    _ulp_close(out, ref)


def _rope_ref(x, pos, inv_freq):
    freqs = pos[:, None].float() * inv_freq[None, :]
    emb = torch.cat((freqs, freqs), -1)
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), -1)
    return x * cos + rot * sin


@pytest.mark.parametrize("nh,nkv,hd,T,start,norm", [(40, 8, 128, 1, 70, True), (4, 2, 80, 5, 0, True),
                                                     (32, 8, 128, 1, 3, False), (5, 1, 64, 2, 10, True)])
def test_qk_rope_cache(nh, nkv, hd, T, start, norm):
    from afterimage_b200.runtime.tp_ops import qk_rope_cache
    g = torch.Generator(device="cuda").manual_seed(nh * hd + T)
    max_len = 96
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, device="cuda", generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).to(torch.bfloat16) if norm else None
    kn = (1 + 0.1 * torch.randn(hd, device="cuda", generator=g)).to(torch.bfloat16) if norm else None
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, hd, 2, dtype=torch.int64).to(device="cuda", dtype=torch.float) / hd))
    pos0 = torch.tensor([start], dtype=torch.int64, device="cuda")
    q_out = torch.empty(nh, T, hd, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(1, nkv, max_len, hd, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    qk_rope_cache(qkv, T, nh, nkv, hd, qn, kn, 1e-6, inv_freq, pos0, q_out, kc, vc)
    q = qkv[:, :nh * hd].view(T, nh, hd)
    k = qkv[:, nh * hd:(nh + nkv) * hd].view(T, nkv, hd)
    v = qkv[:, (nh + nkv) * hd:].view(T, nkv, hd)
    if norm:
        q, k = _rms(q, qn, 1e-6), _rms(k, kn, 1e-6)
    pos = torch.arange(start, start + T, device="cuda")
    q_ref = _rope_ref(q.transpose(0, 1), pos, inv_freq)
    k_ref = _rope_ref(k.transpose(0, 1), pos, inv_freq)
    _ulp_close(q_out, q_ref, 0.97)
    _ulp_close(kc[0, :, start:start + T], k_ref, 0.97)
    assert torch.equal(vc[0, :, start:start + T], v.transpose(0, 1))
    assert int(kc[0, :, :start].abs().sum()) == 0 and int(kc[0, :, start + T:].abs().sum()) == 0


@pytest.mark.parametrize("nh,nkv,hd,L", [(40, 8, 128, 65), (4, 2, 80, 1), (8, 8, 64, 300), (5, 1, 128, 4096)])
def test_decode_attention(nh, nkv, hd, L):
    from afterimage_b200.runtime.tp_ops import decode_attention
    g = torch.Generator(device="cuda").manual_seed(L + nh)
    max_len = max(L, 128)
    q = torch.randn(nh, hd, device="cuda", generator=g).to(torch.bfloat16)
    kc = torch.randn(1, nkv, max_len, hd, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(1, nkv, max_len, hd, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([L - 1], dtype=torch.int64, device="cuda")
    scale = hd ** -0.5
    out = decode_attention(q, kc, vc, nh, nkv, hd, pos, scale)
    grp = nh // nkv
    k = kc[0, :, :L].float().repeat_interleave(grp, 0)
    v = vc[0, :, :L].float().repeat_interleave(grp, 0)
    p = torch.softmax((q.float()[:, None, :] @ k.transpose(1, 2))[:, 0] * scale, -1)
    ref = (p[:, None, :] @ v)[:, 0].reshape(-1)
    assert torch.allclose(out.float(), ref, atol=1e-2, rtol=1e-2), float((out.float() - ref).abs().max())
    sdpa = F.scaled_dot_product_attention(q[None, :, None], kc[:, :, :L], vc[:, :, :L], scale=scale,
                                          enable_gqa=nh != nkv)[0, :, 0].reshape(-1)
    assert torch.allclose(out.float(), sdpa.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("T,I", [(1, 17408), (7, 896), (64, 2176)])
def test_silu_mul(T, I):
    from afterimage_b200.runtime.tp_ops import silu_mul
    g = torch.Generator(device="cuda").manual_seed(T * I)
    gu = (3 * torch.randn(T, 2 * I, device="cuda", generator=g)).to(torch.bfloat16)
    out = silu_mul(gu)
    ref = F.silu(gu[:, :I]) * gu[:, I:]
    _ulp_close(out, ref)
