"""Python side of the fused single-token layer kernels (csrc/tp_ops.cu):
residual add + RMSNorm, q/k RMSNorm + rotary embedding + KV-cache write,
grouped-query attention over the cache, SiLU * up. They replace, for one
token, the chain of small torch ops the tensor-parallel decoder would
otherwise launch between its projections (the layer math of transformers'
Qwen3 / Llama modules, which the reference engine runs). All tensors are
BF16 CUDA tensors except `inv_freq` (fp32) and positions (int64, on the
device so that a captured step reads the current value)."""
from __future__ import annotations

import torch

from .. import _lib


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, eps: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """x += delta (BF16, in place, when given); returns
    weight * rmsnorm(x) per row (transformers' RMSNorm rounding)."""
    cols = x.shape[-1]
    rows = x.numel() // cols
    if out is None:
        out = torch.empty_like(x)
    for t in (x, weight, out) + ((delta,) if delta is not None else ()):
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise ValueError("add_rmsnorm needs contiguous bf16 tensors")
    if delta is not None and delta.numel() != x.numel():
        raise ValueError("delta must match x")
    if weight.numel() != cols or out.numel() != x.numel():
        raise ValueError("weight must have one value per column and out match x")
    L = _lib.load()
    _lib.check(L.aib_add_rmsnorm_bf16(x.data_ptr(), _ptr(delta), weight.data_ptr(), out.data_ptr(), rows, cols,
                                      float(eps), _stream(x)), "add_rmsnorm")
    return out


def qk_rope_cache(qkv: torch.Tensor, T: int, nh: int, nkv: int, hd: int, q_norm: torch.Tensor | None,
                  k_norm: torch.Tensor | None, eps: float, inv_freq: torch.Tensor, pos0: torch.Tensor,
                  q_out: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor) -> None:
    """qkv [T, (nh + 2 nkv) * hd] -> q_out [nh, T, hd]; k and v written into
    the caches [.., nkv, max_len, hd] at positions pos0[0] + t."""
    if qkv.numel() != T * (nh + 2 * nkv) * hd or q_out.numel() != nh * T * hd:
        raise ValueError("qk_rope_cache: shapes do not match")
    if inv_freq.dtype != torch.float32 or pos0.dtype != torch.int64:
        raise ValueError("inv_freq must be fp32 and pos0 int64")
    max_len = k_cache.shape[-2]
    if k_cache.shape[-1] != hd or k_cache.numel() != nkv * max_len * hd or v_cache.shape != k_cache.shape:
        raise ValueError("caches must be [.., nkv, max_len, hd]")
    L = _lib.load()
    _lib.check(L.aib_qk_rope_cache_bf16(qkv.data_ptr(), T, nh, nkv, hd, _ptr(q_norm), _ptr(k_norm), float(eps),
                                        inv_freq.data_ptr(), pos0.data_ptr(), q_out.data_ptr(), k_cache.data_ptr(),
                                        v_cache.data_ptr(), max_len, _stream(qkv)), "qk_rope_cache")


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, nh: int, nkv: int, hd: int,
                     pos: torch.Tensor, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """One query per head over cache positions [0, pos[0]]; returns [nh * hd]."""
    max_len = k_cache.shape[-2]
    if out is None:
        out = torch.empty(nh * hd, dtype=torch.bfloat16, device=q.device)
    L = _lib.load()
    _lib.check(L.aib_decode_attention_bf16(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), nh, nkv, hd,
                                           max_len, pos.data_ptr(), float(scale), out.data_ptr(), _stream(q)),
               "decode_attention")
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """gate_up [T, 2I] -> bf16(bf16(silu(gate)) * up) [T, I]."""
    T = gate_up.numel() // gate_up.shape[-1]
    I = gate_up.shape[-1] // 2
    if out is None:
        out = torch.empty(T, I, dtype=torch.bfloat16, device=gate_up.device)
    L = _lib.load()
    _lib.check(L.aib_silu_mul_bf16(gate_up.data_ptr(), out.data_ptr(), T, I, _stream(gate_up)), "silu_mul")
    return out


def gemv(x: torch.Tensor, w: torch.Tensor, out_dtype=torch.bfloat16, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [m, k] (m <= 8 rows) times w.T, w [n, k] row-major BF16 (csrc/gemv.cu):
    returns [m, n] in BF16 (one rounding of the fp32 sum) or fp32."""
    x2 = x.reshape(-1, x.shape[-1])
    m, k = x2.shape
    n = w.shape[0]
    if x2.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or w.dim() != 2 or w.shape[1] != k:
        raise ValueError("gemv needs bf16 x [m, k] and w [n, k]")
    if x2.stride(-1) != 1 or w.stride(-1) != 1:
        raise ValueError("gemv needs unit stride along k")
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=x.device)
    L = _lib.load()
    _lib.check(L.aib_gemv_bf16(w.data_ptr(), w.stride(0), x2.data_ptr(), x2.stride(0), out.data_ptr(),
                               out.stride(0), n, k, m, int(out.dtype == torch.float32), _stream(x)), "gemv")
    return out.reshape(*x.shape[:-1], n)


def gemm_tc(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [m, k] (1 <= m <= 256 rows) times w.T, w [n, k] row-major BF16, on the
    tensor cores (csrc/gemm_tc.cu); returns BF16 [m, n]. k must be a
    multiple of 64. Raises RuntimeError if a bounded wait in the kernel gave
    up (the status word is read: this synchronises)."""
    from . import _device
    x2 = x.reshape(-1, x.shape[-1])
    m, k = x2.shape
    n = w.shape[0]
    if x2.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or w.dim() != 2 or w.shape[1] != k:
        raise ValueError("gemm_tc needs bf16 x [m, k] and w [n, k]")
    if x2.stride(-1) != 1 or w.stride(-1) != 1:
        raise ValueError("gemm_tc needs unit stride along k")
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    L = _lib.load()
    need = int(L.aib_gemm_bf16_tc_workspace_floats(m, n, k))
    ws = torch.empty(max(need, 1), dtype=torch.float32, device=x.device)
    _lib.check(L.aib_gemm_bf16_tc(w.data_ptr(), w.stride(0), x2.data_ptr(), x2.stride(0), out.data_ptr(),
                                  out.stride(0), m, n, k, ws.data_ptr(), need,
                                  _device.status_word(x.device).data_ptr(), _stream(x)), "gemm_tc")
    return out.reshape(*x.shape[:-1], n)


__all__ = ["add_rmsnorm", "qk_rope_cache", "decode_attention", "silu_mul", "gemv", "gemm_tc"]
