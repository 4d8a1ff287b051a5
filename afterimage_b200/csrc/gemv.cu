// sm_100a BF16 GEMV for the projections that consume a decoded layer when
// few tokens pass through it: Y[m, n] = sum_k X[m, k] * W[n, k] for m <= 8
// tokens (one token of greedy decoding; the k + 1 tokens of a speculative
// verification), W row-major [n, k] as nn.Linear stores it. It replaces, for
// these shapes, the nn.Linear / F.linear the reference calls on the decoded
// weights (afterimage/runtime/streaming_engine.py:1871-1915, :2330).
//
// Such a product reads every weight once and does 2m flops per weight: it is
// bound by HBM, so the kernel is built to keep enough weight bytes in
// flight. Each warp owns kRows rows; every lane streams 16-byte pieces of
// those rows (L1 no-allocate, L2 evict-first: the weights are read once) two
// pieces per row ahead, multiplies them into fp32 accumulators against the
// tokens' activations (read through L1, shared by the CTA's warps), and the
// warp sums its lanes with shuffles. When the rows are too few to fill the
// GPU, S warps split a row group's K range and add their sums through shared
// memory. The sum over k is kept in fp32 and rounded once, as one BF16 GEMM
// with fp32 accumulation rounds it (the order of the additions differs).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "aib_internal.h"

namespace aibgemv {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 2;  // rows per warp

__device__ __forceinline__ uint64_t policy_stream() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint4 ld_weights(const void *p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

// eight BF16 products added into acc (fp32)
__device__ __forceinline__ float dot8(uint4 w, uint4 x, float acc) {
  acc = fmaf(__uint_as_float(w.x << 16), __uint_as_float(x.x << 16), acc);
  acc = fmaf(__uint_as_float(w.x & 0xFFFF0000u), __uint_as_float(x.x & 0xFFFF0000u), acc);
  acc = fmaf(__uint_as_float(w.y << 16), __uint_as_float(x.y << 16), acc);
  acc = fmaf(__uint_as_float(w.y & 0xFFFF0000u), __uint_as_float(x.y & 0xFFFF0000u), acc);
  acc = fmaf(__uint_as_float(w.z << 16), __uint_as_float(x.z << 16), acc);
  acc = fmaf(__uint_as_float(w.z & 0xFFFF0000u), __uint_as_float(x.z & 0xFFFF0000u), acc);
  acc = fmaf(__uint_as_float(w.w << 16), __uint_as_float(x.w << 16), acc);
  acc = fmaf(__uint_as_float(w.w & 0xFFFF0000u), __uint_as_float(x.w & 0xFFFF0000u), acc);
  return acc;
}

// Warp w of a CTA: row group (w / S) of the CTA's kWarps / S groups, K slice
// (w % S). Lane l covers elements 8 * (32 * j + l) .. + 8 of the slice's
// 256-element steps j = s, s + S, ...
template <int M, bool F32OUT>
__global__ void __launch_bounds__(kThreads) gemv_bf16_kernel(const uint16_t *__restrict__ W, int64_t ldw,
                                                             const uint16_t *__restrict__ X, int64_t ldx,
                                                             void *__restrict__ Y, int64_t ldy, int64_t n,
                                                             int64_t k, int S) {
  __shared__ float part[kWarps][kRows][M];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = kWarps / S;
  const int g = warp / S;
  const int s = warp - g * S;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * groups + g) * kRows;
  const uint64_t pol = policy_stream();
  float acc[kRows][M];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int i = 0; i < M; ++i) acc[r][i] = 0.f;
  const uint16_t *wr[kRows];
  bool live[kRows];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    live[r] = row0 + r < n;
    wr[r] = W + (live[r] ? row0 + r : 0) * ldw;
  }
  const int64_t step = static_cast<int64_t>(S) * 256;
  int64_t kb = static_cast<int64_t>(s) * 256 + lane * 8;
  // two steps per iteration: 2 * kRows weight pieces in flight per lane
  for (; kb + step < k; kb += 2 * step) {
    uint4 wa[kRows], wb[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      wa[r] = live[r] ? ld_weights(wr[r] + kb, pol) : make_uint4(0, 0, 0, 0);
      wb[r] = live[r] ? ld_weights(wr[r] + kb + step, pol) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const uint4 xa = __ldg(reinterpret_cast<const uint4 *>(X + i * ldx + kb));
      const uint4 xb = __ldg(reinterpret_cast<const uint4 *>(X + i * ldx + kb + step));
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[r][i] = dot8(wb[r], xb, dot8(wa[r], xa, acc[r][i]));
    }
  }
  if (kb < k) {
    uint4 wa[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) wa[r] = live[r] ? ld_weights(wr[r] + kb, pol) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const uint4 xa = __ldg(reinterpret_cast<const uint4 *>(X + i * ldx + kb));
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[r][i] = dot8(wa[r], xa, acc[r][i]);
    }
  }
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int i = 0; i < M; ++i) {
      float v = acc[r][i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[r][i] = v;
    }
  if (S > 1) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int i = 0; i < M; ++i) part[warp][r][i] = acc[r][i];
    }
    __syncthreads();
    if (s != 0) return;
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kRows; ++r)
#pragma unroll
        for (int i = 0; i < M; ++i) {
          float v = 0.f;
          for (int q = 0; q < S; ++q) v += part[warp + q][r][i];  // K-slice order: deterministic
          acc[r][i] = v;
        }
    }
  }
  if (lane != 0) return;
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    if (!live[r]) continue;
#pragma unroll
    for (int i = 0; i < M; ++i) {
      if (F32OUT)
        static_cast<float *>(Y)[i * ldy + row0 + r] = acc[r][i];
      else
        static_cast<uint16_t *>(Y)[i * ldy + row0 + r] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[r][i]));
    }
  }
}

template <int M>
static cudaError_t launch_m(const uint16_t *W, int64_t ldw, const uint16_t *X, int64_t ldx, void *Y, int64_t ldy,
                            int64_t n, int64_t k, int f32, int sms, cudaStream_t st) {
  // warps enough to keep ~16 per SM busy: split K when the row groups are few
  const int64_t groups = (n + kRows - 1) / kRows;
  int S = 1;
  while (S < kWarps && groups * S < static_cast<int64_t>(sms) * 16 && k >= static_cast<int64_t>(S) * 2 * 256) S *= 2;
  const int64_t per_cta = kWarps / S;
  const int64_t ctas = (groups + per_cta - 1) / per_cta;
  if (f32)
    gemv_bf16_kernel<M, true><<<static_cast<unsigned>(ctas), kThreads, 0, st>>>(W, ldw, X, ldx, Y, ldy, n, k, S);
  else
    gemv_bf16_kernel<M, false><<<static_cast<unsigned>(ctas), kThreads, 0, st>>>(W, ldw, X, ldx, Y, ldy, n, k, S);
  return cudaGetLastError();
}

}  // namespace aibgemv

AIB_API int aib_gemv_bf16(const void *w, int64_t ldw, const void *x, int64_t ldx, void *y, int64_t ldy, int64_t n,
                          int64_t k, int m, int out_fp32, void *stream) {
  using namespace aibgemv;
  if (m < 1 || m > 8) return aib_set_errorf("aib_gemv_bf16: m must be in [1, 8], got %d", m), AIB_EINVAL;
  if (n < 0 || k < 0) return aib_set_error("aib_gemv_bf16: negative size"), AIB_EINVAL;
  if (n == 0) return AIB_OK;
  if (!w || !x || !y) return aib_set_error("aib_gemv_bf16: null pointer"), AIB_EINVAL;
  if (k % 8 || ldw % 8 || ldx % 8 || ldw < k || ldx < k || ldy < n)
    return aib_set_error("aib_gemv_bf16: k, ldw and ldx must be multiples of 8, ldw/ldx >= k, ldy >= n"), AIB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15)
    return aib_set_error("aib_gemv_bf16: w and x must be 16-byte aligned"), AIB_EINVAL;
  if (reinterpret_cast<uintptr_t>(y) & (out_fp32 ? 3 : 1))
    return aib_set_error("aib_gemv_bf16: y is misaligned for its element type"), AIB_EINVAL;
  if ((n + kRows - 1) / kRows > static_cast<int64_t>(INT32_MAX))
    return aib_set_error("aib_gemv_bf16: too many rows"), AIB_EINVAL;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return aib_set_error("aib_gemv_bf16: no CUDA device"), AIB_ECUDA;
  if (k == 0) {
    const size_t bytes = out_fp32 ? 4 : 2;
    for (int i = 0; i < m; ++i)
      if (cudaMemsetAsync(static_cast<char *>(y) + i * ldy * bytes, 0, n * bytes, static_cast<cudaStream_t>(stream)) !=
          cudaSuccess)
        return aib_set_error("aib_gemv_bf16: memset failed"), AIB_ECUDA;
    return AIB_OK;
  }
  const auto *W = static_cast<const uint16_t *>(w);
  const auto *X = static_cast<const uint16_t *>(x);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (m) {
    case 1: e = launch_m<1>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    case 2: e = launch_m<2>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    case 3: e = launch_m<3>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    case 4: e = launch_m<4>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    case 5: e = launch_m<5>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    case 6: e = launch_m<6>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    case 7: e = launch_m<7>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
    default: e = launch_m<8>(W, ldw, X, ldx, y, ldy, n, k, out_fp32, sms, st); break;
  }
  if (e != cudaSuccess) return aib_set_errorf("aib_gemv_bf16: %s", cudaGetErrorString(e)), AIB_ECUDA;
  return AIB_OK;
}
