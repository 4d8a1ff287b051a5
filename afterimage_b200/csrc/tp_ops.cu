// sm_100a kernels for the single-token step of the tensor-parallel decoder
// (afterimage_b200/runtime/tp_decoder.py): the small per-layer operations
// between the projections, fused so that a layer is ~10 launches instead of
// ~60 (residual add + RMSNorm, q/k RMSNorm + rotary embedding + KV-cache
// write, grouped-query attention over the cache, SiLU * up).
//
// The reference runs this layer math in transformers' Qwen3 / Llama
// modules (its engine hooks them, afterimage/runtime/streaming_engine.py:
// 1871-1915); the roundings below follow those modules' BF16 arithmetic:
// every elementwise op computes in fp32 and rounds its result to BF16, the
// norms reduce in fp32.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "aib_internal.h"

namespace aibtp {

__device__ __forceinline__ float b2f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }
__device__ __forceinline__ uint16_t f2b(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ float rb(float f) { return b2f(f2b(f)); }  // round to BF16, back to fp32

// block-wide sum of one float per thread (blockDim.x a multiple of 32, <= 1024)
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < nw ? red[l] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = l < nw ? red[l] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

// x <- bf16(x + delta) (when delta), out = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))
// one block per row
__global__ void add_rmsnorm_kernel(uint16_t *__restrict__ x, const uint16_t *__restrict__ delta,
                                   const uint16_t *__restrict__ w, uint16_t *__restrict__ out, int64_t cols,
                                   float eps) {
  __shared__ float red[32];
  uint16_t *xr = x + blockIdx.x * cols;
  const uint16_t *dr = delta ? delta + blockIdx.x * cols : nullptr;
  uint16_t *orow = out + blockIdx.x * cols;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
    float v = b2f(xr[i]);
    if (dr) {
      v = rb(v + b2f(dr[i]));
      xr[i] = f2b(v);
    }
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, red) / static_cast<float>(cols) + eps);
  for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) orow[i] = f2b(b2f(w[i]) * rb(b2f(xr[i]) * r));
}

// One block of hd threads per (token, head). qkv: [T, (nh + 2 nkv) * hd]
// (q heads, then k heads, then v heads). q heads: optional RMSNorm over hd,
// rotary embedding at position pos0 + t -> q_out [nh, T, hd]. k heads: the
// same, written to k_cache[kvh, pos0 + t, :]. v heads: copied to
// v_cache[kvh, pos0 + t, :]. Rotary: the rotate-half form with
// cos/sin = bf16(cos/sin(pos * inv_freq[d mod hd/2])).
__global__ void qk_rope_cache_kernel(const uint16_t *__restrict__ qkv, int T, int nh, int nkv, int hd,
                                     const uint16_t *__restrict__ qn_w, const uint16_t *__restrict__ kn_w, float eps,
                                     const float *__restrict__ inv_freq, const int64_t *__restrict__ pos0,
                                     uint16_t *__restrict__ q_out, uint16_t *__restrict__ k_cache,
                                     uint16_t *__restrict__ v_cache, int64_t max_len) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const int head = blockIdx.y;
  const int d = threadIdx.x;
  const int64_t width = static_cast<int64_t>(nh + 2 * nkv) * hd;
  const uint16_t *row = qkv + t * width + static_cast<int64_t>(head) * hd;
  const int64_t pos = *pos0 + t;
  const bool in_cache = pos >= 0 && pos < max_len;  // positions outside the cache are not written
  if (head >= nh + nkv) {  // v head: plain copy into the cache
    const int kvh = head - nh - nkv;
    if (d < hd && in_cache) v_cache[(static_cast<int64_t>(kvh) * max_len + pos) * hd + d] = row[d];
    return;
  }
  const bool is_q = head < nh;
  const uint16_t *nw = is_q ? qn_w : kn_w;
  const int half = hd / 2;
  const float xv = d < hd ? b2f(row[d]) : 0.f;
  float r = 1.f;
  if (nw) r = rsqrtf(block_sum(xv * xv, red) / static_cast<float>(hd) + eps);
  if (d >= hd) return;
  const int p = d < half ? d + half : d - half;
  const float xp = b2f(row[p]);
  const float n_d = nw ? rb(b2f(nw[d]) * rb(xv * r)) : xv;
  const float n_p = nw ? rb(b2f(nw[p]) * rb(xp * r)) : xp;
  const float rot = d < half ? -n_p : n_p;
  const float ang = static_cast<float>(pos) * inv_freq[d % half];
  const float c = rb(cosf(ang)), s = rb(sinf(ang));
  const uint16_t o = f2b(rb(n_d * c) + rb(rot * s));
  if (is_q)
    q_out[(static_cast<int64_t>(head) * T + t) * hd + d] = o;
  else if (in_cache)
    k_cache[(static_cast<int64_t>(head - nh) * max_len + pos) * hd + d] = o;
}

// Single-query attention over cache positions [0, *pos], one block per query
// head; kv head = head / (nh / nkv). scores in fp32, softmax in fp32, output
// rounded to BF16: out[head * hd + d].
__global__ void decode_attention_kernel(const uint16_t *__restrict__ q, const uint16_t *__restrict__ k_cache,
                                        const uint16_t *__restrict__ v_cache, int nh, int nkv, int hd,
                                        int64_t max_len, const int64_t *__restrict__ pos, float scale,
                                        uint16_t *__restrict__ out) {
  extern __shared__ float sc[];
  __shared__ float red[32];
  const int h = blockIdx.x;
  const int kvh = h / (nh / nkv);
  const int64_t L = min(*pos + 1, max_len);
  if (L < 1) {
    for (int d = threadIdx.x; d < hd; d += blockDim.x) out[static_cast<int64_t>(h) * hd + d] = 0;
    return;
  }
  const uint16_t *qh = q + static_cast<int64_t>(h) * hd;
  const uint16_t *kb = k_cache + static_cast<int64_t>(kvh) * max_len * hd;
  const uint16_t *vb = v_cache + static_cast<int64_t>(kvh) * max_len * hd;
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int64_t j = w; j < L; j += nw) {
    float acc = 0.f;
    for (int d = l; d < hd; d += 32) acc += b2f(qh[d]) * b2f(kb[j * hd + d]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (l == 0) sc[j] = acc * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < L; j += blockDim.x) m = fmaxf(m, sc[j]);
  m = block_max(m, red);
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
    const float e = expf(sc[j] - m);
    sc[j] = e;
    s += e;
  }
  s = block_sum(s, red);  // (its barriers also order the writes to sc above)
  const float inv = 1.f / s;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.f;
    for (int64_t j = 0; j < L; ++j) acc += sc[j] * b2f(vb[j * hd + d]);
    out[static_cast<int64_t>(h) * hd + d] = f2b(acc * inv);
  }
}

// out[t, i] = bf16(bf16(silu(g)) * u), g = gu[t, i], u = gu[t, I + i]
__global__ void silu_mul_kernel(const uint16_t *__restrict__ gu, uint16_t *__restrict__ out, int64_t T, int64_t I) {
  const int64_t n = T * I;
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = k / I, i = k - t * I;
    const float g = b2f(gu[t * 2 * I + i]);
    const float u = b2f(gu[t * 2 * I + I + i]);
    const float sg = rb(g / (1.f + expf(-g)));
    out[k] = f2b(sg * u);
  }
}

constexpr int kMaxAttnLen = 8192;  // cache positions one attention block holds in shared memory

}  // namespace aibtp

using namespace aibtp;

#define TP_CUDA(call)                                                         \
  do {                                                                        \
    cudaError_t e_ = (call);                                                  \
    if (e_ != cudaSuccess) {                                                  \
      aib_set_errorf("%s: %s (%s)", __func__, cudaGetErrorString(e_), #call); \
      return AIB_ECUDA;                                                       \
    }                                                                         \
  } while (0)

AIB_API int aib_add_rmsnorm_bf16(void *x, const void *delta, const void *weight, void *out, int64_t rows,
                                 int64_t cols, float eps, void *stream) {
  if (rows < 0 || cols < 1) return aib_set_error("add_rmsnorm: bad shape"), AIB_EINVAL;
  if (!x || !weight || !out) return aib_set_error("add_rmsnorm: null pointer"), AIB_EINVAL;
  if (rows == 0) return AIB_OK;
  if (rows > 65535 * 1024LL) return aib_set_error("add_rmsnorm: too many rows"), AIB_EINVAL;
  add_rmsnorm_kernel<<<static_cast<unsigned>(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint16_t *>(x), static_cast<const uint16_t *>(delta), static_cast<const uint16_t *>(weight),
      static_cast<uint16_t *>(out), cols, eps);
  TP_CUDA(cudaGetLastError());
  return AIB_OK;
}

AIB_API int aib_qk_rope_cache_bf16(const void *qkv, int T, int nh, int nkv, int hd, const void *q_norm_w,
                                   const void *k_norm_w, float eps, const float *inv_freq, const int64_t *pos0,
                                   void *q_out, void *k_cache, void *v_cache, int64_t max_len, void *stream) {
  if (T < 0 || nh < 1 || nkv < 1 || hd < 2 || hd % 2 || hd > 1024 || max_len < 1)
    return aib_set_error("qk_rope_cache: bad shape"), AIB_EINVAL;
  if (!qkv || !inv_freq || !pos0 || !q_out || !k_cache || !v_cache)
    return aib_set_error("qk_rope_cache: null pointer"), AIB_EINVAL;
  if ((q_norm_w == nullptr) != (k_norm_w == nullptr))
    return aib_set_error("qk_rope_cache: give both q and k norm weights or neither"), AIB_EINVAL;
  if (T == 0) return AIB_OK;
  const dim3 grid(static_cast<unsigned>(T), static_cast<unsigned>(nh + 2 * nkv));
  const int threads = (hd + 31) / 32 * 32;
  qk_rope_cache_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(qkv), T, nh, nkv, hd, static_cast<const uint16_t *>(q_norm_w),
      static_cast<const uint16_t *>(k_norm_w), eps, inv_freq, pos0, static_cast<uint16_t *>(q_out),
      static_cast<uint16_t *>(k_cache), static_cast<uint16_t *>(v_cache), max_len);
  TP_CUDA(cudaGetLastError());
  return AIB_OK;
}

AIB_API int aib_decode_attention_bf16(const void *q, const void *k_cache, const void *v_cache, int nh, int nkv,
                                      int hd, int64_t max_len, const int64_t *pos, float scale, void *out,
                                      void *stream) {
  if (nh < 1 || nkv < 1 || nh % nkv || hd < 1 || max_len < 1)
    return aib_set_error("decode_attention: bad shape"), AIB_EINVAL;
  if (max_len > kMaxAttnLen)
    return aib_set_errorf("decode_attention: cache length %lld exceeds %d", (long long)max_len, kMaxAttnLen),
           AIB_EINVAL;
  if (!q || !k_cache || !v_cache || !pos || !out) return aib_set_error("decode_attention: null pointer"), AIB_EINVAL;
  decode_attention_kernel<<<static_cast<unsigned>(nh), 128, static_cast<size_t>(max_len) * sizeof(float),
                            static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t *>(q), static_cast<const uint16_t *>(k_cache),
      static_cast<const uint16_t *>(v_cache), nh, nkv, hd, max_len, pos, scale, static_cast<uint16_t *>(out));
  TP_CUDA(cudaGetLastError());
  return AIB_OK;
}

AIB_API int aib_silu_mul_bf16(const void *gate_up, void *out, int64_t T, int64_t I, void *stream) {
  if (T < 0 || I < 1) return aib_set_error("silu_mul: bad shape"), AIB_EINVAL;
  if (!gate_up || !out) return aib_set_error("silu_mul: null pointer"), AIB_EINVAL;
  if (T == 0) return AIB_OK;
  const int64_t n = T * I;
  const int blocks = static_cast<int>(n / 256 + 1 < 4096 ? n / 256 + 1 : 4096);
  silu_mul_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint16_t *>(gate_up),
                                                                       static_cast<uint16_t *>(out), T, I);
  TP_CUDA(cudaGetLastError());
  return AIB_OK;
}
