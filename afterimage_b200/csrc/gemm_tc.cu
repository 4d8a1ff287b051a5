// sm_100a tensor-core GEMM for the projections that consume a decoded layer
// when many tokens pass through it (a prompt's prefill): Y[m, n] =
// X[m, k] W[n, k]^T, BF16 operands, fp32 accumulation in tensor memory. It
// replaces, for these shapes, the nn.Linear / F.linear the reference calls on
// the decoded weights (afterimage/runtime/streaming_engine.py:1871-1915).
//
// With m up to a few hundred tokens the product streams W once and is bound
// by HBM, so the tile is laid out "weights as rows": a CTA owns 128 rows of W
// (the tcgen05.mma M dimension) and all the tokens (the N dimension, up to
// 256, rounded up to 16), and when the row tiles are too few to fill the SMs
// it takes one of `ksplit` K ranges (fp32 partials in a caller workspace,
// summed in K order by a second kernel).
//
// Per CTA (192 threads):
//   warp 4     TMA producer: 128-byte-swizzled tiles of W [128 x 64] and
//              X [tn x 64] into a 4-stage shared-memory ring (one
//              cp.async.bulk.tensor each, mbarrier completion, no multicast);
//   warp 5     owns the tensor-memory accumulator (tcgen05.alloc of tn
//              columns) and issues four tcgen05.mma (K = 16 each) per stage
//              from one thread; tcgen05.commit frees the stage when they
//              complete, and signals the epilogue after the last one;
//   warps 0-3  epilogue: tcgen05.ld of their 32 accumulator lanes (= W rows),
//              16 columns (= tokens) at a time, rounded to BF16 (or kept fp32
//              for a K split) and stored, 32 consecutive outputs per token.
// Every mbarrier wait is bounded; a wait that gives up sets
// AIB_STATUS_WAIT_TIMEOUT and the CTA unwinds (it still frees its tensor
// memory), so a broken launch reports an error instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "aib_internal.h"

namespace aibtc {

constexpr int kBM = 128;  // W rows per CTA (UMMA M)
constexpr int kBK = 64;   // K per stage: one 128-byte swizzle atom of BF16
constexpr int kStages = 4;  // 4 stages: two CTAs of up to 64 tokens fit an SM (better than 8 stages in one)
constexpr int kThreads = 192;
constexpr int kMaxTN = 256;
constexpr int kWTileBytes = kBM * kBK * 2;  // 16 KiB
constexpr unsigned kWaitLimit = AIB_WAIT_LIMIT_POLLS;

__host__ __device__ constexpr int stage_bytes(int tn) { return kWTileBytes + tn * kBK * 2; }
__host__ __device__ constexpr int smem_bytes(int tn) { return kStages * stage_bytes(tn) + 1024; }

struct Params {
  int64_t m, n, k;
  int tn;            // token tile (UMMA N): multiple of 16 in [16, 256]
  int ksplit;        // K ranges (gridDim.y)
  int64_t kchunk;    // K per range, a multiple of kBK
  uint16_t *y;       // bf16 [m, ldy] (ksplit == 1)
  int64_t ldy;
  float *ws;         // fp32 [ksplit, m, n] (ksplit > 1)
  int32_t *status;
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// true when the phase of `parity` completed within the bound
__device__ __forceinline__ bool mbar_wait(uint32_t bar, unsigned parity) {
  for (unsigned spins = 0; spins < kWaitLimit; ++spins) {
    if (mbar_try_wait(bar, parity)) return true;
    if (spins > 64) __nanosleep(32);
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// shared-memory matrix descriptor: K-major tile of 128-byte rows, 128-byte
// swizzle, 8-row groups 1024 bytes apart (leading offset unused: 1)
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}

// instruction descriptor: BF16 x BF16 -> F32, both K-major, M = 128, N = tn
__device__ __forceinline__ uint32_t instr_desc(int tn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(tn >> 3) << 17) | ((kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t tmem_columns(int tn) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(tn)) c <<= 1;
  return c;
}

__global__ void __launch_bounds__(kThreads, 1) gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap map_w,
                                                                   const __grid_constant__ CUtensorMap map_x,
                                                                   const Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kStages];
  __shared__ __align__(8) uint64_t empty_bar[kStages];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int gave_up;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t ring = (smem_u32(smem_raw) + 1023u) & ~1023u;  // 128-byte swizzle wants 1024-byte alignment
  const int sbytes = stage_bytes(p.tn);
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kBM;
  const int64_t kbeg = static_cast<int64_t>(blockIdx.y) * p.kchunk;
  const int nk = static_cast<int>(min(p.kchunk, p.k - kbeg) / kBK);
  const uint32_t ncols = tmem_columns(p.tn);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(&done_bar), 1);
    gave_up = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 4) {
    // ---- TMA producer
    if (lane == 0) {
      const uint32_t tx = static_cast<uint32_t>(sbytes);
      int issued = 0;
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        const unsigned ph = static_cast<unsigned>(it / kStages) & 1u;
        if (!mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u)) {
          atomicOr(&gave_up, 1);
          break;
        }
        const uint32_t fb = smem_u32(&full_bar[s]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"(tx) : "memory");
        const uint32_t st = ring + static_cast<uint32_t>(s * sbytes);
        const int kx = static_cast<int>(kbeg + static_cast<int64_t>(it) * kBK);
        tma_load_2d(st, &map_w, kx, static_cast<int>(row0), fb);
        tma_load_2d(st + kWTileBytes, &map_x, kx, 0, fb);
        issued = it + 1;
      }
      // copies still in flight land before the CTA can exit (bounded)
      for (int it = max(0, issued - kStages); it < issued; ++it)
        (void)mbar_wait(smem_u32(&full_bar[it % kStages]), static_cast<unsigned>(it / kStages) & 1u);
    }
  } else if (warp == 5) {
    // ---- MMA issuer (one thread)
    if (lane == 0) {
      const uint32_t idesc = instr_desc(p.tn);
      for (int it = 0; it < nk; ++it) {
        const int s = it % kStages;
        const unsigned ph = static_cast<unsigned>(it / kStages) & 1u;
        if (!mbar_wait(smem_u32(&full_bar[s]), ph)) {
          atomicOr(&gave_up, 1);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t st = ring + static_cast<uint32_t>(s * sbytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // advancing K by 16 elements inside the swizzle atom moves the start by 32 bytes
          mma_bf16(tmem, smem_desc(st + kk * 32), smem_desc(st + kWTileBytes + kk * 32), idesc,
                   (it > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(smem_u32(&empty_bar[s]));
      }
      // the epilogue waits on this: it arrives once every MMA issued above has completed
      mma_commit(smem_u32(&done_bar));
    }
  } else {
    // ---- epilogue: warps 0-3, TMEM lanes 32w .. 32w + 31 = W rows
    bool ok = mbar_wait(smem_u32(&done_bar), 0);
    if (!ok) atomicOr(&gave_up, 1);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const bool live = ok && !gave_up && nk > 0;
    const int64_t row = row0 + warp * 32 + lane;
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    for (int c0 = 0; c0 < p.tn; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(taddr + static_cast<uint32_t>(c0), v);  // collective: every lane of the warp
      if (!live || row >= p.n) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t tok = c0 + j;
        if (tok >= p.m) break;
        const float f = __uint_as_float(v[j]);
        if (p.ksplit > 1)
          p.ws[(static_cast<int64_t>(blockIdx.y) * p.m + tok) * p.n + row] = f;
        else
          p.y[tok * p.ldy + row] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (threadIdx.x == 0 && gave_up && p.status) atomicOr(p.status, AIB_STATUS_WAIT_TIMEOUT);
  if (warp == 5) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// y[i, j] = bf16(sum over s of ws[s, i, j]), s ascending
__global__ void ksplit_sum_kernel(const float *__restrict__ ws, int ksplit, int64_t m, int64_t n,
                                  uint16_t *__restrict__ y, int64_t ldy) {
  const int64_t total = m * n;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += stride) {
    float a = 0.f;
    for (int s = 0; s < ksplit; ++s) a += ws[s * total + t];
    const int64_t i = t / n, j = t - i * n;
    y[i * ldy + j] = __bfloat16_as_ushort(__float2bfloat16_rn(a));
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// 2-D BF16 tensor [rows, cols] with row stride ld (elements): box [box_rows, 64], 128-byte swizzle,
// zero fill outside
static bool make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Plan {
  int tn, ksplit;
  int64_t kchunk, tiles;
};

static Plan plan(int64_t m, int64_t n, int64_t k, int sms) {
  Plan pl;
  pl.tn = static_cast<int>((m + 15) / 16 * 16);
  pl.tiles = (n + kBM - 1) / kBM;
  const int64_t ksteps = k / kBK;
  int s = 1;
  // split K until the CTAs cover the SMs, keeping a full ring of work per range
  while (pl.tiles * s < sms && ksteps % (2 * s) == 0 && ksteps / (2 * s) >= kStages && s < 16) s *= 2;
  pl.ksplit = s;
  pl.kchunk = ksteps / s * kBK;
  return pl;
}

}  // namespace aibtc

AIB_API int64_t aib_gemm_bf16_tc_workspace_floats(int64_t m, int64_t n, int64_t k) {
  using namespace aibtc;
  if (m < 1 || n < 1 || k < kBK || k % kBK) return 0;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const Plan pl = plan(m, n, k, sms);
  return pl.ksplit > 1 ? static_cast<int64_t>(pl.ksplit) * m * n : 0;
}

AIB_API int aib_gemm_bf16_tc(const void *w, int64_t ldw, const void *x, int64_t ldx, void *y, int64_t ldy,
                             int64_t m, int64_t n, int64_t k, float *workspace, int64_t workspace_floats,
                             int32_t *d_status, void *stream) {
  using namespace aibtc;
  if (m < 1 || m > kMaxTN) return aib_set_errorf("aib_gemm_bf16_tc: m must be in [1, %d], got %lld", kMaxTN,
                                                 (long long)m), AIB_EINVAL;
  if (n < 1 || k < kBK || k % kBK)
    return aib_set_errorf("aib_gemm_bf16_tc: n >= 1 and k a positive multiple of %d needed (n %lld, k %lld)", kBK,
                          (long long)n, (long long)k), AIB_EINVAL;
  if (!w || !x || !y) return aib_set_error("aib_gemm_bf16_tc: null pointer"), AIB_EINVAL;
  if (((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) || ldw % 8 || ldx % 8 || ldw < k ||
      ldx < k || ldy < n || (reinterpret_cast<uintptr_t>(y) & 1))
    return aib_set_error("aib_gemm_bf16_tc: w and x 16-byte aligned with row strides a multiple of 8 and >= k; "
                         "ldy >= n"), AIB_EINVAL;
  if (n > INT32_MAX || k > INT32_MAX) return aib_set_error("aib_gemm_bf16_tc: n and k must fit in 32 bits"), AIB_EINVAL;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return aib_set_error("aib_gemm_bf16_tc: no CUDA device"), AIB_ECUDA;
  const Plan pl = plan(m, n, k, sms);
  if (pl.ksplit > 1 && (!workspace || workspace_floats < static_cast<int64_t>(pl.ksplit) * m * n))
    return aib_set_errorf("aib_gemm_bf16_tc: needs a workspace of %lld floats",
                          (long long)(static_cast<int64_t>(pl.ksplit) * m * n)), AIB_EINVAL;
  CUtensorMap mw, mx;
  if (!make_map(&mw, w, n, k, ldw, kBM) || !make_map(&mx, x, m, k, ldx, pl.tn))
    return aib_set_error("aib_gemm_bf16_tc: cuTensorMapEncodeTiled failed"), AIB_ECUDA;
  static std::once_flag attr;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr, [] {
    attr_err = cudaFuncSetAttribute(gemm_bf16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    smem_bytes(kMaxTN));
  });
  if (attr_err != cudaSuccess) return aib_set_errorf("aib_gemm_bf16_tc: %s", cudaGetErrorString(attr_err)), AIB_ECUDA;
  Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tn = pl.tn;
  p.ksplit = pl.ksplit;
  p.kchunk = pl.kchunk;
  p.y = static_cast<uint16_t *>(y);
  p.ldy = ldy;
  p.ws = workspace;
  p.status = d_status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(pl.tiles), static_cast<unsigned>(pl.ksplit));
  gemm_bf16_tc_kernel<<<grid, kThreads, smem_bytes(pl.tn), st>>>(mw, mx, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return aib_set_errorf("aib_gemm_bf16_tc: %s", cudaGetErrorString(e)), AIB_ECUDA;
  if (pl.ksplit > 1) {
    const int64_t blocks = std::min<int64_t>((m * n + 255) / 256, static_cast<int64_t>(sms) * 8);
    ksplit_sum_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(workspace, pl.ksplit, m, n,
                                                                      static_cast<uint16_t *>(y), ldy);
    e = cudaGetLastError();
    if (e != cudaSuccess) return aib_set_errorf("aib_gemm_bf16_tc: %s", cudaGetErrorString(e)), AIB_ECUDA;
  }
  return AIB_OK;
}
