// One-shot all-reduce of fp32 vectors over NVLink peer memory, for the
// row-parallel projections of the tensor-parallel decoder (o_proj and
// down_proj partial sums; the reference runs single-GPU and has no
// counterpart, its layers call nn.Linear on whole weights,
// afterimage/runtime/streaming_engine.py:1871-1915).
//
// Every rank owns one buffer (cudaMalloc, shared with the other ranks of
// the node through CUDA IPC handles):
//   [0, 8)           the call counter (epoch) and a count of finished CTAs
//                    (local use only)
//   [4 KiB, 8 KiB)   flags[src_rank][cta] (int32), written by the peers
//   [8 KiB, ...)     data[2][max_floats] (fp32), two parities
// Call e on every rank (the same calls in the same order on every rank),
// CTA b of G (G fixed by n, so the same on every rank):
//   1. copy the rank's slice b of `in` into its own data[e & 1];
//   2. fence (system scope), then store e into flags[rank][b] of every rank;
//   3. wait, bounded, until its own flags[p][b] >= e for every rank p;
//   4. out[slice b] = sum over p = 0 .. world-1, in that order, of slice b
//      of data[e & 1] of rank p (NVLink loads): the same order on every
//      rank, so all ranks hold bit-identical sums;
//   5. the last CTA to finish advances the epoch to e.
// A rank writes data[e & 1] again only in call e + 2. Before that, its call
// e + 1 saw a flag of call e + 1 from every peer; a peer's call e + 1 starts
// after its whole call e (stream order), reads included. So two parities
// suffice, with no second barrier, whatever G each call uses.
// A wait that gives up sets AIB_STATUS_PEER_TIMEOUT in the status word and
// the CTA returns without touching `out` (the group is then unusable; the
// host raises and tears it down). No load here uses TMA or cluster
// multicast; peers are read with plain vector loads that bypass L1.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "aib_internal.h"

namespace aibar {

constexpr int kThreads = 256;
constexpr int kMaxCtas = AIB_AR_MAX_CTAS;
constexpr int64_t kCounterOff = 0;
constexpr int64_t kFlagOff = 4096;
constexpr int64_t kDataOff = 8192;
static_assert(AIB_AR_MAX_RANKS * kMaxCtas * 4 <= 4096, "flag block size");

struct Args {
  float *data[AIB_AR_MAX_RANKS];     // each rank's data[0] as mapped here
  int32_t *flags[AIB_AR_MAX_RANKS];  // each rank's flag block as mapped here
  int32_t *counters;                 // this rank's {epoch, finished CTAs}
  int64_t max_floats;
  int32_t rank, world;
};

__device__ __forceinline__ void st_release_sys(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t *p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) oneshot_kernel(const Args a, const float *in, float *out, int64_t n,
                                                           int vec, unsigned max_polls, int32_t *status) {
  __shared__ int32_t s_ep;
  __shared__ int s_fail;
  const int b = blockIdx.x;
  const int64_t per = ((n + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  const int64_t lo = min(n, per * b);
  const int64_t hi = min(n, lo + per);
  if (threadIdx.x == 0) {
    s_ep = a.counters[0] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const int32_t ep = s_ep;
  const int64_t par = static_cast<int64_t>(ep & 1) * a.max_floats;
  float *mine = a.data[a.rank] + par;

  // 1. this rank's slice into its own buffer
  if (vec) {
    for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * kThreads)
      *reinterpret_cast<float4 *>(mine + i) = *reinterpret_cast<const float4 *>(in + i);
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) mine[i] = in[i];
  }
  __threadfence_system();
  __syncthreads();

  // 2. announce call ep to every rank (itself included), 3. wait for theirs
  if (threadIdx.x < a.world) {
    const int p = threadIdx.x;
    st_release_sys(a.flags[p] + a.rank * kMaxCtas + b, ep);
    const int32_t *f = a.flags[a.rank] + p * kMaxCtas + b;
    unsigned polls = 0;
    while (ld_acquire_sys(f) - ep < 0) {
      if (++polls > max_polls) {
        atomicOr(&s_fail, 1);
        break;
      }
      if (polls > 2048) __nanosleep(128);
    }
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0 && status) atomicOr(status, AIB_STATUS_PEER_TIMEOUT);
    return;
  }
  __threadfence_system();

  // 4. the sum in rank order
  if (vec) {
    for (int64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * kThreads) {
      float4 s = __ldcv(reinterpret_cast<const float4 *>(a.data[0] + par + i));
      for (int p = 1; p < a.world; ++p) {
        const float4 v = __ldcv(reinterpret_cast<const float4 *>(a.data[p] + par + i));
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
      *reinterpret_cast<float4 *>(out + i) = s;
    }
  } else {
    for (int64_t i = lo + threadIdx.x; i < hi; i += kThreads) {
      float s = __ldcv(a.data[0] + par + i);
      for (int p = 1; p < a.world; ++p) s += __ldcv(a.data[p] + par + i);
      out[i] = s;
    }
  }
  // 5. the last CTA of the call advances the epoch (read by the next call
  // on this stream, which starts after every CTA of this one)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.counters + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      a.counters[1] = 0;
      a.counters[0] = ep;
    }
  }
}

}  // namespace aibar

using namespace aibar;

AIB_API size_t aib_ar_buffer_bytes(int64_t max_floats) {
  if (max_floats < 0) return 0;
  return static_cast<size_t>(kDataOff + 2 * 4 * ((max_floats + 3) / 4 * 4));
}

AIB_API int aib_ar_alloc(int64_t max_floats, void **d_buffer) {
  if (!d_buffer || max_floats < 1) return aib_set_error("aib_ar_alloc: bad arguments"), AIB_EINVAL;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, aib_ar_buffer_bytes(max_floats));
  if (e == cudaSuccess) e = cudaMemset(p, 0, kDataOff);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return aib_set_errorf("aib_ar_alloc: %s", cudaGetErrorString(e)), AIB_ECUDA;
  }
  *d_buffer = p;
  return AIB_OK;
}

AIB_API int aib_ar_free(void *d_buffer) {
  if (!d_buffer) return AIB_OK;
  const cudaError_t e = cudaFree(d_buffer);
  if (e != cudaSuccess) return aib_set_errorf("aib_ar_free: %s", cudaGetErrorString(e)), AIB_ECUDA;
  return AIB_OK;
}

AIB_API int aib_ar_ipc_handle(void *d_buffer, void *handle_out) {
  if (!d_buffer || !handle_out) return aib_set_error("aib_ar_ipc_handle: null pointer"), AIB_EINVAL;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, d_buffer);
  if (e != cudaSuccess) return aib_set_errorf("aib_ar_ipc_handle: %s", cudaGetErrorString(e)), AIB_ECUDA;
  static_assert(sizeof(h) == AIB_AR_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return AIB_OK;
}

AIB_API int aib_ar_ipc_open(const void *handle, void **d_peer) {
  if (!handle || !d_peer) return aib_set_error("aib_ar_ipc_open: null pointer"), AIB_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return aib_set_errorf("aib_ar_ipc_open: %s", cudaGetErrorString(e)), AIB_ECUDA;
  *d_peer = p;
  return AIB_OK;
}

AIB_API int aib_ar_ipc_close(void *d_peer) {
  if (!d_peer) return AIB_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(d_peer);
  if (e != cudaSuccess) return aib_set_errorf("aib_ar_ipc_close: %s", cudaGetErrorString(e)), AIB_ECUDA;
  return AIB_OK;
}

AIB_API int aib_ar_ctas(int64_t n) {
  if (n <= 0) return 0;
  return static_cast<int>(std::min<int64_t>(kMaxCtas, std::max<int64_t>(1, (n + 4095) / 4096)));
}

AIB_API int aib_allreduce_oneshot_f32(const aib_ar_group *g, const float *in, float *out, int64_t n,
                                      unsigned max_polls, int32_t *d_status, void *stream) {
  if (!g) return aib_set_error("aib_allreduce_oneshot_f32: null group"), AIB_EINVAL;
  if (g->world < 1 || g->world > AIB_AR_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
    return aib_set_errorf("aib_allreduce_oneshot_f32: rank %d / world %d out of range [1, %d]", g->rank, g->world,
                          AIB_AR_MAX_RANKS),
           AIB_EINVAL;
  if (n < 0 || n > g->max_floats)
    return aib_set_errorf("aib_allreduce_oneshot_f32: n %lld not in [0, max_floats %lld]", (long long)n,
                          (long long)g->max_floats),
           AIB_EINVAL;
  if (max_polls < 1) return aib_set_error("aib_allreduce_oneshot_f32: max_polls must be >= 1"), AIB_EINVAL;
  if (n == 0) return AIB_OK;
  if (!in || !out) return aib_set_error("aib_allreduce_oneshot_f32: null in or out"), AIB_EINVAL;
  Args a;
  std::memset(&a, 0, sizeof(a));
  for (int p = 0; p < g->world; ++p) {
    if (!g->buffers[p] || reinterpret_cast<uintptr_t>(g->buffers[p]) % 256)
      return aib_set_errorf("aib_allreduce_oneshot_f32: buffer of rank %d is null or not 256-byte aligned", p),
             AIB_EINVAL;
    unsigned char *base = static_cast<unsigned char *>(g->buffers[p]);
    a.data[p] = reinterpret_cast<float *>(base + kDataOff);
    a.flags[p] = reinterpret_cast<int32_t *>(base + kFlagOff);
  }
  a.counters = reinterpret_cast<int32_t *>(static_cast<unsigned char *>(g->buffers[g->rank]) + kCounterOff);
  a.max_floats = (g->max_floats + 3) / 4 * 4;
  a.rank = g->rank;
  a.world = g->world;
  const int vec =
      n % 4 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0;
  oneshot_kernel<<<aib_ar_ctas(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, in, out, n, vec, max_polls,
                                                                                      d_status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return aib_set_errorf("aib_allreduce_oneshot_f32: %s", cudaGetErrorString(e)), AIB_ECUDA;
  return AIB_OK;
}
