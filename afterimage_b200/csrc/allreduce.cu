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
//   [4 KiB, ...)     recv[2][AIB_AR_MAX_RANKS][max_floats] of 64-bit words,
//                    two parities, written by the peers
// Call e on every rank (the same calls in the same order on every rank):
// element i of this rank's input goes to every peer as ONE 64-bit store of
// (value bits, e) into the peer's recv[e & 1][rank][i]. A receiver polls its
// own recv[e & 1][p][i] until the word carries e, and then holds the value:
// a single-copy-atomic 64-bit store cannot be seen half written, so no
// fence and no separate flag are needed and a value costs one one-way
// NVLink write. out[i] is the sum over p = 0 .. world-1, in that order (the
// rank's own value from `in`), so every rank holds bit-identical sums.
// A rank writes recv[e & 1][rank] of a peer again only in call e + 2. Its
// call e + 1 waited for that peer's words of call e + 1, which the peer
// wrote after its whole call e (stream order), reads included. So two
// parities suffice with no second barrier. The last CTA of a call advances
// the epoch, so the kernel runs unchanged inside a CUDA graph.
// A wait that gives up sets AIB_STATUS_PEER_TIMEOUT in the status word (the
// group is then unusable; the host raises and tears it down). No load here
// uses TMA or cluster multicast; peers are only written, with plain stores.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "aib_internal.h"

namespace aibar {

constexpr int kThreads = 256;
constexpr int kMaxCtas = AIB_AR_MAX_CTAS;
constexpr int64_t kCounterOff = 0;
constexpr int64_t kRecvOff = 4096;

struct Args {
  uint64_t *recv[AIB_AR_MAX_RANKS];  // each rank's recv[0][0] as mapped here
  int32_t *counters;                 // this rank's {epoch, finished CTAs}
  int64_t max_floats;                // words per (parity, source) row
  int32_t rank, world;
};

__device__ __forceinline__ void st_relaxed_sys(uint64_t *p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kThreads) oneshot_kernel(const Args a, const float *in, float *out, int64_t n,
                                                           unsigned max_polls, int32_t *status) {
  __shared__ int32_t s_ep;
  __shared__ int s_fail;
  if (threadIdx.x == 0) {
    s_ep = a.counters[0] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t ep = static_cast<uint32_t>(s_ep);
  const int64_t row = a.max_floats;
  const int64_t par = static_cast<int64_t>(ep & 1u) * AIB_AR_MAX_RANKS * row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;

  // 1. every element to every peer: (value bits, epoch) in one 64-bit store
  for (int64_t i = first; i < n; i += stride) {
    const uint64_t w = static_cast<uint64_t>(__float_as_uint(in[i])) | (static_cast<uint64_t>(ep) << 32);
    for (int p = 0; p < a.world; ++p)
      if (p != a.rank) st_relaxed_sys(a.recv[p] + par + a.rank * row + i, w);
  }

  // 2. wait for each peer's word of each element, sum in rank order
  const uint64_t *mine = a.recv[a.rank] + par;
  bool fail = false;
  for (int64_t i = first; i < n && !fail; i += stride) {
    float s = 0.f;
    for (int p = 0; p < a.world; ++p) {
      float x;
      if (p == a.rank) {
        x = in[i];
      } else {
        const uint64_t *q = mine + p * row + i;
        uint64_t w = ld_relaxed_sys(q);
        unsigned polls = 0;
        while (static_cast<uint32_t>(w >> 32) != ep) {
          if (++polls > max_polls) {
            fail = true;
            break;
          }
          if (polls > 4096) __nanosleep(64);
          w = ld_relaxed_sys(q);
        }
        if (fail) break;
        x = __uint_as_float(static_cast<uint32_t>(w));
      }
      s = p == 0 ? x : s + x;
    }
    if (!fail) out[i] = s;
  }
  if (fail) atomicOr(&s_fail, 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (s_fail && status) atomicOr(status, AIB_STATUS_PEER_TIMEOUT);
    // 3. the last CTA of the call advances the epoch (read by the next call
    // on this stream, which starts after every CTA of this one)
    __threadfence();
    if (atomicAdd(a.counters + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      a.counters[1] = 0;
      a.counters[0] = static_cast<int32_t>(ep);
    }
  }
}

}  // namespace aibar

using namespace aibar;

AIB_API size_t aib_ar_buffer_bytes(int64_t max_floats) {
  if (max_floats < 0) return 0;
  return static_cast<size_t>(kRecvOff + 2 * AIB_AR_MAX_RANKS * 8 * max_floats);
}

AIB_API int aib_ar_alloc(int64_t max_floats, void **d_buffer) {
  if (!d_buffer || max_floats < 1) return aib_set_error("aib_ar_alloc: bad arguments"), AIB_EINVAL;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, aib_ar_buffer_bytes(max_floats));
  // all of it zeroed: a word whose high half equals a call's epoch is data
  if (e == cudaSuccess) e = cudaMemset(p, 0, aib_ar_buffer_bytes(max_floats));
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
  return static_cast<int>(std::min<int64_t>(kMaxCtas, std::max<int64_t>(1, (n + 1023) / 1024)));
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
    a.recv[p] = reinterpret_cast<uint64_t *>(static_cast<unsigned char *>(g->buffers[p]) + kRecvOff);
  }
  a.counters = reinterpret_cast<int32_t *>(static_cast<unsigned char *>(g->buffers[g->rank]) + kCounterOff);
  a.max_floats = g->max_floats;
  a.rank = g->rank;
  a.world = g->world;
  oneshot_kernel<<<aib_ar_ctas(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, in, out, n, max_polls,
                                                                                      d_status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return aib_set_errorf("aib_allreduce_oneshot_f32: %s", cudaGetErrorString(e)), AIB_ECUDA;
  return AIB_OK;
}
