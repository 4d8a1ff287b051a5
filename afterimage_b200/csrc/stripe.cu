// Striped resident layout of a compressed stream.
//
// The reference keeps each chunk's bytes where the encoder wrote them
// (afterimage/runtime/huffman_chunked.py:180-206: chunk c at
// packed[chunk_offsets[c]], chunks back to back, 8 slack bytes at the end)
// and its decoder reads them there (afterimage/runtime/gpu_decode_v2.py:36-52).
// The decode kernel gives each lane of a warp one of 32 consecutive chunks,
// so in that layout a warp's 16-byte stream copies land in 32 places about a
// chunk apart. The striped layout stores the same bytes so that those copies
// are one 512-byte run: in the region of group g (chunks 32g .. 32g + 31) the
// chunk in column l keeps its 16-byte block i at block i * 32 + l. A region
// has as many rows as its longest chunk has blocks; the blocks past a shorter
// chunk's end are zero. Nothing else changes: the decode reads the same bits
// in the same order, only from other addresses.
//
// huffman_chunked.py:180-187 records why the encoder does not pad every chunk
// to the layer's longest one (one rare chunk set the stride for all). Here
// the padding is per group of 32 neighbours and exists only in the device
// copy; the stored and transferred stream keeps the reference's format.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "aib_internal.h"

namespace aibstripe {

constexpr int kThreads = 256;

// One CTA per group region (grid-stride over groups). Thread t of a region
// writes its blocks t, t + kThreads, ...: block b is row b / 32, column
// b % 32, i.e. bytes 16 * (b / 32) .. + 16 of chunk 32 g + b % 32.
__global__ void __launch_bounds__(kThreads) stripe_kernel(const uint8_t *__restrict__ src, int64_t src_nbytes,
                                                          int64_t offset_base, const int32_t *__restrict__ offs,
                                                          const int32_t *__restrict__ nbytes, int64_t n_chunks,
                                                          const int64_t *__restrict__ group_base, int64_t n_groups,
                                                          uint4 *__restrict__ dst, int64_t dst_blocks,
                                                          int32_t *status) {
  for (int64_t g = blockIdx.x; g < n_groups; g += gridDim.x) {
    const int64_t b0 = group_base[g];
    const int64_t b1 = group_base[g + 1];
    if (b0 < 0 || b1 < b0 || b1 > dst_blocks || (b1 - b0) % 32) {
      if (status && threadIdx.x == 0) atomicOr(status, AIB_STATUS_BAD_CHUNK_RANGE);
      continue;
    }
    for (int64_t b = threadIdx.x; b < b1 - b0; b += kThreads) {
      const int64_t c = g * 32 + (b & 31);
      const int64_t k0 = (b >> 5) * 16;  // first byte of the block within its chunk
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if (c < n_chunks) {
        const int64_t nb = nbytes[c];
        const int64_t off = static_cast<int64_t>(offs[c]) - offset_base;
        if (off < 0 || nb < 0 || off + nb > src_nbytes) {
          if (status) atomicOr(status, AIB_STATUS_BAD_CHUNK_RANGE);
        } else {
          const int64_t n = nb - k0 < 16 ? nb - k0 : 16;
          for (int i = 0; i < n; ++i) w[i >> 2] |= static_cast<uint32_t>(__ldg(src + off + k0 + i)) << (8 * (i & 3));
        }
      }
      dst[b0 + b] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

}  // namespace aibstripe

using namespace aibstripe;

AIB_API int aib_stripe_layout(const int32_t *chunk_nbytes, int64_t n_chunks, int64_t *group_base,
                              int64_t *total_blocks) {
  if (n_chunks < 0) return aib_set_error("aib_stripe_layout: negative n_chunks"), AIB_EINVAL;
  if (!group_base || !total_blocks || (n_chunks > 0 && !chunk_nbytes))
    return aib_set_error("aib_stripe_layout: null pointer"), AIB_EINVAL;
  const int64_t n_groups = (n_chunks + 31) / 32;
  int64_t base = 0;
  for (int64_t g = 0; g < n_groups; ++g) {
    group_base[g] = base;
    int64_t rows = 0;
    for (int64_t c = g * 32; c < std::min(n_chunks, g * 32 + 32); ++c) {
      if (chunk_nbytes[c] < 0)
        return aib_set_errorf("aib_stripe_layout: chunk %lld has a negative byte count", (long long)c), AIB_EINVAL;
      rows = std::max<int64_t>(rows, (static_cast<int64_t>(chunk_nbytes[c]) + 15) / 16);
    }
    base += rows * 32;
  }
  group_base[n_groups] = base;
  *total_blocks = base;
  return AIB_OK;
}

AIB_API int aib_stripe_stream_host(const uint8_t *src, int64_t src_nbytes, int64_t offset_base,
                                   const int32_t *chunk_offsets, const int32_t *chunk_nbytes, int64_t n_chunks,
                                   const int64_t *group_base, uint8_t *dst, int64_t dst_nbytes) {
  if (n_chunks < 0 || src_nbytes < 0 || dst_nbytes < 0)
    return aib_set_error("aib_stripe_stream_host: negative size"), AIB_EINVAL;
  if (n_chunks == 0) return AIB_OK;
  if (!src || !chunk_offsets || !chunk_nbytes || !group_base || !dst)
    return aib_set_error("aib_stripe_stream_host: null pointer"), AIB_EINVAL;
  const int64_t n_groups = (n_chunks + 31) / 32;
  if (group_base[n_groups] * 16 > dst_nbytes)
    return aib_set_errorf("aib_stripe_stream_host: dst holds %lld bytes, the layout needs %lld",
                          (long long)dst_nbytes, (long long)(group_base[n_groups] * 16)),
           AIB_EINVAL;
  for (int64_t g = 0; g < n_groups; ++g) {
    const int64_t b0 = group_base[g], b1 = group_base[g + 1];
    if (b0 < 0 || b1 < b0 || (b1 - b0) % 32)
      return aib_set_errorf("aib_stripe_stream_host: group %lld has a bad region [%lld, %lld)", (long long)g,
                            (long long)b0, (long long)b1),
             AIB_EINVAL;
    std::memset(dst + b0 * 16, 0, static_cast<size_t>((b1 - b0) * 16));
    const int64_t rows = (b1 - b0) / 32;
    for (int64_t c = g * 32; c < std::min(n_chunks, g * 32 + 32); ++c) {
      const int64_t nb = chunk_nbytes[c];
      const int64_t off = static_cast<int64_t>(chunk_offsets[c]) - offset_base;
      if (off < 0 || nb < 0 || off + nb > src_nbytes || (nb + 15) / 16 > rows)
        return aib_set_errorf("aib_stripe_stream_host: chunk %lld does not fit the stream or its region",
                              (long long)c),
               AIB_EINVAL;
      for (int64_t k = 0; k < nb; k += 16)
        std::memcpy(dst + (b0 + (c & 31) + 32 * (k / 16)) * 16, src + off + k,
                    static_cast<size_t>(std::min<int64_t>(16, nb - k)));
    }
  }
  return AIB_OK;
}

AIB_API int aib_stripe_stream(const uint8_t *src, int64_t src_nbytes, int64_t offset_base,
                              const int32_t *chunk_offsets, const int32_t *chunk_nbytes, int64_t chunk_base,
                              int64_t n_chunks, const int64_t *group_base, uint8_t *dst, int64_t dst_nbytes,
                              int32_t *d_status, void *stream) {
  if (n_chunks < 0 || src_nbytes < 0 || dst_nbytes < 0)
    return aib_set_error("aib_stripe_stream: negative size"), AIB_EINVAL;
  if (chunk_base < 0 || chunk_base % 32)
    return aib_set_errorf("aib_stripe_stream: chunk_base %lld must be a non-negative multiple of 32",
                          (long long)chunk_base),
           AIB_EINVAL;
  if (n_chunks == 0) return AIB_OK;
  if (!src || !chunk_offsets || !chunk_nbytes || !group_base || !dst)
    return aib_set_error("aib_stripe_stream: null pointer"), AIB_EINVAL;
  if (reinterpret_cast<uintptr_t>(dst) % 16 || dst_nbytes % 16)
    return aib_set_error("aib_stripe_stream: dst must be 16-byte aligned and hold whole 16-byte blocks"), AIB_EINVAL;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return aib_set_errorf("aib_stripe_stream: %s", cudaGetErrorString(e)), AIB_ECUDA;
  const int64_t n_groups = (n_chunks + 31) / 32;
  const int grid = static_cast<int>(std::min<int64_t>(n_groups, static_cast<int64_t>(sms) * 16));
  stripe_kernel<<<grid, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      src, src_nbytes, offset_base, chunk_offsets, chunk_nbytes, n_chunks, group_base, n_groups,
      reinterpret_cast<uint4 *>(dst), dst_nbytes / 16, d_status);
  e = cudaGetLastError();
  if (e != cudaSuccess) return aib_set_errorf("aib_stripe_stream: %s", cudaGetErrorString(e)), AIB_ECUDA;
  return AIB_OK;
}
