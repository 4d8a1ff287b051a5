// sm_100a kernels for the lossless BF16 weight-decode path, plus their C ABI.
//
// Format (reference: afterimage/runtime/huffman_chunked.py:135-207): the
// exponent stream of a tensor is split into chunks of `chunk_size` symbols;
// chunk c is an MSB-first canonical-Huffman bitstream, byte aligned, at byte
// chunk_offsets[c] of `packed`. The reference decoder (ChunkedBitReader,
// huffman_chunked.py:210-244; Triton kernel gpu_decode_v2.py:27-68) looks up
// sym_lut/len_lut with the next max_bits bits, emits one symbol and consumes
// its length.
//
// Kernel design (one launch decodes any number of whole or partial tensors):
//   * one chunk per lane, 32 consecutive chunks per warp ("group");
//   * a 12-bit first-level table, built once per tensor from the reference
//     LUTs (aib_build_tables), staged into shared memory with one TMA bulk
//     copy per CTA. An entry holds up to four symbols whose codes fit
//     entirely inside the 12 bits, with their total length; codes longer
//     than that (rare: the table covers every code of <= 12 bits) take an
//     exact slow path through the reference LUT in global memory, so every
//     decoded symbol equals the reference's LUT result;
//   * each lane's chunk bytes stream through a per-lane shared-memory ring
//     of 16-byte blocks filled by cp.async a few blocks ahead; each loop
//     iteration builds a 64-bit window of the stream from three ring words
//     at the lane's bit position and makes five table lookups in it;
//   * symbols are flushed four at a time into a per-lane shared-memory
//     ring; every 64 symbols the warp merges the ring with the sign/mantissa
//     bytes (the reference's _recombine, compressed_store.py:94-114) and
//     writes 16-byte vectorised BF16 stores, 128 contiguous bytes per chunk.
// The decoder uses no tensor cores and no scratch global memory: the
// exponent never round-trips through HBM. The fused decode -> GEMV kernels
// further down share the reader and table; they keep one fp32 partial sum
// per chunk in scratch (their per-lane reader refills its bit buffer a word
// at a time from the same kind of ring).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "aib_internal.h"

// ---------------------------------------------------------------------------
// error plumbing
// ---------------------------------------------------------------------------
static thread_local char g_err[512] = "";

void aib_set_error(const char *msg) { std::snprintf(g_err, sizeof(g_err), "%s", msg); }

void aib_set_errorf(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

#define AIB_CUDA(call)                                                          \
  do {                                                                          \
    cudaError_t e_ = (call);                                                    \
    if (e_ != cudaSuccess) {                                                    \
      aib_set_errorf("%s: %s (%s)", __func__, cudaGetErrorString(e_), #call);  \
      return AIB_ECUDA;                                                         \
    }                                                                           \
  } while (0)

namespace aib {

// Tuning parameters (compile-time; -D overrides exist for sweeps).
#ifndef AIB_WARPS
#define AIB_WARPS 18
#endif
#ifndef AIB_PHASE
#define AIB_PHASE 64
#endif
#ifndef AIB_MIN_BLOCKS
#define AIB_MIN_BLOCKS 1
#endif
#ifndef AIB_SLOTS
#define AIB_SLOTS 4
#endif
#ifndef AIB_FAST_BITS
#define AIB_FAST_BITS 12
#endif
// Launches with fewer groups than a wave of warps spread them over every SM
// (fewer active warps per CTA) instead of filling few CTAs; groups are
// dealt to CTAs round-robin.
#ifndef AIB_SPREAD
#define AIB_SPREAD 1
#endif
constexpr int kFastBits = AIB_FAST_BITS;
constexpr int kFastSize = 1 << kFastBits;
constexpr int kFastBytes = kFastSize * 8;
constexpr int kTablesBytes = kFastBytes + 16;  // fast table + {flags, max_bits, pad}
constexpr int kWarps = AIB_WARPS;
constexpr int kThreads = kWarps * 32;
constexpr int kPhase = AIB_PHASE;  // symbols per lane between merges (multiple of 32)
#ifndef AIB_RING_MULT
#define AIB_RING_MULT 2
#endif
// ring bytes per lane (a power of two >= kPhase + 4 * kLookups + 4); what
// exceeds kPhase is the slack a lane may decode ahead of its warp's merge
constexpr int kRing = kPhase * AIB_RING_MULT;
constexpr int kRow = kRing + 8;   // padded row: lanes at equal k hit different banks
constexpr int kRingWarpBytes = 32 * kRow;
constexpr int kSlots = AIB_SLOTS;                // stream ring slots per lane (power of two >= 2)
constexpr int kSlotRow = kSlots * 16 + 16;       // padded: lanes' slot k spread over the banks
constexpr int kStreamWarpBytes = 32 * kSlotRow;
constexpr int kSmemBytes = kFastBytes + kWarps * (kRingWarpBytes + kStreamWarpBytes);
constexpr unsigned kWaitLimit = AIB_WAIT_LIMIT_POLLS;  // bounded mbarrier wait (polls, with backoff)

enum Mode { kModeBF16 = 0, kModeU8 = 1, kModeI32 = 2 };
constexpr int kDefaultChunk = 1024;  // compress_layer's default chunk_size

struct Job {
  const uint8_t *packed;
  int64_t packed_cap;
  int64_t packed_nbytes;
  int64_t offset_base;
  const int32_t *offs;    // entry c - chunk_base describes chunk c
  const int32_t *nbytes;
  const int64_t *stripe;  // striped layout: first block of group g at entry g - chunk_base / 32; else null
  int64_t chunk_base;
  const uint2 *fast;
  const int32_t *flags;
  const int32_t *sym_lut;
  const int8_t *len_lut;
  const uint8_t *sm;
  void *out;
  int64_t n_symbols;
  int64_t e0, e1;
  int64_t c_begin, c_end;  // covering chunk range
  int64_t n_groups;        // ceil((c_end - c_begin) / 32)
  int32_t max_bits;
  int32_t chunk_size;
  int32_t cta_begin;
  int32_t ctas;
  int32_t vec_ok;
  int32_t pad;
};

struct Batch {
  Job job[AIB_MAX_BATCH];
  int32_t count;
};

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// 1-D TMA bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint32_t bswap(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

// 8 exponents + 8 sign/mantissa bytes -> 8 bf16 (bits = s<<15 | e<<7 | m).
__device__ __forceinline__ uint4 combine8(uint2 ex, uint2 sm) {
  const uint32_t M = 0x807F807Fu;
  uint4 o;
  // the fields are disjoint, so e * 128 + rest == e << 7 | rest
  o.x = __byte_perm(ex.x, 0, 0x4140) * 128u + (__byte_perm(sm.x, 0, 0x1100) & M);
  o.y = __byte_perm(ex.x, 0, 0x4342) * 128u + (__byte_perm(sm.x, 0, 0x3322) & M);
  o.z = __byte_perm(ex.y, 0, 0x4140) * 128u + (__byte_perm(sm.y, 0, 0x1100) & M);
  o.w = __byte_perm(ex.y, 0, 0x4342) * 128u + (__byte_perm(sm.y, 0, 0x3322) & M);
  return o;
}

__device__ __forceinline__ uint16_t combine1(uint32_t e, uint32_t sm) {
  return static_cast<uint16_t>((e << 7) | (sm & 0x7Fu) | ((sm & 0x80u) << 8));
}

// ---------------------------------------------------------------------------
// table construction (prepare_decode_tables)
// ---------------------------------------------------------------------------
__global__ void validate_lut_kernel(const int32_t *__restrict__ sym_lut, const int8_t *__restrict__ len_lut,
                                    int max_bits, int32_t *flags) {
  const int size = 1 << max_bits;
  int bad = 0;
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < size; w += gridDim.x * blockDim.x) {
    const int s = sym_lut[w];
    const int l = len_lut[w];
    if (s < 0 || s > 255 || l < 0 || l > max_bits) {
      bad |= AIB_STATUS_LUT_RANGE;
    } else if (l > 0) {
      // a prefix-code LUT repeats an entry across every window sharing the
      // code's l leading bits (huffman.py:140-148)
      const int base = w & ~((1 << (max_bits - l)) - 1);
      if (sym_lut[base] != s || len_lut[base] != l) bad |= AIB_STATUS_LUT_NOT_PREFIX;
    }
  }
  if (bad) atomicOr(flags, bad);
}

// Entry format of the first-level table (uint2 per 12-bit window):
//   x = up to four decoded symbols, symbol i in byte i (unused bytes zero)
//   y = bits consumed (bits 0..4) | 8 * symbol count (bits 8..15)
// y == 0 marks a window whose first code is longer than 12 bits (or not
// decidable from 12 bits): the kernel then looks the window up in the
// reference LUT itself.
__global__ void build_fast_kernel(const int32_t *__restrict__ sym_lut, const int8_t *__restrict__ len_lut,
                                  int max_bits, uint2 *fast, int32_t *header) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v == 0) header[1] = max_bits;
  if (v >= kFastSize) return;
  const uint32_t mask = (max_bits >= 32) ? 0xFFFFFFFFu : ((1u << max_bits) - 1u);
  uint32_t syms = 0;
  int cnt = 0, p = 0;
  while (cnt < 4) {
    uint32_t w;
    bool full;
    if (p + max_bits <= kFastBits) {
      w = (static_cast<uint32_t>(v) >> (kFastBits - p - max_bits)) & mask;
      full = true;
    } else {
      const int known = kFastBits - p;  // bits of v left; the rest of the window is unknown
      const uint32_t kbits = known > 0 ? (static_cast<uint32_t>(v) & ((1u << known) - 1u)) : 0u;
      w = kbits << (max_bits - known);
      full = false;
    }
    const int s = sym_lut[w];
    const int l = len_lut[w];
    // a partially known window is decided only when its code lies entirely
    // inside the known bits (a prefix code is fixed by its leading bits)
    if (!full && !(l >= 1 && l <= kFastBits - p)) break;
    if (l < 0 || l > 16) break;
    syms |= (static_cast<uint32_t>(s) & 0xFFu) << (8 * cnt);
    ++cnt;
    p += l;
  }
  fast[v] = cnt == 0 ? make_uint2(0u, 0u)
                     : make_uint2(syms, static_cast<uint32_t>(p) | (static_cast<uint32_t>(8 * cnt) << 8));
}

// ---------------------------------------------------------------------------
// the decode kernel
// ---------------------------------------------------------------------------
// L2 policies: a chunk's compressed bytes are fetched 16 bytes at a time
// over its whole decode, so they are kept (evict_last) and fetched 256 bytes
// at a time; sign/mantissa bytes and BF16 output are touched once and leave
// L2 first.
__device__ __forceinline__ uint64_t policy_keep() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_stream() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint2 ld_once8(const void *p, uint64_t pol) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ void st_once16(void *p, uint4 v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.u32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w), "l"(pol)
               : "memory");
}

__device__ __forceinline__ void st_once8(void *p, uint2 v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v2.u32 [%0], {%1,%2}, %3;" ::"l"(p), "r"(v.x), "r"(v.y),
               "l"(pol)
               : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// 16-byte asynchronous global -> shared copy (no register involvement); each
// copy is its own commit group so a lane can wait for its oldest block only.
__device__ __forceinline__ void cp_async16(void *sdst, const void *gsrc, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint.L2::256B [%0], [%1], 16, 16, %2;\n"
               "cp.async.commit_group;" ::"r"(smem_u32(sdst)),
               "l"(gsrc), "l"(pol)
               : "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Per-lane bit reader over one chunk: a 64-bit MSB-aligned buffer held as
// two 32-bit halves (ah:al) with `nb` valid bits, refilled 32 bits at a time
// straight from the lane's shared-memory stream ring (word `wi`, counted
// from the 16-byte block that holds the chunk's first byte). Every shift
// amount is below 32 (consumption <= 16 bits per lookup, refills while
// nb < 32), so each step is a single funnel shift. The ring has kSlots
// 16-byte slots, block k in slot k % kSlots; entering block k waits for its
// copy and requests block k + kSlots - 1 into the slot block k - 1 used, so
// kSlots - 1 copies stay in flight ~(kSlots - 1) * 16 bytes ahead.
struct Reader {
  uint32_t ah, al;
  int nb;
  int wi;      // next word to load (block wi / 4, slot (wi / 4) % kSlots)
  int64_t bi;  // next 16-byte block to request
  int end;     // bit index of the chunk's end, counted like wi * 32 - nb
};

// The reference reader stops refilling at the chunk's last byte and shifts
// in zeros (huffman_chunked.py:225-231, cpu_decode.py:84-88); this reader
// refills from whatever follows in `packed`. A prefix-code lookup never
// depends on those bits, but the exact slow path looks up the whole window,
// so it clears the window bits that lie past the chunk's end first.
__device__ __forceinline__ uint32_t slow_window(const Reader &r, int max_bits) {
  uint32_t w = (r.ah >> 16) >> (16 - max_bits);
  const int rem = r.end - (r.wi * 32 - r.nb);  // chunk bits not yet consumed
  if (rem < max_bits) w &= rem <= 0 ? 0u : ~((1u << (max_bits - rem)) - 1u);
  return w;
}

// entering the block of word wi: its copy has landed; request the one
// kSlots - 1 blocks ahead
__device__ __forceinline__ void reader_next_block(Reader &r, unsigned char *ring, const uint4 *src, int64_t bmax,
                                                  uint64_t pol) {
  cp_async_wait<kSlots - 2>();
  cp_async16(ring + (((r.wi >> 2) + kSlots - 1) & (kSlots - 1)) * 16, src + min(r.bi, bmax), pol);
  ++r.bi;
}

// nb < 32: append the next word below the valid bits
__device__ __forceinline__ void reader_refill(Reader &r, unsigned char *ring, const uint4 *src, int64_t bmax,
                                              uint64_t pol) {
  if ((r.wi & 3) == 0) reader_next_block(r, ring, src, bmax, pol);
  const uint32_t w = bswap(*reinterpret_cast<const uint32_t *>(ring + (r.wi & (kSlots * 4 - 1)) * 4));
  r.ah |= w >> r.nb;
  r.al |= __funnelshift_r(0u, w, static_cast<uint32_t>(r.nb));  // w << (32 - nb); 0 when nb == 0
  r.nb += 32;
  ++r.wi;
}

// drop `n` (< 32) consumed bits
__device__ __forceinline__ void reader_consume(Reader &r, uint32_t n) {
  r.ah = __funnelshift_l(r.al, r.ah, n);
  r.al <<= n;
  r.nb -= static_cast<int>(n);
}

__device__ __forceinline__ void reader_init(Reader &r, unsigned char *ring, const uint4 *src, int64_t bmax,
                                            int64_t pos, int64_t nbytes, uint64_t pol) {
  const int64_t b0 = pos >> 4;
  r.end = static_cast<int>(min(static_cast<int64_t>(pos & 15) * 8 + nbytes * 8, static_cast<int64_t>(INT32_MAX)));
#pragma unroll
  for (int s = 0; s < kSlots - 1; ++s) cp_async16(ring + s * 16, src + min(b0 + s, bmax), pol);
  r.bi = b0 + kSlots - 1;
  r.wi = 0;
  reader_next_block(r, ring, src, bmax, pol);  // block b0 landed; request block b0 + kSlots - 1
  r.wi = static_cast<int>((pos >> 2) & 3);
  r.ah = 0;
  r.al = 0;
  r.nb = 0;
  // first word (block b0 is already entered), then drop the bytes before the chunk start
  const uint32_t w = bswap(*reinterpret_cast<const uint32_t *>(ring + r.wi * 4));
  r.ah = w;
  r.nb = 32;
  ++r.wi;
  reader_consume(r, static_cast<uint32_t>(pos & 3) * 8);
}

// ---------------------------------------------------------------------------
// Windowed reader: the lane's position in its chunk is one bit counter, and
// each loop iteration builds a 64-bit window of the stream from three
// consecutive 32-bit words of the lane's shared-memory ring (no per-lookup
// refill, no branch). The ring holds kSlots 16-byte blocks of the chunk plus
// a two-word guard after the last slot that repeats the first two words of
// slot 0, so three consecutive words never wrap. A window covers any
// kLookups table lookups of at most kFastBits bits each plus one exact
// long-code lookup of up to 16 bits.
// ---------------------------------------------------------------------------
#ifndef AIB_LOOKUPS
#define AIB_LOOKUPS 5
#endif
constexpr int kLookups = AIB_LOOKUPS;
// the window covers kLookups full lookups, or a long-code lookup (up to 16
// bits) after kLookups - 1 of them
static_assert(kLookups * kFastBits <= 64 && (kLookups - 1) * kFastBits + 16 <= 64, "a window holds 64 bits");
static_assert(kSlots >= 4, "the window needs the current and the next block, two more in flight");
static_assert((kRing & (kRing - 1)) == 0 && kRing >= kPhase + 4 * kLookups + 4, "ring: a power of two with slack");

struct Window {
  int pos;   // bits consumed, counted from the first byte of block b0 (the block of the chunk's first byte)
  int lo;    // the lowest block (relative to b0) the window may still read
  int end;   // bit index of the chunk's end, same origin as pos
  int sh;    // the chunk's j-th block is block b0 + (j << sh): 0 in the reference layout, 5 striped
  int64_t b0;
};

// Request block j (relative to b0) into its slot; slot 0's first two words
// also go to the guard. One commit group per block.
__device__ __forceinline__ void win_request(const Window &r, int j, unsigned char *ring, const uint4 *src,
                                            int64_t bmax, uint64_t pol) {
  const int slot = j & (kSlots - 1);
  const uint4 *g = src + min(r.b0 + (static_cast<int64_t>(j) << r.sh), bmax);
  asm volatile("cp.async.cg.shared.global.L2::cache_hint.L2::256B [%0], [%1], 16, 16, %2;" ::"r"(
                   smem_u32(ring + slot * 16)),
               "l"(g), "l"(pol)
               : "memory");
  if (slot == 0)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, 8;" ::"r"(smem_u32(ring + kSlots * 16)), "l"(g)
                 : "memory");
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// pos: the chunk's first byte (reference layout: its byte offset; striped:
// 16 x its first block). sh: log2 of the block stride.
__device__ __forceinline__ void win_init(Window &r, unsigned char *ring, const uint4 *src, int64_t bmax,
                                         int64_t pos, int64_t nbytes, int sh, uint64_t pol) {
  r.b0 = pos >> 4;
  r.sh = sh;
  r.pos = static_cast<int>(pos & 15) * 8;
  r.lo = 0;
  r.end = static_cast<int>(min(static_cast<int64_t>(r.pos) + nbytes * 8, static_cast<int64_t>(INT32_MAX)));
#pragma unroll
  for (int j = 0; j < kSlots; ++j) win_request(r, j, ring, src, bmax, pol);
}

// Before reading the window: when the position has entered a new block, the
// slot of the block before it is free and takes the block kSlots - 1
// ahead; then wait until the current and the next block have landed (every
// request but the newest kSlots - 2). An iteration consumes fewer than 128
// bits, so the position enters at most one new block per iteration.
__device__ __forceinline__ void win_stage(Window &r, unsigned char *ring, const uint4 *src, int64_t bmax,
                                          uint64_t pol) {
  const int nlo = r.pos >> 7;
  if (nlo != r.lo) {
    r.lo = nlo;
    win_request(r, nlo + kSlots - 1, ring, src, bmax, pol);
  }
  cp_async_wait<kSlots - 2>();
}

// The 64 stream bits from r.pos on, MSB first, as hi:lo.
__device__ __forceinline__ void win_read(const Window &r, const unsigned char *ring, uint32_t &hi, uint32_t &lo) {
  const uint32_t *w = reinterpret_cast<const uint32_t *>(ring) + ((r.pos >> 5) & (kSlots * 4 - 1));
  const uint32_t a0 = bswap(w[0]), a1 = bswap(w[1]), a2 = bswap(w[2]);
  hi = __funnelshift_l(a1, a0, static_cast<uint32_t>(r.pos));  // shift amount taken mod 32
  lo = __funnelshift_l(a2, a1, static_cast<uint32_t>(r.pos));
}

// emit() for the windowed loop: the pending word's high part is always zero
// before a payload is added (a flush leaves only the spill of the payload
// that crossed the word), so the spill is assigned rather than merged.
__device__ __forceinline__ void emit_w(uint2 e, uint32_t &olo, int &n8, int &k, unsigned char *my_ring) {
  olo |= e.x << n8;
  const uint32_t spill = __funnelshift_l(e.x, 0u, static_cast<uint32_t>(n8));
  n8 += static_cast<int>(e.y >> 8);
  if (n8 >= 32) {
    *reinterpret_cast<uint32_t *>(my_ring + (k & (kRing - 1))) = olo;
    olo = spill;
    n8 -= 32;
    k += 4;
  }
}

// A warp's first group of its job; later ones follow every ctas * kWarps.
__device__ __forceinline__ int64_t first_group(int cta_begin, int ctas, int warp) {
  const int64_t b = static_cast<int64_t>(blockIdx.x) - cta_begin;
  return AIB_SPREAD ? b + static_cast<int64_t>(warp) * ctas : b * kWarps + warp;
}

// The group loop: every warp decodes groups of 32 consecutive chunks of job
// J. CSC != 0 makes the chunk size a compile-time constant (the merge's
// address offsets become immediates).
template <int MODE, int CSC>
__device__ __forceinline__ void decode_groups(const Job &J, const uint2 *s_fast, unsigned char *smem,
                                              int32_t *status) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned char *ring_base = smem + kFastBytes + warp * kRingWarpBytes;
  unsigned char *my_ring = ring_base + lane * kRow;
  unsigned char *my_stream = smem + kFastBytes + kWarps * kRingWarpBytes + warp * kStreamWarpBytes + lane * kSlotRow;
  const int64_t cs = CSC ? static_cast<int64_t>(CSC) : static_cast<int64_t>(J.chunk_size);
  const int max_bits = J.max_bits;
  const uint4 *src = reinterpret_cast<const uint4 *>(J.packed);
  const int64_t bmax = J.packed_cap / 16 - 1;
  // lane's slot in the interior merge: each chunk's kPhase symbols are kVecs
  // 8-symbol vectors; at step it the lane covers vector (lane % kVecs) of
  // chunk it + kIters * (lane / kVecs). The lanes of a half warp then read
  // two rows kIters apart, whose 8-byte slots fall in disjoint bank pairs.
  constexpr int kVecs = kPhase / 8;
  constexpr int kRowsPerIt = 32 / kVecs;
  constexpr int kIters = kPhase * 32 / 8 / 32;
  static_assert(kIters * kRowsPerIt == 32, "the merge covers the warp's 32 chunks");
  const int64_t lane_elem = (lane / kVecs) * kIters * cs + (lane % kVecs) * 8;
  const int64_t it_stride = cs;
  const int ring_rd = (lane / kVecs) * kIters * kRow + (lane % kVecs) * 8;
  const uint64_t pol_keep = policy_keep();
  const uint64_t pol_once = policy_stream();

  for (int64_t grp = first_group(J.cta_begin, J.ctas, warp); grp < J.n_groups;
       grp += static_cast<int64_t>(J.ctas) * kWarps) {
    const int64_t c0 = J.c_begin + grp * 32;
    const int64_t c = c0 + lane;
    const bool active = c < J.c_end;
    const int64_t ge0 = c0 * cs;  // first element of the group
    // warp-uniform: all 32 chunks complete and inside [e0, e1), phases whole
    const bool fast = J.vec_ok && (cs % kPhase) == 0 && ge0 >= J.e0 && ge0 + 32 * cs <= J.e1;
    const int need = active ? static_cast<int>(min(cs, J.e1 - c * cs)) : 0;

    Window rd;
    rd.pos = 0; rd.lo = 0; rd.end = 0; rd.sh = 0; rd.b0 = 0;
    if (active) {
      int64_t nbyt = J.nbytes[c - J.chunk_base];
      int64_t pos;
      bool bad;
      if (J.stripe) {
        // block i of the chunk: stripe_base[group] + (c mod 32) + 32 i
        const int64_t sb = J.stripe[(c >> 5) - (J.chunk_base >> 5)];
        bad = sb < 0 || sb > J.packed_nbytes / 16 || nbyt < 0;
        pos = bad ? 0 : (sb + (c & 31)) * 16;
        bad = bad || (nbyt > 0 && pos + ((nbyt - 1) >> 4) * 512 + 16 > J.packed_nbytes);
      } else {
        pos = static_cast<int64_t>(J.offs[c - J.chunk_base]) - J.offset_base;
        bad = pos < 0 || nbyt < 0 || pos + nbyt > J.packed_nbytes;
      }
      if (bad) {
        if (status) atomicOr(status, AIB_STATUS_BAD_CHUNK_RANGE);
        pos = 0;
        nbyt = 0;
      }
      win_init(rd, my_stream, src, bmax, pos, nbyt, J.stripe ? 5 : 0, pol_keep);
    }

    const int max_need = fast ? static_cast<int>(cs)
                              : static_cast<int>(__reduce_max_sync(0xffffffffu, static_cast<unsigned>(need)));
    int k = 0;              // symbols flushed to the ring (multiple of 4)
    int n8 = 0;             // 8 x symbols pending in olo:ohi
    uint32_t olo = 0;
    const int64_t grp_out = ge0 - J.e0;  // output index of the group's first element (fast path)

    for (int ph = 0; ph < max_need; ph += kPhase) {
      uint2 smv[kIters];
      if (MODE == kModeBF16 && fast) {
        // issue this phase's sign/mantissa loads now; they land while the
        // lanes decode
        const uint8_t *smp = J.sm + grp_out + lane_elem + ph;
#pragma unroll
        for (int it = 0; it < kIters; ++it) smv[it] = ld_once8(smp + it * it_stride, pol_once);
        // warm L2 with this lane's chunk segment of the next phase
        if (ph + kPhase < max_need) prefetch_l2(J.sm + grp_out + static_cast<int64_t>(lane) * cs + ph + kPhase);
      }
      const int target = min(ph + kPhase, need);
      // Lanes that reach this phase's target keep decoding into the ring's
      // slack, up to `cap`: an iteration starting below it writes fewer than
      // 4 * kLookups + 4 more symbols, never into the region still to be
      // merged. A warp then waits on its slowest lane about once per chunk.
      // positions in units of 8 x symbols: 8 * k + n8 counts the symbols decoded
      const int target8 = 8 * target;
      const int cap8 = 8 * min(ph + kRing - 4 * kLookups - 4, need);
      while (__any_sync(0xffffffffu, 8 * k + n8 < target8)) {
        if (8 * k + n8 < cap8) {
          win_stage(rd, my_stream, src, bmax, pol_keep);
          uint32_t hi, lo;
          win_read(rd, my_stream, hi, lo);
          // kLookups first-level lookups. A window whose first code is longer
          // than the table has entry 0: it consumes and emits nothing, so
          // the lookups after it see the same window (the last one included);
          // the exact lookup below resolves it.
          uint32_t acc = 0;  // bits 0..7: bits consumed; bits 8..15: 8 x symbols
          uint32_t ylast = 0;
#pragma unroll
          for (int u = 0; u < kLookups; ++u) {
            const uint2 e = s_fast[hi >> (32 - kFastBits)];
            ylast = e.y;
            hi = __funnelshift_l(lo, hi, e.y);  // consume e.y & 31 bits
            lo = __funnelshift_l(0u, lo, e.y);
            acc += e.y;
            emit_w(e, olo, n8, k, my_ring);
          }
          if (__any_sync(__activemask(), ylast == 0u)) {
            if (ylast == 0u) {
              // at least 64 - (kLookups - 1) * kFastBits >= 16 window bits remain
              uint32_t w = (hi >> 16) >> (16 - max_bits);
              const int rem = rd.end - rd.pos - static_cast<int>(acc & 0xFFu);
              if (rem < max_bits) w &= rem <= 0 ? 0u : ~((1u << (max_bits - rem)) - 1u);
              const uint32_t sy = static_cast<uint32_t>(__ldg(J.sym_lut + w)) & 0xFFu;
              const uint32_t l = static_cast<uint32_t>(static_cast<int>(__ldg(J.len_lut + w))) & 31u;
              acc += l;
              emit_w(make_uint2(sy, 8u << 8), olo, n8, k, my_ring);
            }
          }
          rd.pos += static_cast<int>(acc & 0xFFu);
        }
      }
      // end of this lane's range: flush the partial word (idempotent)
      if (k < need && k + (n8 >> 3) >= need)
        *reinterpret_cast<uint32_t *>(my_ring + (k & (kRing - 1))) = olo;
      __syncwarp();

      if (fast) {
        // ---- merge, interior group: 32 chunks x kPhase symbols, 16-byte stores
        const unsigned char *rr = ring_base + ring_rd + (ph & (kRing - 1));
        const int64_t ob = grp_out + lane_elem + ph;
#pragma unroll
        for (int it = 0; it < kIters; ++it) {
          const uint2 ex = *reinterpret_cast<const uint2 *>(rr + it * kRow);
          const int64_t oi = ob + it * it_stride;
          if (MODE == kModeBF16) {
            st_once16(static_cast<uint16_t *>(J.out) + oi, combine8(ex, smv[it]), pol_once);
          } else if (MODE == kModeU8) {
            st_once8(static_cast<uint8_t *>(J.out) + oi, ex, pol_once);
          } else {
            uint4 a, b;
            a.x = __byte_perm(ex.x, 0, 0x4440); a.y = __byte_perm(ex.x, 0, 0x4441);
            a.z = __byte_perm(ex.x, 0, 0x4442); a.w = __byte_perm(ex.x, 0, 0x4443);
            b.x = __byte_perm(ex.y, 0, 0x4440); b.y = __byte_perm(ex.y, 0, 0x4441);
            b.z = __byte_perm(ex.y, 0, 0x4442); b.w = __byte_perm(ex.y, 0, 0x4443);
            int32_t *o = static_cast<int32_t *>(J.out) + oi;
            __stcs(reinterpret_cast<uint4 *>(o), a);
            __stcs(reinterpret_cast<uint4 *>(o + 4), b);
          }
        }
      } else {
        // ---- merge, general group: ragged ranges, odd chunk sizes, edges
        for (int it = 0; it < kIters; ++it) {
          const int r = it * kRowsPerIt + lane / kVecs;
          const int q8 = (lane % kVecs) * 8;
          const int64_t cr = c0 + r;
          if (cr >= J.c_end) continue;
          const int64_t base = cr * cs;
          const int64_t lo = max(base, J.e0);
          const int64_t hi = min(base + cs, J.e1);
          const int64_t g = base + ph + q8;
          if (g >= hi || g + 8 <= lo) continue;
          const unsigned char *rrow = ring_base + r * kRow;
          const int ro = (ph + q8) & (kRing - 1);
          const int64_t oi = g - J.e0;
          if (J.vec_ok && g >= lo && g + 8 <= hi) {
            const uint2 ex = *reinterpret_cast<const uint2 *>(rrow + ro);
            if (MODE == kModeBF16) {
              const uint2 s8 = __ldcs(reinterpret_cast<const uint2 *>(J.sm + oi));
              __stcs(reinterpret_cast<uint4 *>(static_cast<uint16_t *>(J.out) + oi), combine8(ex, s8));
            } else if (MODE == kModeU8) {
              __stcs(reinterpret_cast<uint2 *>(static_cast<uint8_t *>(J.out) + oi), ex);
            } else {
              int32_t *o = static_cast<int32_t *>(J.out) + oi;
              for (int jj = 0; jj < 8; ++jj) o[jj] = static_cast<int32_t>(rrow[ro + jj]);
            }
          } else {
            for (int jj = 0; jj < 8; ++jj) {
              const int64_t gg = g + jj;
              if (gg < lo || gg >= hi) continue;
              const uint32_t e = rrow[(ro + jj) & (kRing - 1)];
              const int64_t o = gg - J.e0;
              if (MODE == kModeBF16)
                static_cast<uint16_t *>(J.out)[o] = combine1(e, J.sm[o]);
              else if (MODE == kModeU8)
                static_cast<uint8_t *>(J.out)[o] = static_cast<uint8_t>(e);
              else
                static_cast<int32_t *>(J.out)[o] = static_cast<int32_t>(e);
            }
          }
        }
      }
      __syncwarp();
    }
    // drain this lane's stream copies before its slots are reused (or the
    // kernel exits)
    cp_async_wait<0>();
  }
}

// Stages a tensor's first-level table into shared memory with one bulk copy
// (TMA 1-D, mbarrier completion, bounded wait) and zeroes it when the
// table's flags say the reference LUT is not a plain prefix-code table
// (every lookup then takes the exact slow path). Returns false, uniformly
// for the CTA, when the copy did not complete in time.
// Polls `bar` for the phase of `parity` at most `limit` times, with backoff.
// Every thread of the CTA gets the same answer: true when the wait gave up.
__device__ __forceinline__ bool cta_wait_gave_up(uint64_t *bar, unsigned parity, unsigned limit) {
  unsigned spins = 0;
  int timed_out = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++spins > limit) {
      timed_out = 1;
      break;
    }
    __nanosleep(64);
  }
  // the whole CTA leaves together so no barrier below misses a thread
  return __syncthreads_or(timed_out) != 0;
}

__device__ __forceinline__ bool stage_table(uint2 *s_fast, const uint2 *src, const int32_t *flags, uint64_t *bar,
                                            int32_t *status) {
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_expect_tx(bar, kFastBytes);
    bulk_g2s(s_fast, src, kFastBytes, bar);
  }
  __syncthreads();
  if (cta_wait_gave_up(bar, 0, kWaitLimit)) {
    if (status && threadIdx.x == 0) atomicOr(status, AIB_STATUS_WAIT_TIMEOUT);
    // The copy may still be in flight: give it a second bounded wait before
    // the CTA exits and its shared memory goes to another CTA. The launch
    // has failed either way; its outputs are to be discarded.
    (void)cta_wait_gave_up(bar, 0, kWaitLimit);
    return false;
  }
  if (*flags != 0) {
    for (int i = threadIdx.x; i < kFastSize; i += blockDim.x) s_fast[i] = make_uint2(0u, 0u);
    __syncthreads();
  }
  return true;
}

// CSC selects the group loop: 1024 (every job has the reference's default
// chunk size), 0 (any chunk size) or -1 (per job: jobs with chunk size 1024
// take the specialised loop, the others the general one; a CTA serves one
// job, so the choice is uniform per CTA).
template <int MODE, int CSC>
__global__ void __launch_bounds__(kThreads, AIB_MIN_BLOCKS) decode_kernel(const __grid_constant__ Batch batch,
                                                                          int32_t *status) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar;

  int jsel = 0;
  for (int t = 1; t < batch.count; ++t)
    if (static_cast<int>(blockIdx.x) >= batch.job[t].cta_begin) jsel = t;
  const Job &J = batch.job[jsel];

  uint2 *s_fast = reinterpret_cast<uint2 *>(smem);
  if (!stage_table(s_fast, J.fast, J.flags, &bar, status)) return;

  if (CSC < 0) {
    if (J.chunk_size == kDefaultChunk)
      decode_groups<MODE, kDefaultChunk>(J, s_fast, smem, status);
    else
      decode_groups<MODE, 0>(J, s_fast, smem, status);
  } else {
    decode_groups<MODE, (CSC > 0 ? CSC : 0)>(J, s_fast, smem, status);
  }
}

// ---------------------------------------------------------------------------
// fused decode -> GEMV: y = W x for one input vector (a single-token
// projection), W read only in compressed form and never written out
// ---------------------------------------------------------------------------
// The range is whole rows of a row-major [rows, cols] tensor whose rows are
// whole chunks (cols % chunk_size == 0). A warp takes 32 consecutive rows at
// one column chunk j: lane l decodes chunk (row0 + l, j) on its own -- no
// ring, no merge, no warp synchronisation inside the chunk -- and every
// lane reads the same stretch x[j*cs ...] of the input (one broadcast
// load). Each complete word of four exponents is combined with its four
// sign/mantissa bytes into BF16 weights (the reference's _recombine,
// compressed_store.py:94-114) and multiplied into an fp32 partial sum. The
// chunk's partial is stored; a second kernel sums each row's partials in
// column order and rounds to BF16, so the result is deterministic.
struct GemvJob {
  const uint8_t *packed;
  int64_t packed_cap;
  int64_t packed_nbytes;
  int64_t offset_base;
  const int32_t *offs;
  const int32_t *nbytes;
  int64_t chunk_base;
  const uint2 *fast;
  const int32_t *flags;
  const int32_t *sym_lut;
  const int8_t *len_lut;
  const uint8_t *sm;     // element e0 at index 0
  const uint16_t *x;     // bf16[cols]
  float *partial;        // chunk (r, j) of the range at r * cpr + j
  uint16_t *y;           // bf16[rows]
  int64_t c0;            // global index of the range's first chunk
  int64_t rows;
  int64_t n_groups;      // ceil(rows / 32) * cpr
  int64_t row_begin;     // rows of the batch's earlier jobs
  int64_t cols;
  int32_t cpr;           // chunks per row
  int32_t chunk_size;
  int32_t max_bits;
  int32_t cta_begin;
  int32_t ctas;
  int32_t pad;
};

struct GemvBatch {
  GemvJob job[AIB_MAX_BATCH];
  int32_t count;
};

constexpr int kGemvSmemBytes = kFastBytes + kThreads * kSlotRow;

// four weights (exponent bytes of `ew`, sign/mantissa bytes smp[k..k+3])
// times x[k..k+3] (bf16, read through L1: every lane of the warp is at
// about the same column), accumulated in fp32
__device__ __forceinline__ void dot4(uint32_t ew, int k, const uint8_t *smp, const uint16_t *xp, float &a0,
                                     float &a1) {
  const uint32_t sw = __ldg(reinterpret_cast<const unsigned int *>(smp + k));
  const uint2 xv = __ldg(reinterpret_cast<const uint2 *>(xp + k));
  const uint32_t M = 0x807F807Fu;
  const uint32_t p01 = __byte_perm(ew, 0, 0x4140) * 128u + (__byte_perm(sw, 0, 0x1100) & M);
  const uint32_t p23 = __byte_perm(ew, 0, 0x4342) * 128u + (__byte_perm(sw, 0, 0x3322) & M);
  a0 = fmaf(__uint_as_float(p01 << 16), __uint_as_float(xv.x << 16), a0);
  a1 = fmaf(__uint_as_float(p01 & 0xFFFF0000u), __uint_as_float(xv.x & 0xFFFF0000u), a1);
  a0 = fmaf(__uint_as_float(p23 << 16), __uint_as_float(xv.y << 16), a0);
  a1 = fmaf(__uint_as_float(p23 & 0xFFFF0000u), __uint_as_float(xv.y & 0xFFFF0000u), a1);
}

// emit() for the GEMV: a full word of four symbols is multiplied in at once
// (only words inside the chunk: need is a multiple of four)
__device__ __forceinline__ void emit_dot(uint2 e, uint32_t &olo, uint32_t &ohi, int &n8, int &k, int need,
                                         const uint8_t *smp, const uint16_t *xp, float &a0, float &a1) {
  olo |= e.x << n8;
  ohi |= __funnelshift_l(e.x, 0u, static_cast<uint32_t>(n8));
  n8 += static_cast<int>(e.y >> 8);
  if (n8 >= 32) {
    if (k < need) dot4(olo, k, smp, xp, a0, a1);
    olo = ohi;
    ohi = 0;
    n8 -= 32;
    k += 4;
  }
}

template <int CSC>
__device__ __forceinline__ void gemv_groups(const GemvJob &G, const uint2 *s_fast, unsigned char *smem,
                                            int32_t *status) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  unsigned char *my_stream = smem + kFastBytes + (warp * 32 + lane) * kSlotRow;
  const int cs = CSC ? CSC : G.chunk_size;
  const int max_bits = G.max_bits;
  const uint4 *src = reinterpret_cast<const uint4 *>(G.packed);
  const int64_t bmax = G.packed_cap / 16 - 1;
  const uint64_t pol_keep = policy_keep();
  for (int64_t grp = first_group(G.cta_begin, G.ctas, warp); grp < G.n_groups;
       grp += static_cast<int64_t>(G.ctas) * kWarps) {
    const int64_t rb = grp / G.cpr;
    const int j = static_cast<int>(grp - rb * G.cpr);
    const int64_t row = rb * 32 + lane;
    const bool active = row < G.rows;
    const int64_t cl = row * G.cpr + j;  // chunk index within the range
    const uint8_t *smp = G.sm + cl * cs;
    const uint16_t *xp = G.x + static_cast<int64_t>(j) * cs;
    Reader rd;
    rd.ah = 0; rd.al = 0; rd.nb = 0; rd.wi = 0; rd.bi = 0; rd.end = 0;
    if (active) {
      const int64_t c = G.c0 + cl;
      int64_t pos = static_cast<int64_t>(G.offs[c - G.chunk_base]) - G.offset_base;
      int64_t nbyt = G.nbytes[c - G.chunk_base];
      if (pos < 0 || nbyt < 0 || pos + nbyt > G.packed_nbytes) {
        if (status) atomicOr(status, AIB_STATUS_BAD_CHUNK_RANGE);
        pos = 0;
        nbyt = 0;
      }
      reader_init(rd, my_stream, src, bmax, pos, nbyt, pol_keep);
      for (int q = 0; q < cs; q += 128) prefetch_l2(smp + q);
    }
    const int need = active ? cs : 0;
    int k = 0, n8 = 0;
    uint32_t olo = 0, ohi = 0;
    float a0 = 0.f, a1 = 0.f;
    while (__any_sync(0xffffffffu, k < need)) {
      if (k < need) {
        if (rd.nb < 32) reader_refill(rd, my_stream, src, bmax, pol_keep);
        uint32_t ymin = 0xFFFFFFFFu;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const uint2 e = s_fast[rd.ah >> (32 - kFastBits)];
          ymin = min(ymin, e.y);
          reader_consume(rd, e.y & 31u);
          emit_dot(e, olo, ohi, n8, k, need, smp, xp, a0, a1);
        }
        if (__any_sync(__activemask(), ymin == 0u)) {
          if (ymin == 0u) {
            // a code longer than the table: the reference LUT (>= 20 valid bits here)
            const uint32_t w = slow_window(rd, max_bits);
            const uint32_t sy = static_cast<uint32_t>(__ldg(G.sym_lut + w)) & 0xFFu;
            const uint32_t l = static_cast<uint32_t>(static_cast<int>(__ldg(G.len_lut + w))) & 31u;
            reader_consume(rd, l);
            emit_dot(make_uint2(sy, 8u << 8), olo, ohi, n8, k, need, smp, xp, a0, a1);
          }
        }
      }
    }
    if (active) G.partial[cl] = a0 + a1;
    cp_async_wait<0>();
  }
}

template <int CSC>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvBatch batch,
                                                           int32_t *status) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar;
  int jsel = 0;
  for (int t = 1; t < batch.count; ++t)
    if (static_cast<int>(blockIdx.x) >= batch.job[t].cta_begin) jsel = t;
  const GemvJob &G = batch.job[jsel];
  uint2 *s_fast = reinterpret_cast<uint2 *>(smem);
  if (!stage_table(s_fast, G.fast, G.flags, &bar, status)) return;
  if (CSC < 0) {
    if (G.chunk_size == kDefaultChunk)
      gemv_groups<kDefaultChunk>(G, s_fast, smem, status);
    else
      gemv_groups<0>(G, s_fast, smem, status);
  } else {
    gemv_groups<(CSC > 0 ? CSC : 0)>(G, s_fast, smem, status);
  }
}

// y[r] = bf16(sum over j of partial[r * cpr + j]), j ascending
__global__ void gemv_rows_kernel(const __grid_constant__ GemvBatch batch, int64_t total_rows) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total_rows; t += stride) {
    int jsel = 0;
    for (int q = 1; q < batch.count; ++q)
      if (t >= batch.job[q].row_begin) jsel = q;
    const GemvJob &G = batch.job[jsel];
    const int64_t r = t - G.row_begin;
    const float *p = G.partial + r * G.cpr;
    float acc = 0.f;
    for (int q = 0; q < G.cpr; ++q) acc += p[q];
    G.y[r] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
  }
}

__global__ void recombine_kernel(const uint8_t *__restrict__ e, const uint8_t *__restrict__ sm, int64_t n,
                                 uint16_t *__restrict__ out, int vec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t nv = n / 8;
    for (int64_t v = i; v < nv; v += stride) {
      const uint2 ex = __ldcs(reinterpret_cast<const uint2 *>(e) + v);
      const uint2 s = __ldcs(reinterpret_cast<const uint2 *>(sm) + v);
      __stcs(reinterpret_cast<uint4 *>(out) + v, combine8(ex, s));
    }
    for (int64_t t = nv * 8 + i; t < n; t += stride) out[t] = combine1(e[t], sm[t]);
  } else {
    for (int64_t t = i; t < n; t += stride) out[t] = combine1(e[t], sm[t]);
  }
}

// Self-test of the bounded wait: one CTA waits on an mbarrier whose phase
// nothing completes (no copy is issued, nobody arrives), gives up after
// `limit` polls and reports it the way a stalled table copy does.
__global__ void wait_timeout_selftest_kernel(unsigned limit, int32_t *status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) mbar_init(&bar, 1);
  __syncthreads();
  if (cta_wait_gave_up(&bar, 0, limit) && threadIdx.x == 0) atomicOr(status, AIB_STATUS_WAIT_TIMEOUT);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct DeviceInfo {
  int sms = 0;
  int occ[3] = {0, 0, 0};
  int gemv_occ = 1;
  bool ready = false;
};
static DeviceInfo g_dev[64];
static std::mutex g_dev_mu;

template <int MODE, int CSC>
static int setup_one(DeviceInfo &di) {
  AIB_CUDA(cudaFuncSetAttribute(decode_kernel<MODE, CSC>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  int occ = 0;
  AIB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel<MODE, CSC>, kThreads, kSmemBytes));
  di.occ[MODE] = di.occ[MODE] ? std::min(di.occ[MODE], std::max(1, occ)) : std::max(1, occ);
  return AIB_OK;
}

template <int MODE>
static int setup_kernel(int dev, DeviceInfo &di) {
  (void)dev;
  int rc = setup_one<MODE, 0>(di);
  if (rc == AIB_OK) rc = setup_one<MODE, kDefaultChunk>(di);
  if (rc == AIB_OK) rc = setup_one<MODE, -1>(di);
  return rc;
}

static int device_info(DeviceInfo **out) {
  int dev = 0;
  AIB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    aib_set_error("device index out of range");
    return AIB_EINVAL;
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo &di = g_dev[dev];
  if (!di.ready) {
    AIB_CUDA(cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev));
    int rc;
    if ((rc = setup_kernel<kModeBF16>(dev, di)) != AIB_OK) return rc;
    if ((rc = setup_kernel<kModeU8>(dev, di)) != AIB_OK) return rc;
    if ((rc = setup_kernel<kModeI32>(dev, di)) != AIB_OK) return rc;
    AIB_CUDA(cudaFuncSetAttribute(gemv_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemBytes));
    AIB_CUDA(cudaFuncSetAttribute(gemv_kernel<kDefaultChunk>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kGemvSmemBytes));
    AIB_CUDA(cudaFuncSetAttribute(gemv_kernel<-1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemBytes));
    int occ = 0;
    AIB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel<-1>, kThreads, kGemvSmemBytes));
    di.gemv_occ = std::max(1, occ);
    di.ready = true;
  }
  *out = &di;
  return AIB_OK;
}

static bool aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Fills a Job from a descriptor; returns AIB_OK, or AIB_EINVAL with the
// message set. *empty is set when there is nothing to produce.
static int make_job(const aib_stream_desc *d, int mode, Job *j, bool *empty) {
  if (!d) {
    aib_set_error("null descriptor");
    return AIB_EINVAL;
  }
  *empty = false;
  // the kernels count a chunk's bits in 32-bit integers: 2^26 symbols of at most 16 bits stay in range
  if (d->chunk_size < 1 || d->chunk_size > (1 << 26))
    return aib_set_errorf("chunk_size must be in [1, 2^26], got %d", d->chunk_size), AIB_EINVAL;
  if (d->max_bits < 0 || d->max_bits > 16)
    return aib_set_errorf("max_bits must be in [0, 16], got %d", d->max_bits), AIB_EINVAL;
  if (d->n_symbols < 0 || d->elem_begin < 0 || d->elem_end < d->elem_begin || d->elem_end > d->n_symbols)
    return aib_set_errorf("bad element range [%lld, %lld) for %lld symbols", (long long)d->elem_begin,
                          (long long)d->elem_end, (long long)d->n_symbols),
           AIB_EINVAL;
  if (d->elem_end == d->elem_begin) {
    *empty = true;
    return AIB_OK;
  }
  const int64_t n_chunks = (d->n_symbols + d->chunk_size - 1) / d->chunk_size;
  if (n_chunks > INT32_MAX) return aib_set_error("too many chunks for int32 chunk indices"), AIB_EINVAL;
  if (!d->packed || !aligned(d->packed, 16)) return aib_set_error("packed must be a 16-byte aligned device pointer"), AIB_EINVAL;
  if (d->packed_capacity < 16 || (d->packed_capacity & 15) || d->packed_nbytes < 0 ||
      d->packed_nbytes > d->packed_capacity)
    return aib_set_errorf("packed_capacity %lld must be a multiple of 16, >= 16 and >= packed_nbytes %lld",
                          (long long)d->packed_capacity, (long long)d->packed_nbytes),
           AIB_EINVAL;
  if ((!d->chunk_offsets && !d->stripe_base) || !d->chunk_nbytes || !d->tables || !d->sym_lut || !d->len_lut ||
      !d->out)
    return aib_set_error("null device pointer in descriptor"), AIB_EINVAL;
  if (d->stripe_base && d->chunk_base % 32)
    return aib_set_errorf("a striped stream's chunk_base must be a multiple of 32, got %lld", (long long)d->chunk_base),
           AIB_EINVAL;
  if (!aligned(d->tables, 16)) return aib_set_error("tables must be 16-byte aligned"), AIB_EINVAL;
  if (mode == kModeBF16 && !d->sign_mantissa) return aib_set_error("sign_mantissa is required"), AIB_EINVAL;
  if (!aligned(d->out, mode == kModeBF16 ? 2 : (mode == kModeI32 ? 4 : 1)))
    return aib_set_error("out is misaligned for its element type"), AIB_EINVAL;

  j->packed = d->packed;
  j->packed_cap = d->packed_capacity;
  j->packed_nbytes = d->packed_nbytes;
  j->offset_base = d->offset_base;
  j->offs = d->chunk_offsets;
  j->nbytes = d->chunk_nbytes;
  j->stripe = d->stripe_base;
  j->chunk_base = d->chunk_base;
  j->fast = static_cast<const uint2 *>(d->tables);
  j->flags = reinterpret_cast<const int32_t *>(static_cast<const unsigned char *>(d->tables) + kFastBytes);
  j->sym_lut = d->sym_lut;
  j->len_lut = d->len_lut;
  j->sm = d->sign_mantissa;
  j->out = d->out;
  j->n_symbols = d->n_symbols;
  j->e0 = d->elem_begin;
  j->e1 = d->elem_end;
  j->chunk_size = d->chunk_size;
  j->max_bits = d->max_bits;
  j->c_begin = d->elem_begin / d->chunk_size;
  j->c_end = (d->elem_end + d->chunk_size - 1) / d->chunk_size;
  j->n_groups = (j->c_end - j->c_begin + 31) / 32;
  if (d->chunk_base < 0 || d->chunk_base > j->c_begin)
    return aib_set_errorf("chunk_base %lld must be in [0, %lld]", (long long)d->chunk_base,
                          (long long)j->c_begin),
           AIB_EINVAL;
  const bool base_ok = (d->chunk_size % 8 == 0) && (d->elem_begin % 8 == 0);
  if (mode == kModeBF16)
    j->vec_ok = base_ok && aligned(d->out, 16) && aligned(d->sign_mantissa, 8);
  else if (mode == kModeU8)
    j->vec_ok = base_ok && aligned(d->out, 8);
  else
    j->vec_ok = base_ok && aligned(d->out, 16);
  j->pad = 0;
  return AIB_OK;
}

// groups of 32 chunks handled per warp before a CTA is considered full
static constexpr int kGroupsPerWarp = 1;
#ifndef AIB_WAVES
#define AIB_WAVES 4
#endif
// most CTAs a launch uses, in waves of (SMs x resident CTAs per SM)
static constexpr int kMaxWaves = AIB_WAVES;

// Splits `cap` CTAs over n jobs in proportion to their groups by largest
// remainder, each job at least 1 CTA and at most max_useful[i]. The shares
// add up to cap unless the per-job bounds force otherwise, so a launch
// sized to whole waves does not spill a few CTAs into one more wave.
static void apportion(int64_t cap, const int64_t *groups, const int64_t *max_useful, int n, int64_t total,
                      int32_t *share) {
  int64_t sum = 0;
  int64_t rem[AIB_MAX_BATCH];  // cap * groups - share * total: what the job is still owed
  for (int i = 0; i < n; ++i) {
    const int64_t q = cap * groups[i];
    const int64_t s = std::max<int64_t>(1, std::min(q / total, max_useful[i]));
    rem[i] = q - s * total;
    share[i] = static_cast<int32_t>(s);
    sum += s;
  }
  while (sum < cap) {
    int best = -1;
    for (int i = 0; i < n; ++i)
      if (share[i] < max_useful[i] && (best < 0 || rem[i] > rem[best])) best = i;
    if (best < 0) break;
    ++share[best];
    rem[best] -= total;
    ++sum;
  }
}

// max_ctas > 0 caps the grid (one CTA holds one SM): the warps then loop
// over more groups each and the SMs left over run other streams' kernels.
template <int MODE>
static int launch(const aib_stream_desc *descs, int count, int32_t *status, void *stream, int max_ctas = 0) {
  if (count < 1 || count > AIB_MAX_BATCH) {
    aib_set_errorf("batch count must be in [1, %d], got %d", AIB_MAX_BATCH, count);
    return AIB_EINVAL;
  }
  if (!descs) return aib_set_error("null descriptor array"), AIB_EINVAL;
  // validate every descriptor on the host before touching the device
  Batch batch;
  std::memset(&batch, 0, sizeof(batch));
  int64_t total_groups = 0;
  int n = 0;
  int rc = AIB_OK;
  for (int i = 0; i < count; ++i) {
    bool empty = false;
    rc = make_job(&descs[i], MODE, &batch.job[n], &empty);
    if (rc != AIB_OK) return rc;
    if (empty) continue;
    total_groups += batch.job[n].n_groups;
    ++n;
  }
  if (n == 0) return AIB_OK;
  DeviceInfo *di = nullptr;
  rc = device_info(&di);
  if (rc != AIB_OK) return rc;
  batch.count = n;
  // CTAs: as many as the work needs at kGroupsPerWarp groups per warp, capped
  // at a few full waves; split across jobs in proportion to their groups.
  const int64_t wave = static_cast<int64_t>(di->sms) * di->occ[MODE];
  int64_t want = (total_groups + kWarps * kGroupsPerWarp - 1) / (kWarps * kGroupsPerWarp);
  if (AIB_SPREAD) want = std::max(want, std::min(total_groups, wave));
  int64_t cap = std::min<int64_t>(std::max<int64_t>(want, 1), kMaxWaves * wave);
  if (max_ctas > 0) cap = std::min<int64_t>(cap, max_ctas);
  int64_t groups[AIB_MAX_BATCH], max_useful[AIB_MAX_BATCH];
  int32_t share[AIB_MAX_BATCH];
  for (int i = 0; i < n; ++i) {
    groups[i] = batch.job[i].n_groups;
    max_useful[i] = AIB_SPREAD ? groups[i] : (groups[i] + kWarps - 1) / kWarps;
  }
  apportion(cap, groups, max_useful, n, total_groups, share);
  int cta = 0;
  for (int i = 0; i < n; ++i) {
    batch.job[i].cta_begin = cta;
    batch.job[i].ctas = share[i];
    cta += share[i];
  }
  int n_default = 0;
  for (int i = 0; i < n; ++i) n_default += batch.job[i].chunk_size == kDefaultChunk;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_default == n)
    decode_kernel<MODE, kDefaultChunk><<<cta, kThreads, kSmemBytes, st>>>(batch, status);
  else if (n_default > 0)
    decode_kernel<MODE, -1><<<cta, kThreads, kSmemBytes, st>>>(batch, status);
  else
    decode_kernel<MODE, 0><<<cta, kThreads, kSmemBytes, st>>>(batch, status);
  AIB_CUDA(cudaGetLastError());
  return AIB_OK;
}

static int gemv_launch(const aib_gemv_desc *descs, int count, int32_t *status, void *stream) {
  if (count < 1 || count > AIB_MAX_BATCH) {
    aib_set_errorf("batch count must be in [1, %d], got %d", AIB_MAX_BATCH, count);
    return AIB_EINVAL;
  }
  if (!descs) return aib_set_error("null descriptor array"), AIB_EINVAL;
  GemvBatch batch;
  std::memset(&batch, 0, sizeof(batch));
  int64_t total_groups = 0, total_rows = 0;
  int n = 0;
  for (int i = 0; i < count; ++i) {
    const aib_gemv_desc *g = &descs[i];
    const aib_stream_desc &d = g->stream;
    if (d.elem_begin == d.elem_end && d.elem_begin >= 0 && d.elem_end <= d.n_symbols) continue;  // no rows
    if (!g->x || !g->partial || !g->y) return aib_set_error("gemv: null x, partial or y"), AIB_EINVAL;
    if (!aligned(g->x, 8) || !aligned(g->partial, 4) || !aligned(g->y, 2))
      return aib_set_error("gemv: x must be 8-byte, partial 4-byte and y 2-byte aligned"), AIB_EINVAL;
    if (d.chunk_size < 4 || d.chunk_size % 4)
      return aib_set_errorf("gemv: chunk_size must be a positive multiple of 4, got %d", d.chunk_size), AIB_EINVAL;
    if (g->cols < 1 || g->cols % d.chunk_size)
      return aib_set_errorf("gemv: cols %lld must be a positive multiple of chunk_size %d", (long long)g->cols,
                            d.chunk_size),
             AIB_EINVAL;
    if (d.elem_begin % g->cols || d.elem_end % g->cols)
      return aib_set_error("gemv: the element range must be whole rows"), AIB_EINVAL;
    if (!d.sign_mantissa || !aligned(d.sign_mantissa, 4))
      return aib_set_error("gemv: sign_mantissa must be a 4-byte aligned device pointer"), AIB_EINVAL;
    if (d.stripe_base) return aib_set_error("gemv: the stream must be in the reference layout (stripe_base NULL)"), AIB_EINVAL;
    // the stream checks shared with the decode (out is not written here)
    aib_stream_desc copy = d;
    copy.out = g->y;
    Job j;
    bool empty = false;
    const int rc = make_job(&copy, kModeBF16, &j, &empty);
    if (rc != AIB_OK) return rc;
    if (empty) continue;
    GemvJob &G = batch.job[n];
    G.packed = j.packed;
    G.packed_cap = j.packed_cap;
    G.packed_nbytes = j.packed_nbytes;
    G.offset_base = j.offset_base;
    G.offs = j.offs;
    G.nbytes = j.nbytes;
    G.chunk_base = j.chunk_base;
    G.fast = j.fast;
    G.flags = j.flags;
    G.sym_lut = j.sym_lut;
    G.len_lut = j.len_lut;
    G.sm = j.sm;
    G.x = static_cast<const uint16_t *>(g->x);
    G.partial = g->partial;
    G.y = static_cast<uint16_t *>(g->y);
    G.c0 = d.elem_begin / d.chunk_size;
    G.rows = (d.elem_end - d.elem_begin) / g->cols;
    G.cols = g->cols;
    G.cpr = static_cast<int32_t>(g->cols / d.chunk_size);
    G.n_groups = (G.rows + 31) / 32 * G.cpr;
    G.row_begin = total_rows;
    G.chunk_size = d.chunk_size;
    G.max_bits = d.max_bits;
    total_groups += G.n_groups;
    total_rows += G.rows;
    ++n;
  }
  if (n == 0) return AIB_OK;
  DeviceInfo *di = nullptr;
  int rc = device_info(&di);
  if (rc != AIB_OK) return rc;
  batch.count = n;
  const int64_t wave = static_cast<int64_t>(di->sms) * di->gemv_occ;
  int64_t want = std::max<int64_t>(1, (total_groups + kWarps - 1) / kWarps);
  if (AIB_SPREAD) want = std::max(want, std::min(total_groups, wave));
  const int64_t cap = std::min<int64_t>(want, kMaxWaves * wave);
  int64_t groups[AIB_MAX_BATCH], max_useful[AIB_MAX_BATCH];
  int32_t share[AIB_MAX_BATCH];
  for (int i = 0; i < n; ++i) {
    groups[i] = batch.job[i].n_groups;
    max_useful[i] = AIB_SPREAD ? groups[i] : (groups[i] + kWarps - 1) / kWarps;
  }
  apportion(cap, groups, max_useful, n, total_groups, share);
  int cta = 0;
  int n_default = 0;
  for (int i = 0; i < n; ++i) {
    GemvJob &G = batch.job[i];
    G.cta_begin = cta;
    G.ctas = share[i];
    cta += G.ctas;
    n_default += G.chunk_size == kDefaultChunk;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_default == n)
    gemv_kernel<kDefaultChunk><<<cta, kThreads, kGemvSmemBytes, st>>>(batch, status);
  else if (n_default > 0)
    gemv_kernel<-1><<<cta, kThreads, kGemvSmemBytes, st>>>(batch, status);
  else
    gemv_kernel<0><<<cta, kThreads, kGemvSmemBytes, st>>>(batch, status);
  AIB_CUDA(cudaGetLastError());
  const int64_t blocks = std::min<int64_t>((total_rows + 255) / 256, 4 * static_cast<int64_t>(di->sms));
  gemv_rows_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(batch, total_rows);
  AIB_CUDA(cudaGetLastError());
  return AIB_OK;
}

}  // namespace aib

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using namespace aib;

AIB_API const char *aib_last_error(void) { return g_err; }
AIB_API int aib_abi_version(void) { return 2; }
AIB_API size_t aib_tables_bytes(void) { return kTablesBytes; }

AIB_API int aib_build_tables(const int32_t *d_sym_lut, const int8_t *d_len_lut, int max_bits, void *d_tables,
                             void *stream) {
  if (!d_sym_lut || !d_len_lut || !d_tables) return aib_set_error("aib_build_tables: null pointer"), AIB_EINVAL;
  if (max_bits < 0 || max_bits > 16) return aib_set_errorf("aib_build_tables: max_bits %d not in [0, 16]", max_bits), AIB_EINVAL;
  if (!aligned(d_tables, 16)) return aib_set_error("aib_build_tables: tables must be 16-byte aligned"), AIB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char *base = static_cast<unsigned char *>(d_tables);
  int32_t *header = reinterpret_cast<int32_t *>(base + kFastBytes);
  AIB_CUDA(cudaMemsetAsync(header, 0, 16, s));
  const int lut = 1 << max_bits;
  validate_lut_kernel<<<std::min(64, (lut + 255) / 256), 256, 0, s>>>(d_sym_lut, d_len_lut, max_bits, header);
  AIB_CUDA(cudaGetLastError());
  build_fast_kernel<<<kFastSize / 256, 256, 0, s>>>(d_sym_lut, d_len_lut, max_bits, reinterpret_cast<uint2 *>(base),
                                                    header);
  AIB_CUDA(cudaGetLastError());
  return AIB_OK;
}

AIB_API int aib_tables_flags(const void *d_tables, int32_t *flags_out, void *stream) {
  if (!d_tables || !flags_out) return aib_set_error("aib_tables_flags: null pointer"), AIB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t v = 0;
  AIB_CUDA(cudaMemcpyAsync(&v, static_cast<const unsigned char *>(d_tables) + kFastBytes, 4, cudaMemcpyDeviceToHost, s));
  AIB_CUDA(cudaStreamSynchronize(s));
  *flags_out = v;
  return AIB_OK;
}

AIB_API int aib_decode_bf16(const aib_stream_desc *desc, int32_t *d_status, void *stream) {
  return launch<kModeBF16>(desc, 1, d_status, stream);
}

AIB_API int aib_decode_exponents_u8(const aib_stream_desc *desc, int32_t *d_status, void *stream) {
  return launch<kModeU8>(desc, 1, d_status, stream);
}

AIB_API int aib_decode_exponents_i32(const aib_stream_desc *desc, int32_t *d_status, void *stream) {
  return launch<kModeI32>(desc, 1, d_status, stream);
}

AIB_API int aib_decode_bf16_batch_ctas(const aib_stream_desc *descs, int count, int max_ctas, int32_t *d_status,
                                       void *stream) {
  if (max_ctas < 1) return aib_set_errorf("max_ctas must be >= 1, got %d", max_ctas), AIB_EINVAL;
  return launch<kModeBF16>(descs, count, d_status, stream, max_ctas);
}

AIB_API int aib_decode_bf16_batch(const aib_stream_desc *descs, int count, int32_t *d_status, void *stream) {
  return launch<kModeBF16>(descs, count, d_status, stream);
}

AIB_API int aib_decode_gemv_bf16_batch(const aib_gemv_desc *descs, int count, int32_t *d_status, void *stream) {
  return gemv_launch(descs, count, d_status, stream);
}

// Library-owned scratch for aib_decode_gemv_bf16_batch_noalloc. Some callers
// cannot allocate device memory themselves: a binding from another host
// language that only receives device pointers from the framework owning the
// memory, or code running under a framework whose allocator must see every
// byte (a VRAM budget that a side cudaMalloc would silently break). They get
// the per-chunk partial sums placed here instead: AIB_GEMV_SCRATCH_FLOATS
// floats (4 MiB), held by every GPU that loads the library until exit. In
// host code the array's name is only a stand-in for the device copy; its
// device address is looked up once per device (below) and passed on.
static __device__ __align__(256) float g_gemv_scratch[AIB_GEMV_SCRATCH_FLOATS];

static float *g_scratch_addr[64];
static std::mutex g_scratch_mu;

// Device address of g_gemv_scratch on the current device, looked up with
// cudaGetSymbolAddress on the first call for that device.
static int scratch_address(float **out) {
  int dev = 0;
  AIB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return aib_set_error("device index out of range"), AIB_EINVAL;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void *p = nullptr;
    AIB_CUDA(cudaGetSymbolAddress(&p, g_gemv_scratch));
    if (!p) return aib_set_error("gemv: no device address for the library scratch"), AIB_ECUDA;
    g_scratch_addr[dev] = static_cast<float *>(p);
  }
  *out = g_scratch_addr[dev];
  return AIB_OK;
}

AIB_API int aib_decode_gemv_bf16_batch_noalloc(const aib_gemv_desc *descs, int count, int32_t *d_status,
                                               void *stream) {
  if (count < 1 || count > AIB_MAX_BATCH) {
    aib_set_errorf("batch count must be in [1, %d], got %d", AIB_MAX_BATCH, count);
    return AIB_EINVAL;
  }
  if (!descs) return aib_set_error("null descriptor array"), AIB_EINVAL;
  // Each descriptor's area of the array (256-byte aligned), laid out and
  // checked against the array's size before any device call. The sums stop
  // at the first area that does not fit, so no bogus range can overflow them.
  int64_t area[AIB_MAX_BATCH];
  int64_t end = 0;
  for (int i = 0; i < count; ++i) {
    const aib_stream_desc &d = descs[i].stream;
    if (d.chunk_size < 1) return aib_set_errorf("chunk_size must be >= 1, got %d", d.chunk_size), AIB_EINVAL;
    if (d.n_symbols < 0 || d.elem_begin < 0 || d.elem_end < d.elem_begin || d.elem_end > d.n_symbols)
      return aib_set_error("gemv: bad element range"), AIB_EINVAL;
    const int64_t len = d.elem_end - d.elem_begin;
    const int64_t need = len / d.chunk_size + (len % d.chunk_size != 0);
    if (need > AIB_GEMV_SCRATCH_FLOATS - end)
      return aib_set_errorf("gemv: the batch needs more than the %d scratch floats the library holds "
                            "(descriptor %d needs %lld at offset %lld)",
                            AIB_GEMV_SCRATCH_FLOATS, i, (long long)need, (long long)end),
             AIB_EINVAL;
    area[i] = end;
    end += (need + 63) / 64 * 64;  // the next area starts 256-byte aligned
  }
  // Nothing in the scratch has to start at zero: the decode kernel writes
  // every partial sum of the batch before the row kernel reads it.
  float *base = nullptr;
  const int rc = scratch_address(&base);
  if (rc != AIB_OK) return rc;
  aib_gemv_desc local[AIB_MAX_BATCH];
  for (int i = 0; i < count; ++i) {
    local[i] = descs[i];
    local[i].partial = base + area[i];
  }
  return gemv_launch(local, count, d_status, stream);
}

AIB_API int aib_selftest_wait_timeout(unsigned polls, int32_t *d_status, void *stream) {
  if (!d_status) return aib_set_error("aib_selftest_wait_timeout: null status"), AIB_EINVAL;
  if (polls < 1 || polls > kWaitLimit)
    return aib_set_errorf("aib_selftest_wait_timeout: polls must be in [1, %u], got %u", kWaitLimit, polls),
           AIB_EINVAL;
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls, d_status);
  AIB_CUDA(cudaGetLastError());
  return AIB_OK;
}

AIB_API int aib_recombine(const uint8_t *exponent, const uint8_t *sign_mantissa, int64_t n, uint16_t *out,
                          void *stream) {
  if (n < 0) return aib_set_error("aib_recombine: negative n"), AIB_EINVAL;
  if (n == 0) return AIB_OK;
  if (!exponent || !sign_mantissa || !out) return aib_set_error("aib_recombine: null pointer"), AIB_EINVAL;
  if (!aligned(out, 2)) return aib_set_error("aib_recombine: out must be 2-byte aligned"), AIB_EINVAL;
  DeviceInfo *di = nullptr;
  int rc = device_info(&di);
  if (rc != AIB_OK) return rc;
  const int vec = aligned(exponent, 8) && aligned(sign_mantissa, 8) && aligned(out, 16);
  const int64_t work = vec ? (n + 7) / 8 : n;
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, static_cast<int64_t>(di->sms) * 8);
  recombine_kernel<<<static_cast<int>(std::max<int64_t>(blocks, 1)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      exponent, sign_mantissa, n, out, vec);
  AIB_CUDA(cudaGetLastError());
  return AIB_OK;
}
