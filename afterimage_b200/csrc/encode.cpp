// Product encoder for the chunked canonical-Huffman exponent format.
//
// Byte-identical to the reference encoder (Afterimage, paths within the
// project):
//   aib_split_bf16        afterimage/runtime/compressed_store.py:78-88
//                         (compress_layer's field split: exponent byte and
//                         (sign << 7) | mantissa byte per weight)
//   aib_histogram         afterimage/runtime/huffman_chunked.py:159
//                         (np.bincount(flat, minlength=256))
//   aib_build_code        afterimage/runtime/huffman.py:41-125
//                         (_natural_lengths with heapq tie-breaking on the
//                         insertion counter, _package_merge_limit when the
//                         natural depth exceeds max_bits, canonical_codes)
//   aib_build_decode_lut  afterimage/runtime/huffman.py:128-150
//   aib_pack_chunks       afterimage/runtime/huffman_chunked.py:41-98,
//                         :178-201 (MSB-first per-chunk packing, byte
//                         aligned, exclusive prefix-sum offsets, 8 zero
//                         tail bytes)
//
// The packer runs in two passes so chunks can be packed in parallel: pass 1
// sums each chunk's code lengths into its byte count, an exclusive prefix
// sum places every chunk, pass 2 packs each chunk at its offset. Each
// chunk's bytes depend only on its own symbols, so the output equals the
// reference's serial packer byte for byte.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <queue>
#include <vector>

#include "aib_internal.h"

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

struct HeapItem {
  int64_t freq;
  int64_t id;
  bool operator>(const HeapItem &o) const {
    return freq != o.freq ? freq > o.freq : id > o.id;
  }
};

// Natural Huffman depths with the reference's tie-breaking: heap entries
// are [freq, counter, symbols]; leaves take counters 0..k-1 in ascending
// symbol order, merged nodes take k, k+1, ... in creation order.
void natural_lengths(const int64_t counts[256], int lengths[256]) {
  std::vector<int> present;
  for (int s = 0; s < 256; ++s)
    if (counts[s] > 0) present.push_back(s);
  for (int s = 0; s < 256; ++s) lengths[s] = 0;
  if (present.empty()) return;
  if (present.size() == 1) {
    lengths[present[0]] = 1;
    return;
  }
  // node payloads: the list of symbols under each node
  std::vector<std::vector<int>> members;
  std::priority_queue<HeapItem, std::vector<HeapItem>, std::greater<HeapItem>> heap;
  for (size_t i = 0; i < present.size(); ++i) {
    members.push_back({present[i]});
    heap.push({counts[present[i]], (int64_t)i});
  }
  while (heap.size() > 1) {
    HeapItem lo = heap.top(); heap.pop();
    HeapItem hi = heap.top(); heap.pop();
    for (int s : members[lo.id]) lengths[s] += 1;
    for (int s : members[hi.id]) lengths[s] += 1;
    std::vector<int> merged = members[lo.id];
    merged.insert(merged.end(), members[hi.id].begin(), members[hi.id].end());
    members.push_back(std::move(merged));
    heap.push({lo.freq + hi.freq, (int64_t)members.size() - 1});
  }
}

struct PMItem {
  int64_t freq;
  std::vector<int> syms;
};

// Python orders (freq, [symbols]) tuples by freq, then by the symbol lists
// compared lexicographically.
bool pm_less(const PMItem &a, const PMItem &b) {
  if (a.freq != b.freq) return a.freq < b.freq;
  return std::lexicographical_compare(a.syms.begin(), a.syms.end(), b.syms.begin(), b.syms.end());
}

void package_merge(const int64_t counts[256], int max_bits, int lengths[256]) {
  std::vector<std::pair<int64_t, int>> items;
  for (int s = 0; s < 256; ++s)
    if (counts[s] > 0) items.push_back({counts[s], s});
  std::sort(items.begin(), items.end());
  for (int s = 0; s < 256; ++s) lengths[s] = 0;
  const size_t n = items.size();
  if (n <= 1) {
    if (n == 1) lengths[items[0].second] = 1;
    return;
  }
  std::vector<PMItem> prev;
  for (int k = 0; k < max_bits; ++k) {
    std::vector<PMItem> level;
    for (auto &it : items) level.push_back({it.first, {it.second}});
    if (k > 0) {
      for (size_t i = 0; i + 1 < prev.size(); i += 2) {
        PMItem p{prev[i].freq + prev[i + 1].freq, prev[i].syms};
        p.syms.insert(p.syms.end(), prev[i + 1].syms.begin(), prev[i + 1].syms.end());
        level.push_back(std::move(p));
      }
      std::stable_sort(level.begin(), level.end(), pm_less);
    }
    prev = std::move(level);
  }
  std::stable_sort(prev.begin(), prev.end(), pm_less);
  size_t take = std::min(prev.size(), 2 * (n - 1));
  for (size_t i = 0; i < take; ++i)
    for (int s : prev[i].syms) lengths[s] += 1;
}

int set_err(const char *msg) {
  aib_set_error(msg);
  return AIB_EINVAL;
}

}  // namespace

extern "C" {

AIB_API int aib_split_bf16(const uint16_t *bits, int64_t n, uint8_t *exponent,
                           uint8_t *sign_mantissa) {
  if (n < 0 || (n > 0 && (!bits || !exponent || !sign_mantissa)))
    return set_err("aib_split_bf16: bad arguments");
  int64_t i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < n; ++i) {
    uint32_t b = bits[i];
    exponent[i] = (uint8_t)((b >> 7) & 0xFF);
    sign_mantissa[i] = (uint8_t)((((b >> 15) & 1u) << 7) | (b & 0x7Fu));
  }
  return AIB_OK;
}

AIB_API int aib_histogram(const uint8_t *symbols, int64_t n, int64_t counts[256]) {
  if (n < 0 || !counts || (n > 0 && !symbols)) return set_err("aib_histogram: bad arguments");
  for (int s = 0; s < 256; ++s) counts[s] = 0;
#pragma omp parallel
  {
    int64_t local[256] = {0};
    int64_t i;
#pragma omp for schedule(static) nowait
    for (i = 0; i < n; ++i) local[symbols[i]]++;
#pragma omp critical
    for (int s = 0; s < 256; ++s) counts[s] += local[s];
  }
  return AIB_OK;
}

AIB_API int aib_build_code(const int64_t counts[256], int max_bits_limit, int32_t lengths_out[256],
                           uint32_t codes_out[256], int32_t *max_bits_out) {
  if (!counts || !lengths_out || !codes_out || !max_bits_out)
    return set_err("aib_build_code: null argument");
  if (max_bits_limit < 1 || max_bits_limit > 24)
    return set_err("aib_build_code: max_bits must be in [1, 24]");
  int lengths[256];
  natural_lengths(counts, lengths);
  int deepest = 0;
  for (int s = 0; s < 256; ++s) deepest = std::max(deepest, lengths[s]);
  if (deepest > max_bits_limit) package_merge(counts, max_bits_limit, lengths);
  // canonical codes: symbols ordered by (length, symbol)
  std::vector<std::pair<int, int>> order;
  for (int s = 0; s < 256; ++s)
    if (lengths[s] > 0) order.push_back({lengths[s], s});
  std::sort(order.begin(), order.end());
  for (int s = 0; s < 256; ++s) {
    lengths_out[s] = lengths[s];
    codes_out[s] = 0;
  }
  uint64_t code = 0;
  int prev_len = order.empty() ? 0 : order[0].first;
  int mb = 0;
  for (auto &o : order) {
    code <<= (o.first - prev_len);
    codes_out[o.second] = (uint32_t)code;
    code += 1;
    prev_len = o.first;
    mb = std::max(mb, o.first);
  }
  *max_bits_out = mb;
  return AIB_OK;
}

AIB_API int aib_build_decode_lut(const int32_t lengths[256], const uint32_t codes[256], int max_bits,
                                 int32_t *sym_lut, int8_t *len_lut) {
  if (max_bits < 0 || max_bits > 24 || !lengths || !codes || !sym_lut || !len_lut)
    return set_err("aib_build_decode_lut: bad arguments");
  const int64_t size = int64_t(1) << max_bits;
  std::memset(sym_lut, 0, sizeof(int32_t) * size);
  std::memset(len_lut, 0, sizeof(int8_t) * size);
  std::vector<std::pair<int, int>> order;
  for (int s = 0; s < 256; ++s)
    if (lengths[s] > 0) order.push_back({lengths[s], s});
  std::sort(order.begin(), order.end());
  for (auto &o : order) {
    const int ln = o.first, s = o.second;
    if (ln > max_bits) return set_err("aib_build_decode_lut: code longer than max_bits");
    const int64_t base = int64_t(codes[s]) << (max_bits - ln);
    const int64_t span = int64_t(1) << (max_bits - ln);
    for (int64_t w = base; w < base + span && w < size; ++w) {
      sym_lut[w] = s;
      len_lut[w] = (int8_t)ln;
    }
  }
  return AIB_OK;
}

AIB_API int aib_chunk_nbytes(const uint8_t *symbols, int64_t n, int64_t chunk_size,
                             const int32_t lengths[256], int32_t *chunk_nbytes,
                             int64_t *total_bytes) {
  if (n < 0 || chunk_size < 1 || !lengths || !total_bytes || (n > 0 && (!symbols || !chunk_nbytes)))
    return set_err("aib_chunk_nbytes: bad arguments");
  const int64_t n_chunks = (n + chunk_size - 1) / chunk_size;
  int64_t total = 0;
  int64_t c;
  bool bad = false;
#pragma omp parallel for schedule(static) reduction(+ : total) reduction(|| : bad)
  for (c = 0; c < n_chunks; ++c) {
    const int64_t a = c * chunk_size, b = std::min(a + chunk_size, n);
    int64_t bits = 0;
    for (int64_t i = a; i < b; ++i) {
      int l = lengths[symbols[i]];
      if (l <= 0) bad = true;
      bits += l;
    }
    const int64_t nb = (bits + 7) / 8;
    if (nb > INT32_MAX) bad = true;
    chunk_nbytes[c] = (int32_t)nb;
    total += nb;
  }
  if (bad) return set_err("aib_chunk_nbytes: a symbol has no code (or a chunk overflows int32)");
  *total_bytes = total;
  return AIB_OK;
}

// Packs every chunk at chunk_offsets[c]; chunk_offsets is an exclusive
// prefix sum of chunk_nbytes (computed here) and must fit int32, as the
// reference stores it. out must hold sum(chunk_nbytes) + 8 bytes; the
// 8-byte zero tail is written here too.
AIB_API int aib_pack_chunks(const uint8_t *symbols, int64_t n, int64_t chunk_size,
                            const int32_t lengths[256], const uint32_t codes[256],
                            const int32_t *chunk_nbytes, int32_t *chunk_offsets, uint8_t *out,
                            int64_t out_capacity) {
  if (n < 0 || chunk_size < 1 || !lengths || !codes || !out || (n > 0 && (!symbols || !chunk_nbytes || !chunk_offsets)))
    return set_err("aib_pack_chunks: bad arguments");
  const int64_t n_chunks = (n + chunk_size - 1) / chunk_size;
  int64_t pos = 0;
  for (int64_t c = 0; c < n_chunks; ++c) {
    if (pos > INT32_MAX) return set_err("aib_pack_chunks: packed stream exceeds int32 offsets");
    chunk_offsets[c] = (int32_t)pos;
    pos += chunk_nbytes[c];
  }
  if (pos + 8 > out_capacity) return set_err("aib_pack_chunks: output buffer too small");
  std::memset(out + pos, 0, 8);
  int64_t c;
#pragma omp parallel for schedule(static)
  for (c = 0; c < n_chunks; ++c) {
    const int64_t a = c * chunk_size, b = std::min(a + chunk_size, n);
    uint8_t *dst = out + chunk_offsets[c];
    uint64_t acc = 0;
    int nbits = 0;
    int64_t w = 0;
    for (int64_t i = a; i < b; ++i) {
      const int s = symbols[i];
      const int ln = lengths[s];
      acc |= uint64_t(codes[s]) << (64 - nbits - ln);
      nbits += ln;
      while (nbits >= 8) {
        dst[w++] = uint8_t(acc >> 56);
        acc <<= 8;
        nbits -= 8;
      }
    }
    if (nbits > 0) dst[w++] = uint8_t(acc >> 56);
  }
  return AIB_OK;
}

AIB_API int aib_host_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
