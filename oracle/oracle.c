/*
 * CPU ORACLE -- test infrastructure only, never part of the product path.
 *
 * A plain-C restatement of Afterimage's reference decode algorithm for the
 * lossless BF16 weight-decode path. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg load this library, and only as the checker
 * (or, in bench.py, as the timed CPU baseline). The CUDA product path never
 * links or calls it.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks every function here
 * against golden vectors produced by running the reference's own encoder and
 * decoders (tests/golden/make_golden.py).
 *
 * Functions and the reference code each one restates (paths are within the
 * Afterimage project):
 *   orc_decode_chunk       afterimage/runtime/huffman_chunked.py:210-253
 *                          (ChunkedBitReader._refill / decode_one,
 *                          decode_chunk_reference): 32-bit MSB-aligned
 *                          buffer, one-byte refills while fewer than
 *                          max_bits bits are valid and the chunk has bytes
 *                          left, window = buf >> (32 - max_bits).
 *   orc_decode_chunks      afterimage/runtime/cpu_decode.py:67-113
 *                          (_decode_numba / decode_chunks_numba): the same
 *                          reader over chunks [c_lo, c_hi), bounded by each
 *                          chunk's own [offset, offset + nbytes), parallel
 *                          over chunks (numba prange -> OpenMP).
 *   orc_recombine          afterimage/runtime/compressed_store.py:94-114
 *                          (_recombine): bf16 = sign<<15 | e<<7 | mantissa.
 *   orc_decompress_range   afterimage/runtime/compressed_store.py:186-240 and
 *                          :254-303 (decompress_layer_gpu with device="cpu",
 *                          decompress_rows_gpu): decode the covering chunks
 *                          of an element range and recombine it with the
 *                          sign/mantissa bytes.
 */
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Decode one chunk: chunk_size symbols from bytes [0, nbytes). Matches
 * ChunkedBitReader exactly, including reading zeros once the chunk's bytes
 * are exhausted (the reader stops refilling at the chunk end). */
static void decode_chunk(const uint8_t *bytes, int64_t nbytes,
                         const int32_t *sym_lut, const int8_t *len_lut,
                         int max_bits, int64_t n_out, uint8_t *out)
{
    uint32_t buf = 0;
    int nbits = 0;
    int64_t pos = 0;
    const uint32_t mask = (max_bits >= 32) ? 0xFFFFFFFFu : ((1u << max_bits) - 1u);
    for (int64_t i = 0; i < n_out; ++i) {
        while (nbits < max_bits && pos < nbytes) {
            buf |= (uint32_t)bytes[pos] << (24 - nbits);
            pos += 1;
            nbits += 8;
        }
        uint32_t window = max_bits == 0 ? 0u : ((buf >> (32 - max_bits)) & mask);
        int consumed = (int)len_lut[window];
        out[i] = (uint8_t)sym_lut[window];
        buf = consumed >= 32 ? 0u : (uint32_t)(buf << consumed);
        nbits -= consumed;
    }
}

/* Single chunk, all chunk_size symbols (decode_chunk_reference). */
void orc_decode_chunk(const uint8_t *bytes, int64_t nbytes,
                      const int32_t *sym_lut, const int8_t *len_lut,
                      int max_bits, int64_t chunk_size, uint8_t *out)
{
    decode_chunk(bytes, nbytes, sym_lut, len_lut, max_bits, chunk_size, out);
}

/* Chunks [c_lo, c_hi) into out[(c - c_lo) * chunk_size ...], full chunk_size
 * symbols each (decode_chunks_numba; callers truncate to n_symbols). */
void orc_decode_chunks(const uint8_t *packed, const int32_t *chunk_offsets,
                       const int32_t *chunk_nbytes, const int32_t *sym_lut,
                       const int8_t *len_lut, int max_bits, int64_t chunk_size,
                       int64_t c_lo, int64_t c_hi, int n_threads, uint8_t *out)
{
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
    int64_t c;
#pragma omp parallel for schedule(static)
    for (c = c_lo; c < c_hi; ++c) {
        decode_chunk(packed + chunk_offsets[c], chunk_nbytes[c], sym_lut, len_lut,
                     max_bits, chunk_size, out + (c - c_lo) * chunk_size);
    }
}

/* _recombine: int16 bits = (e << 7) | (sm & 0x7F), minus 32768 when sm >= 128,
 * i.e. the sign bit lands in bit 15. Written on uint16 here. */
void orc_recombine(const uint8_t *exponent, const uint8_t *sign_mantissa,
                   int64_t n, uint16_t *out)
{
    for (int64_t i = 0; i < n; ++i) {
        uint16_t sm = sign_mantissa[i];
        out[i] = (uint16_t)(((uint16_t)exponent[i] << 7) | (sm & 0x7Fu) | ((sm & 0x80u) << 8));
    }
}

/* Elements [e0, e1) of a tensor: decode the covering chunks and recombine.
 * sign_mantissa is indexed by absolute element (the full tensor's bytes).
 * out receives e1 - e0 bf16 bit patterns. Work is split across threads by
 * chunk, each chunk decoded into a private stack buffer. */
void orc_decompress_range(const uint8_t *packed, const int32_t *chunk_offsets,
                          const int32_t *chunk_nbytes, const int32_t *sym_lut,
                          const int8_t *len_lut, int max_bits, int64_t chunk_size,
                          int64_t n_symbols, const uint8_t *sign_mantissa,
                          int64_t e0, int64_t e1, int n_threads, uint16_t *out)
{
    if (e1 > n_symbols) e1 = n_symbols;
    if (e1 <= e0 || chunk_size <= 0) return;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
    int64_t c_lo = e0 / chunk_size;
    int64_t c_hi = (e1 + chunk_size - 1) / chunk_size;
    int64_t c;
#pragma omp parallel
    {
        uint8_t local[4096];
        uint8_t *exp = local;
        uint8_t *heap = 0;
        if (chunk_size > (int64_t)sizeof(local)) {
            heap = (uint8_t *)__builtin_malloc((size_t)chunk_size);
            exp = heap;
        }
#pragma omp for schedule(static)
        for (c = c_lo; c < c_hi; ++c) {
            int64_t base = c * chunk_size;
            int64_t lo = base > e0 ? base : e0;
            int64_t hi = base + chunk_size < e1 ? base + chunk_size : e1;
            /* decode only as far as this range needs; the reader is
             * sequential so the prefix [base, hi) is always decoded */
            decode_chunk(packed + chunk_offsets[c], chunk_nbytes[c], sym_lut, len_lut,
                         max_bits, hi - base, exp);
            for (int64_t g = lo; g < hi; ++g) {
                uint16_t sm = sign_mantissa[g];
                out[g - e0] = (uint16_t)(((uint16_t)exp[g - base] << 7) | (sm & 0x7Fu)
                                         | ((sm & 0x80u) << 8));
            }
        }
        if (heap) __builtin_free(heap);
    }
}

int orc_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
