/*
 * afterimage_b200 -- C ABI of the B200 lossless BF16 weight-decode library
 * (libafterimage_b200.so).
 *
 * The library replaces Afterimage's weight-reconstruction hot path: the
 * chunked canonical-Huffman decode of BF16 exponent streams, merged with the
 * raw (sign << 7) | mantissa bytes back into bit-identical BF16 weights.
 * Every entry point takes plain pointers and sizes; device pointers are CUDA
 * global-memory addresses on the current device, `stream` is a cudaStream_t
 * (NULL = legacy default stream). Work is enqueued on `stream` and nothing
 * synchronises unless the entry point says so. No entry point allocates
 * device memory: callers own every buffer.
 *
 * Status: every function returns AIB_OK (0) or a nonzero AIB_E* code; the
 * calling thread's message is available from aib_last_error().
 *
 * References are paths within the Afterimage project (afterimage-llm 0.3.0).
 */
#ifndef AFTERIMAGE_B200_H
#define AFTERIMAGE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AIB_OK 0
#define AIB_EINVAL 1 /* bad argument: caught on the host before any launch */
#define AIB_ECUDA 2  /* a CUDA runtime call failed */
#define AIB_EIO 3    /* a host read failed */
#define AIB_ESHORT 4 /* a host read ended before the requested bytes (end of file) */

/* Bits the decode kernels OR into the optional device status word. */
#define AIB_STATUS_BAD_CHUNK_RANGE 1 /* a chunk's [offset, offset + nbytes) lies outside packed */
#define AIB_STATUS_LUT_NOT_PREFIX 2  /* tables: LUT is not a prefix-code table; decoded exactly via the slow path */
#define AIB_STATUS_LUT_RANGE 4       /* tables: a symbol outside [0, 255] or a length outside [0, max_bits] */
#define AIB_STATUS_WAIT_TIMEOUT 8    /* a bounded wait on a bulk copy gave up; the CTA returned early */
#define AIB_STATUS_PEER_TIMEOUT 16   /* all-reduce: a bounded wait for a peer's flag gave up */

/* Polls of the kernels' one device-side wait (the table's bulk copy, with a
 * short sleep between polls) before the CTA gives up with
 * AIB_STATUS_WAIT_TIMEOUT. */
#define AIB_WAIT_LIMIT_POLLS (1u << 22)

/* Thread-local message for the last failing call on this thread (the
 * library's error channel; no counterpart in the reference). */
const char *aib_last_error(void);
/* ABI version: bump on any signature change. */
int aib_abi_version(void);

/* ------------------------------------------------------------------------
 * Encoder (host). Byte-identical to the reference encoder.
 * ------------------------------------------------------------------------ */

/* Field split of compress_layer (afterimage/runtime/compressed_store.py:78-88):
 * exponent[i] = (bits >> 7) & 0xFF, sign_mantissa[i] = ((bits >> 15) & 1) << 7 | (bits & 0x7F). */
int aib_split_bf16(const uint16_t *bits, int64_t n, uint8_t *exponent, uint8_t *sign_mantissa);
/* np.bincount(symbols, minlength=256) (afterimage/runtime/huffman_chunked.py:159). */
int aib_histogram(const uint8_t *symbols, int64_t n, int64_t counts[256]);
/* build_lengths + canonical_codes (afterimage/runtime/huffman.py:41-125):
 * natural Huffman depths (heapq tie-breaking), package-merge when deeper than
 * max_bits_limit, canonical code assignment. *max_bits_out = longest code. */
int aib_build_code(const int64_t counts[256], int max_bits_limit, int32_t lengths_out[256],
                   uint32_t codes_out[256], int32_t *max_bits_out);
/* build_decode_lut (afterimage/runtime/huffman.py:128-150): 2^max_bits entries. */
int aib_build_decode_lut(const int32_t lengths[256], const uint32_t codes[256], int max_bits,
                         int32_t *sym_lut, int8_t *len_lut);
/* First packing pass (afterimage/runtime/huffman_chunked.py:41-78): bytes per chunk. */
int aib_chunk_nbytes(const uint8_t *symbols, int64_t n, int64_t chunk_size,
                     const int32_t lengths[256], int32_t *chunk_nbytes, int64_t *total_bytes);
/* Second packing pass + offsets + 8-byte zero tail
 * (afterimage/runtime/huffman_chunked.py:41-98, :178-201). */
int aib_pack_chunks(const uint8_t *symbols, int64_t n, int64_t chunk_size,
                    const int32_t lengths[256], const uint32_t codes[256],
                    const int32_t *chunk_nbytes, int32_t *chunk_offsets, uint8_t *out,
                    int64_t out_capacity);
/* Host threads the encoder uses (OpenMP); a utility with no counterpart in
 * the reference. */
int aib_host_threads(void);

/* ------------------------------------------------------------------------
 * Store reads -- the extents of BinaryWeightReader.read_many
 * (afterimage/runtime/binstore.py:109-192)
 * ------------------------------------------------------------------------ */
/* Replaces the extent reads of BinaryWeightReader.read_many
 * (afterimage/runtime/binstore.py:109-192).
 * n positional reads of file descriptor fd: piece i fills dests[i] with
 * sizes[i] bytes from offsets[i]. `threads` host threads read pieces
 * concurrently; *bytes_read receives the bytes read. If min_sizes is not
 * NULL, a piece that reaches end of file after min_sizes[i] bytes is
 * complete (O_DIRECT reads round their size up past the end of the file).
 * Returns AIB_ESHORT if the file ends early, AIB_EIO for a read error
 * (the message names the piece). Works with O_DIRECT descriptors when
 * offsets, sizes and dests meet its alignment. */
int aib_pread_batch(int fd, const int64_t *offsets, const int64_t *sizes, const int64_t *min_sizes,
                    void *const *dests, int64_t n, int threads, int64_t *bytes_read);

/* ------------------------------------------------------------------------
 * Decode tables -- replaces prepare_decode_tables
 * (afterimage/runtime/gpu_decode_v2.py:71-76).
 * ------------------------------------------------------------------------ */

/* Size in bytes of one device table block (16-byte aligned buffer). */
size_t aib_tables_bytes(void);
/* Builds a tensor's table block from its reference LUTs, already on the
 * device (sym_lut int32[2^max_bits], len_lut int8[2^max_bits]). The block
 * holds a multi-symbol first-level table for shared memory plus validation
 * flags; the decode kernels also read d_sym_lut / d_len_lut for codes longer
 * than the first level, so those must stay alive while decoding.
 * 0 <= max_bits <= 16. Stream-ordered; no synchronisation. */
int aib_build_tables(const int32_t *d_sym_lut, const int8_t *d_len_lut, int max_bits,
                     void *d_tables, void *stream);
/* Copies the block's validation flags (AIB_STATUS_LUT_*) to *flags_out;
 * synchronises `stream`. */
int aib_tables_flags(const void *d_tables, int32_t *flags_out, void *stream);

/* ------------------------------------------------------------------------
 * Decode. One descriptor names one tensor's compressed stream and the
 * element range [elem_begin, elem_end) to produce.
 * ------------------------------------------------------------------------ */
typedef struct aib_stream_desc {
  const uint8_t *packed;        /* device; 16-byte aligned; readable for packed_capacity bytes */
  int64_t packed_capacity;      /* readable bytes at packed: multiple of 16, >= packed_nbytes */
  int64_t packed_nbytes;        /* bytes of real stream data (chunk ranges are checked against it) */
  int64_t offset_base;          /* chunk c starts at packed + chunk_offsets[c] - offset_base */
  const int32_t *chunk_offsets; /* device; entry c - chunk_base is chunk c's byte offset */
  const int32_t *chunk_nbytes;  /* device; entry c - chunk_base is chunk c's byte count */
  int64_t chunk_base;           /* first chunk the two arrays above describe (0 = whole tensor) */
  const void *tables;           /* device table block from aib_build_tables */
  const int32_t *sym_lut;       /* device, int32[2^max_bits] */
  const int8_t *len_lut;        /* device, int8[2^max_bits] */
  int32_t max_bits;             /* 0..16, as stored with the tensor */
  int32_t chunk_size;           /* symbols per chunk, >= 1 */
  int64_t n_symbols;            /* symbols in the whole tensor */
  int64_t elem_begin;           /* first element produced (0 <= elem_begin <= elem_end) */
  int64_t elem_end;             /* one past the last element (<= n_symbols) */
  const uint8_t *sign_mantissa; /* device; element elem_begin at index 0 (bf16 decode only) */
  void *out;                    /* device; element elem_begin at index 0 */
  const int64_t *stripe_base;   /* NULL: `packed` holds the reference stream (chunk c at
                                   packed + chunk_offsets[c - chunk_base] - offset_base).
                                   Non-NULL: `packed` holds the striped layout that
                                   aib_stripe_stream writes and entry g - chunk_base / 32 is
                                   the first 16-byte block of chunk group g; chunk_base is then
                                   a multiple of 32, chunk_offsets and offset_base are unused
                                   and packed_nbytes is the striped size. */
} aib_stream_desc;

/* Striped resident layout (no counterpart in the reference, which reads
 * each chunk's bytes where the encoder put them). Chunks are taken in groups
 * of 32 (group g = chunks 32g .. 32g + 31); in a group's region the 16-byte
 * block i of the chunk in column l (= c mod 32) is block i * 32 + l, so the
 * 32 lanes of a decoding warp, one chunk each, read 512 consecutive bytes per
 * step instead of 32 scattered 16-byte blocks. A group's region has as many
 * rows as its longest chunk has blocks; blocks past a chunk's end are zero.
 * The stream is the same bits; only the bytes' places differ.
 *
 * aib_stripe_layout (host): from the chunks' byte counts (host int32[n_chunks])
 * writes group_base[g] = the region's first block for g in
 * [0, ceil(n_chunks / 32)] (the last entry is the total) and returns that
 * total in *total_blocks. */
int aib_stripe_layout(const int32_t *chunk_nbytes, int64_t n_chunks, int64_t *group_base, int64_t *total_blocks);
/* aib_stripe_stream (device, stream-ordered): writes the striped copy of the
 * reference stream `src` (chunks [chunk_base, chunk_base + n_chunks) described
 * as in aib_stream_desc; chunk_base a multiple of 32) into dst (16-byte
 * aligned, dst_nbytes >= 16 * group_base[last], a multiple of 16). group_base
 * is the device copy of aib_stripe_layout's array. A chunk whose bytes lie
 * outside src_nbytes, or a group region outside dst, sets
 * AIB_STATUS_BAD_CHUNK_RANGE in d_status (optional); such a chunk is written
 * as zeros and such a region not at all. */
int aib_stripe_stream(const uint8_t *src, int64_t src_nbytes, int64_t offset_base, const int32_t *chunk_offsets,
                      const int32_t *chunk_nbytes, int64_t chunk_base, int64_t n_chunks,
                      const int64_t *group_base, uint8_t *dst, int64_t dst_nbytes, int32_t *d_status,
                      void *stream);

/* aib_stripe_stream_host: the same striped copy made on the host (for
 * images that are built on the host and copied whole), chunk c of the
 * arrays at src + chunk_offsets[c] - offset_base. Returns AIB_EINVAL when
 * dst is smaller than 16 * group_base[last] (nothing written), or at the
 * first group with a bad region or a chunk that lies outside src or does
 * not fit its region (dst then holds the groups before it). */
int aib_stripe_stream_host(const uint8_t *src, int64_t src_nbytes, int64_t offset_base,
                           const int32_t *chunk_offsets, const int32_t *chunk_nbytes, int64_t n_chunks,
                           const int64_t *group_base, uint8_t *dst, int64_t dst_nbytes);

/* Fused decode + recombine: out (uint16 bf16 bits) = the reference's
 * decompress output for elements [elem_begin, elem_end). Replaces the
 * decode + _recombine pair of decompress_layer_gpu / decompress_rows_gpu
 * (afterimage/runtime/compressed_store.py:186-240, :254-303, :94-114).
 * d_status (optional, device int32) accumulates AIB_STATUS_* bits. */
int aib_decode_bf16(const aib_stream_desc *desc, int32_t *d_status, void *stream);

/* Exponent-only decode to uint8: replaces the _huffman_decode_kernel_v2
 * launch of decode_gpu_v2 (afterimage/runtime/gpu_decode_v2.py:27-68, :107-114). */
int aib_decode_exponents_u8(const aib_stream_desc *desc, int32_t *d_status, void *stream);

/* Exponent-only decode to int32: replaces the _huffman_decode_kernel launch
 * of decode_gpu (afterimage/runtime/gpu_decode.py:26-58, :61-75). */
int aib_decode_exponents_i32(const aib_stream_desc *desc, int32_t *d_status, void *stream);

/* Several tensors in one launch (a decoder layer's projections): replaces
 * the per-tensor _decode_tensor loop of the layer streamer
 * (afterimage/runtime/streaming_engine.py:1834-1842, :1074-1138).
 * 1 <= count <= AIB_MAX_BATCH. */
#define AIB_MAX_BATCH 16
int aib_decode_bf16_batch(const aib_stream_desc *descs, int count, int32_t *d_status, void *stream);
/* The same launch on at most max_ctas CTAs (>= 1; one CTA holds one SM; a
 * job still gets at least one CTA). The decode then leaves SMs to kernels
 * of other streams: the tensor-parallel decoder decodes layer i + 1 on a
 * side stream this way while layer i's projections run. No counterpart in
 * the reference, which decodes and multiplies one after the other. */
int aib_decode_bf16_batch_ctas(const aib_stream_desc *descs, int count, int max_ctas, int32_t *d_status,
                               void *stream);

/* Fused decode -> GEMV for one input vector (a single-token projection):
 * y = W x with W given only in compressed form. `stream` describes the
 * tensor as for the decode; its element range must be whole rows of the
 * row-major [rows, cols] matrix (elem_begin and elem_end multiples of
 * cols), cols a multiple of chunk_size, chunk_size a multiple of 4,
 * sign_mantissa 4-byte aligned;
 * stream.out is ignored and stream.stripe_base must be NULL (its lanes
 * read chunks a row apart, not 32 neighbours). Replaces, for M = 1, the decode followed by the
 * consuming nn.Linear / F.linear on the decoded weights
 * (afterimage/runtime/streaming_engine.py:1871-1915 layer hooks around the
 * transformers decoder layer; the chunked head's F.linear, :2330). */
typedef struct aib_gemv_desc {
  aib_stream_desc stream;
  int64_t cols;       /* row length */
  const void *x;      /* device bf16[cols], 8-byte aligned */
  float *partial;     /* device scratch: (elem_end - elem_begin) / chunk_size floats */
  void *y;            /* device bf16[(elem_end - elem_begin) / cols] */
} aib_gemv_desc;

/* Replaces, for one token, a layer's decode followed by the nn.Linear /
 * F.linear that consumes it (afterimage/runtime/streaming_engine.py:1871-1915,
 * :2330): y = W x with W read only in compressed form.
 * Up to AIB_MAX_BATCH GEMVs (each with its own x) in one launch pair: the
 * decode-and-multiply kernel writes one fp32 partial per chunk, a second
 * kernel sums each row's partials in column order and rounds to BF16
 * (deterministic). Work is enqueued on `stream`; no synchronisation. */
int aib_decode_gemv_bf16_batch(const aib_gemv_desc *descs, int count, int32_t *d_status, void *stream);

/* The same fused decode -> GEMV for callers that cannot allocate device
 * memory: it has no counterpart in the reference. Such callers hold only
 * the device pointers someone else gave them -- a binding from another host
 * language that is handed buffers by the framework owning the memory, or a
 * caller under a framework whose allocator must account for every byte, so
 * a side cudaMalloc would break its budget. The caller passes the stream
 * descriptors, x and y as for aib_decode_gemv_bf16_batch; descs[i].partial
 * is ignored, and the per-chunk partial sums go to a fixed array inside the
 * library instead (AIB_GEMV_SCRATCH_FLOATS floats, 4 MiB, held by every
 * GPU that loads the library until the process exits). Each descriptor's
 * share starts 256-byte aligned, so a batch needs the sum over descriptors
 * of ceil(chunks / 64) * 64 floats; a batch needing more than the array
 * returns AIB_EINVAL before touching the device; nothing is allocated. The
 * first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and caches it: make that first call before any
 * stream capture. The cached address is not refreshed if the device is
 * reset (cudaDeviceReset) or its context is recreated later in the
 * process; do not call this entry point after that. The array is shared by every call of the process on
 * that device and keeps the last call's contents (nothing in it needs to
 * start at zero: each call writes every partial it reads); two calls that
 * overlap on the GPU -- different streams, no ordering between them --
 * race on it and corrupt each other's results. */
#define AIB_GEMV_SCRATCH_FLOATS (1 << 20)
int aib_decode_gemv_bf16_batch_noalloc(const aib_gemv_desc *descs, int count, int32_t *d_status, void *stream);

/* ------------------------------------------------------------------------
 * Single-token step of the tensor-parallel decoder: the small operations
 * between a layer's projections, fused. They replace the layer math the
 * reference runs in transformers' Qwen3 / Llama modules around its hooks
 * (afterimage/runtime/streaming_engine.py:1871-1915), with the same BF16
 * rounding points. Row-major BF16 (uint16 bits), work on `stream`.
 * ------------------------------------------------------------------------ */
/* x <- bf16(x + delta) when delta is not NULL (in place), then
 * out = bf16(weight * bf16(x * rsqrt(mean(x^2) + eps))) per row. */
int aib_add_rmsnorm_bf16(void *x, const void *delta, const void *weight, void *out, int64_t rows, int64_t cols,
                         float eps, void *stream);
/* qkv [T, (nh + 2 nkv) * hd]: per-head RMSNorm of q and k (when both norm
 * weights are given), rotary embedding at positions *pos0 + t (rotate-half,
 * cos/sin of pos * inv_freq rounded to BF16); q -> q_out [nh, T, hd],
 * k and v -> k_cache / v_cache [nkv, max_len, hd] at those positions. */
int aib_qk_rope_cache_bf16(const void *qkv, int T, int nh, int nkv, int hd, const void *q_norm_w,
                           const void *k_norm_w, float eps, const float *inv_freq, const int64_t *pos0, void *q_out,
                           void *k_cache, void *v_cache, int64_t max_len, void *stream);
/* One query per head (q [nh, hd]) over cache positions [0, *pos]; kv head =
 * head / (nh / nkv); out [nh * hd]. max_len <= 8192. */
int aib_decode_attention_bf16(const void *q, const void *k_cache, const void *v_cache, int nh, int nkv, int hd,
                              int64_t max_len, const int64_t *pos, float scale, void *out, void *stream);
/* gate_up [T, 2I] (gate then up per row) -> out [T, I] = bf16(bf16(silu(gate)) * up). */
int aib_silu_mul_bf16(const void *gate_up, void *out, int64_t T, int64_t I, void *stream);

/* Y[i, r] = sum_j X[i, j] * W[r, j] for i < m (1..8 tokens), r < n, j < k:
 * the projections that consume a decoded layer when few tokens pass
 * through it (a greedy step; the k + 1 tokens of a speculative verification).
 * Replaces, for these shapes, the nn.Linear / F.linear the reference calls
 * on decoded weights (afterimage/runtime/streaming_engine.py:1871-1915,
 * :2330). W row-major [n, k] with row stride ldw, X [m, k] with row stride
 * ldx (BF16, 16-byte aligned, k, ldw and ldx multiples of 8); Y [m, n] with
 * row stride ldy, BF16 (rounded once from the fp32 sum) or fp32 when
 * out_fp32 is set. Work is enqueued on `stream`. */
int aib_gemv_bf16(const void *w, int64_t ldw, const void *x, int64_t ldx, void *y, int64_t ldy, int64_t n,
                  int64_t k, int m, int out_fp32, void *stream);

/* Y[i, r] = sum_j X[i, j] * W[r, j] for i < m (1..256 tokens, a prompt's
 * prefill), r < n, j < k, on the tensor cores (tcgen05.mma, fp32
 * accumulation in tensor memory, TMA-staged 128-byte-swizzled tiles). The
 * projections that consume a decoded layer for many tokens: replaces, for
 * these shapes, the nn.Linear the reference calls on decoded weights
 * (afterimage/runtime/streaming_engine.py:1871-1915). W row-major [n, k] with
 * row stride ldw, X [m, k] with row stride ldx (BF16, 16-byte aligned, row
 * strides multiples of 8, k a multiple of 64); Y [m, n] BF16 with row stride
 * ldy. When the 128-row tiles of W are too few to fill the GPU the K range is
 * split: then `workspace` must hold aib_gemm_bf16_tc_workspace_floats(m, n, k)
 * floats (0 when no split is needed). A bounded wait that gives up sets
 * AIB_STATUS_WAIT_TIMEOUT in *d_status. Work is enqueued on `stream`. */
int aib_gemm_bf16_tc(const void *w, int64_t ldw, const void *x, int64_t ldx, void *y, int64_t ldy, int64_t m,
                     int64_t n, int64_t k, float *workspace, int64_t workspace_floats, int32_t *d_status,
                     void *stream);
int64_t aib_gemm_bf16_tc_workspace_floats(int64_t m, int64_t n, int64_t k);

/* Elementwise recombine of an already-decoded exponent field: replaces
 * recombine_exponent_and_sign_mantissa / _recombine
 * (afterimage/runtime/compressed_store.py:94-130). */
int aib_recombine(const uint8_t *exponent, const uint8_t *sign_mantissa, int64_t n, uint16_t *out,
                  void *stream);

/* Self-test of the bounded device wait; it has no counterpart in the
 * reference. One CTA waits on an mbarrier that nothing completes, gives up
 * after `polls` polls (1..AIB_WAIT_LIMIT_POLLS) and ORs
 * AIB_STATUS_WAIT_TIMEOUT into *d_status, as a table copy that never lands
 * would. No copy is issued, so nothing outlives the CTA. Enqueued on
 * `stream`; no synchronisation. */
int aib_selftest_wait_timeout(unsigned polls, int32_t *d_status, void *stream);

/* ------------------------------------------------------------------------
 * One-shot all-reduce over NVLink peer memory (tensor-parallel decoder:
 * the row-parallel o_proj / down_proj partial sums). The reference runs on
 * one GPU and has no counterpart; this replaces the NCCL all-reduce the
 * tensor-parallel decoder would otherwise make.
 *
 * Each rank allocates one buffer (aib_ar_alloc), shares its IPC handle
 * (aib_ar_ipc_handle, AIB_AR_HANDLE_BYTES bytes) with the other ranks of
 * the node, opens theirs (aib_ar_ipc_open) and fills an aib_ar_group with
 * every rank's buffer as mapped in this process. After a host barrier (the
 * buffers start zeroed) every rank makes the same aib_allreduce_oneshot_f32
 * calls in the same order: out = sum over ranks of in, fp32, added in rank
 * order, so every rank gets bit-identical sums. in == out is allowed.
 * Stream-ordered. A wait for a peer polls at most max_polls times (with
 * backoff); when it gives up it sets AIB_STATUS_PEER_TIMEOUT in *d_status
 * and the group must not be used again. Ranks of one group must run on
 * different GPUs.
 * ------------------------------------------------------------------------ */
#define AIB_AR_MAX_RANKS 8
#define AIB_AR_MAX_CTAS 64
#define AIB_AR_HANDLE_BYTES 64
typedef struct aib_ar_group {
  void *buffers[AIB_AR_MAX_RANKS]; /* rank p's buffer as mapped here; [rank] is this rank's own */
  int32_t rank;
  int32_t world;                   /* 1 .. AIB_AR_MAX_RANKS */
  int64_t max_floats;              /* the capacity every buffer was allocated with */
} aib_ar_group;
/* 4 KiB + 2 x AIB_AR_MAX_RANKS x 8 bytes x max_floats: every element
 * travels as one 64-bit (value, call number) word per rank and parity. */
size_t aib_ar_buffer_bytes(int64_t max_floats);
/* cudaMalloc of aib_ar_buffer_bytes(max_floats) on the current device,
 * zeroed; synchronises the device. */
int aib_ar_alloc(int64_t max_floats, void **d_buffer);
int aib_ar_free(void *d_buffer);
int aib_ar_ipc_handle(void *d_buffer, void *handle_out);
int aib_ar_ipc_open(const void *handle, void **d_peer);
int aib_ar_ipc_close(void *d_peer);
/* CTAs a call of n floats uses. */
int aib_ar_ctas(int64_t n);
int aib_allreduce_oneshot_f32(const aib_ar_group *g, const float *in, float *out, int64_t n, unsigned max_polls,
                              int32_t *d_status, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* AFTERIMAGE_B200_H */
