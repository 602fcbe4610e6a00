/*
 * cbq.h -- C ABI of the B200 codebook decode-matmul library (libcbq.so).
 *
 * Computes out = x @ W^T where W[r,k] = codebook[min(idx(r*K+k), C-1)] is
 * never materialised: every call reads the compressed index stream itself.
 * Two stream formats are accepted, both byte-for-byte the reference's
 * on-disk `.npz` payloads (bigattichouse/Codebook-Quantization):
 *
 *   fixed width  `indices`: LSB-first, b bits per index (src/bitpack.py:32-94)
 *   Huffman      `huff_stream` + `huff_lengths` + `huff_row_bit_starts`:
 *                MSB-first canonical codes (src/huffman_codebook.py:126-226)
 *
 * Conventions
 *   - Every pointer named *_dev is device memory; sizes are int64_t.
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued there and
 *     the call returns without synchronising.
 *   - Return value: CBQ_OK or a CBQ_ERR_* code (argument errors are detected
 *     on the host before any launch).  Errors found while decoding (a code
 *     that matches no symbol, a row that ends where the next does not start,
 *     a wait that timed out) are recorded in the optional device status word
 *     `status_dev` (uint32_t[4], see CBQ_STATUS_*), which the caller zeroes
 *     and reads back when it chooses.  No kernel traps.
 *   - dtype codes: CBQ_F32 or CBQ_BF16 for activations and outputs; the
 *     codebook is always fp32 and accumulation is always fp32.
 *   - Handles do not exist: callers own every buffer.  Buffers that the
 *     kernels read past their logical end must be allocated with the sizes
 *     the *_bytes() queries return (zero-filled padding) and be 16-byte
 *     aligned.
 *
 * The functions replace the reference's GPU entry points (paths relative
 * to the reference project root):
 *   fused_compressed_linear     src/gpu_accelerated_functions.py:238-274
 *   fused_compressed_embedding  src/gpu_accelerated_functions.py:276-307
 *   huffman_decode_to_i32 + huffman_i32_linear
 *                               src/gpu_huffman_functions.py:297-370
 *   huffman_decode_to_i32 + huffman_i32_embedding
 *                               src/gpu_huffman_functions.py:372-405
 * and follow the status-code style of the reference's HIP C ABI
 * (rocm/compressed_kernel.h:37-39, rocm/compressed_kernel.hip:607-616).
 */
#ifndef CBQ_H
#define CBQ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (rocm/compressed_kernel.h:37-39 has 0/1/2) ---- */
#define CBQ_OK              0
#define CBQ_ERR_CUDA        1   /* a CUDA runtime call failed */
#define CBQ_ERR_ARG         2   /* invalid argument (checked on the host) */
#define CBQ_ERR_CORRUPT     3   /* decode error recorded in a status word */
#define CBQ_ERR_TIMEOUT     4   /* a bounded device wait gave up */
#define CBQ_ERR_UNSUPPORTED 5   /* shape/format outside what the kernels accept */

/* ---- device status word layout: uint32_t status_dev[4] ---- */
#define CBQ_STATUS_FLAGS     0  /* OR of CBQ_FLAG_* */
#define CBQ_STATUS_FIRST_ROW 1  /* smallest row index with an error (init 0xffffffff) */
#define CBQ_STATUS_COUNT     2  /* number of decode errors */
#define CBQ_FLAG_CORRUPT  1u    /* a Huffman code matched no symbol (reference emits symbol 0, advances 1 bit) */
#define CBQ_FLAG_ROW_END  2u    /* a row's decoded end != next row's start */
#define CBQ_FLAG_TIMEOUT  4u    /* an mbarrier wait exceeded its bound */
#define CBQ_FLAG_SPAN     8u    /* a tile's stream span exceeded the staging buffer */

/* ---- dtypes ---- */
#define CBQ_F32  0
#define CBQ_BF16 1

const char *cbq_status_string(int status);
int cbq_version(void);

/* ======================================================================
 * Fixed-width streams
 * ====================================================================== */

/* Device bytes to allocate for an M x K, `bits`-wide stream: the on-disk
 * ceil(M*K*bits/8) bytes plus zero padding the kernels may read.  The
 * reference pads +4 bytes on the GPU (src/gpu_accelerated_functions.py:860-864). */
int64_t cbq_fixed_stream_bytes(int64_t M, int64_t K, int bits);

/* Workspace bytes cbq_linear_fixed may use for an M x K matrix and T tokens
 * (rows split between warps leave piece sums and an arrival counter there).
 * The caller zero-fills it once; every call leaves it zeroed again. */
int64_t cbq_linear_fixed_workspace_bytes(int64_t M, int64_t K, int64_t T);

/* out[t, r] = sum_k x[t, k] * codebook[min(idx(r*K + k), C-1)] (+ bias[r]).
 * Replaces fused_compressed_linear (src/gpu_accelerated_functions.py:238-274)
 * and ck_linear_f32 (rocm/compressed_kernel.hip:607-616).
 *   x_dev      [T, ldx] rows of K activations, dtype x_dtype
 *   packed_dev fixed-width stream, packed_bytes >= cbq_fixed_stream_bytes()
 *   codebook_dev fp32[C], C >= 1;  bits in [1, 16]
 *   bias_dev   fp32[M] or NULL
 *   out_dev    [T, ldo] rows of M outputs, dtype out_dtype (overwritten)
 *   workspace_dev  NULL, or a zero-filled buffer of at least
 *              cbq_linear_fixed_workspace_bytes(M, K, T) bytes: lets the
 *              kernel balance work at 1024-index granularity instead of
 *              whole rows.  Every call leaves it zero-filled, so calls of
 *              any shape may share it; calls sharing one workspace must not
 *              overlap on the GPU (the same stream is fine). */
int cbq_linear_fixed(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                     const uint8_t *packed_dev, int64_t packed_bytes,
                     const float *codebook_dev, int64_t C, int bits,
                     int64_t M, int64_t K, const float *bias_dev,
                     void *out_dev, int out_dtype, int64_t ldo,
                     void *workspace_dev, int64_t workspace_bytes, void *stream);

/* Epilogues of cbq_linear_fixed_multi. */
#define CBQ_EPI_STORE     0   /* out[m] = x @ W[m]^T (+ bias[m]) */
#define CBQ_EPI_RESIDUAL  1   /* out[m] = resid[m] + round(x @ W[m]^T (+ bias[m])); resid may alias out */
#define CBQ_EPI_SILU_MUL  2   /* nmat == 2, equal M: out[0] = round(silu(round(x@W0^T)) * round(x@W1^T)) */

/* Several fixed-width matrices that share the activations, K, the bit width
 * and the codebook, decoded by one launch (for example q/k/v, or gate/up),
 * with an optional fused epilogue.  `round` is the rounding to out_dtype, so
 * each epilogue gives the same values as the separate operations: the
 * residual update `x + linear(h)` and the SiLU-gated product
 * `silu(gate(h)) * up(h)` of a transformer block (HF Qwen3 MLP).  No
 * counterpart in the reference, which launches one kernel per linear layer
 * (src/gpu_accelerated_functions.py:238-274) and does the rest in torch.
 * Host arrays (nmat entries): packed_dev, packed_bytes, M, bias_dev (array
 * may be NULL), out_dev, ldo, resid_dev (CBQ_EPI_RESIDUAL only).
 * Supports T <= 2 with 16-byte aligned x rows and streams, K % 128 == 0;
 * anything else returns CBQ_ERR_UNSUPPORTED before launching (the caller then
 * uses cbq_linear_fixed per matrix). */
int cbq_linear_fixed_multi(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat,
                           const uint8_t *const *packed_dev, const int64_t *packed_bytes,
                           const int64_t *M, const float *codebook_dev, int64_t C, int bits,
                           int64_t K, const float *const *bias_dev, void *const *out_dev,
                           const int64_t *ldo, const void *const *resid_dev, int out_dtype,
                           int epilogue, void *stream);

/* cbq_linear_fixed_multi with the RMSNorm that precedes the linear layers
 * applied to the activations as they are loaded: x is the un-normalised
 * residual stream, and every CTA computes rsqrt(mean(x[t]^2) + eps) of each
 * token row over K itself, then uses round(w[k] * round(x[t,k] * scale))
 * (HF Qwen3RMSNorm; round = the activation dtype; norm_weight_dev fp32 [K]
 * or NULL for unit weights).  One launch replaces a norm launch and the
 * GEMV.  Same support rules as cbq_linear_fixed_multi (T <= 2, else
 * CBQ_ERR_UNSUPPORTED before launching).  No counterpart in the reference. */
int cbq_linear_fixed_multi_norm(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat,
                                const uint8_t *const *packed_dev, const int64_t *packed_bytes, const int64_t *M,
                                const float *codebook_dev, int64_t C, int bits, int64_t K,
                                const float *const *bias_dev, void *const *out_dev, const int64_t *ldo,
                                const void *const *resid_dev, int out_dtype, int epilogue,
                                const float *norm_weight_dev, float eps, void *stream);

/* cbq_linear_fixed_multi_norm whose input is the tensor-parallel all-reduce
 * of the row-parallel layer before it (the consumer of
 * cbq_linear_fixed_peer): every CTA waits, bounded (2 s; CBQ_FLAG_TIMEOUT in
 * status_dev, after which later calls do not wait), until
 * local_counts_dev[s] >= *epoch_dev * expect for every rank s < world, then
 * forms x[t] = round(resid_in[t] + round(sum_s slot_s[t])) in rank order
 * (slot s row t at local_slots_dev + (s * T + t) * K elements), writes it to
 * x_dev (the updated residual stream; resid_in_dev is a different buffer,
 * same ldx) and runs the normalised GEMV on it.  One launch replaces the
 * all-reduce consumer, the RMSNorm and the GEMV.  With local_counts_dev NULL
 * the slots are in the flagged form of cbq_linear_fixed_peer_flagged (slot s
 * at local_slots_dev + s * T * K/2 words for bf16, s * T * K words for fp32;
 * expect unused): each CTA reads the words until they carry *epoch_dev
 * (bounded likewise), with no counter and no fence.  No counterpart in the
 * reference (single device). */
int cbq_linear_fixed_multi_allreduce_norm(
    const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat, const uint8_t *const *packed_dev,
    const int64_t *packed_bytes, const int64_t *M, const float *codebook_dev, int64_t C, int bits, int64_t K,
    const float *const *bias_dev, void *const *out_dev, const int64_t *ldo, const void *const *resid_dev,
    int out_dtype, int epilogue, const float *norm_weight_dev, float eps, int world, const void *resid_in_dev,
    const void *local_slots_dev, const uint32_t *local_counts_dev, const uint32_t *epoch_dev, int64_t expect,
    uint32_t *status_dev, void *stream);

/* cbq_linear_fixed_peer with flagged slots instead of counters: every
 * output is stored into rank p's slot (slot_dev[p], 8-byte aligned) as a
 * 64-bit word holding 32 bits of data (two bf16 rows (row, row + 1) at word
 * t * ldo/2 + row/2, or one fp32 row at word t * ldo + row) and *epoch_dev in
 * its high 32 bits, with one relaxed system-scope store, so the consumer
 * (cbq_linear_fixed_multi_allreduce_norm with local_counts_dev NULL) knows a
 * word is this step's by its epoch alone.  bf16 needs even M and ldo (else
 * CBQ_ERR_UNSUPPORTED).  The epoch grows by one per use of a slot; slots start
 * zeroed.  No counterpart in the reference (single device). */
int cbq_linear_fixed_peer_flagged(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, const uint8_t *packed_dev,
                                  int64_t packed_bytes, const float *codebook_dev, int64_t C, int bits, int64_t M,
                                  int64_t K, const float *bias_dev, int world, void *const *slot_dev,
                                  const uint32_t *epoch_dev, int64_t ldo, int out_dtype, void *stream);

/* Tensor-parallel row-parallel layer (o_proj, down_proj), fused with the
 * data movement of its all-reduce: the GEMV of this rank's K-block writes its
 * partial product [T, M] into every rank's slot for this rank
 * (slot_dev[p]: device pointer into rank p's memory, e.g. a symmetric
 * buffer, world <= 8), then each CTA adds its row count to every rank's
 * arrival counter for this rank (count_dev[p], system-scope release), so the
 * counters grow by M per call.  cbq_rmsnorm_allreduce is the consumer.  No
 * counterpart in the reference (single device).  Host arrays of world
 * pointers; T <= 2 and the alignment rules of cbq_linear_fixed_multi, else
 * CBQ_ERR_UNSUPPORTED before launching. */
int cbq_linear_fixed_peer(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                          const uint8_t *packed_dev, int64_t packed_bytes, const float *codebook_dev,
                          int64_t C, int bits, int64_t M, int64_t K, const float *bias_dev, int world,
                          void *const *slot_dev, uint32_t *const *count_dev, int64_t ldo, int out_dtype,
                          void *stream);

/* cbq_linear_fixed_peer followed, in the same launch, by what
 * cbq_rmsnorm_allreduce does: the CTA that finishes last (counted on
 * arrive_dev, a uint32 that is 0 before the call and left 0) waits, bounded,
 * until local_counts_dev[s] >= *epoch_dev * expect for every rank s, then
 * resid[t] = round(resid[t] + round(sum_s slot_s[t])) in rank order (slot s
 * row t at local_slots_dev + (s * T + t) * ldo elements) and norm_out[t] =
 * RMSNorm(resid[t]) with norm_weight_dev (may be NULL) and eps.  A wait that
 * gives up sets CBQ_FLAG_TIMEOUT in status_dev, after which later calls do
 * not wait.  One launch replaces the two of the unfused pair. */
int cbq_linear_fixed_peer_norm(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                               const uint8_t *packed_dev, int64_t packed_bytes, const float *codebook_dev,
                               int64_t C, int bits, int64_t M, int64_t K, const float *bias_dev, int world,
                               void *const *slot_dev, uint32_t *const *count_dev, int64_t ldo, int out_dtype,
                               const void *local_slots_dev, const uint32_t *local_counts_dev,
                               const uint32_t *epoch_dev, int64_t expect, void *resid_dev, int64_t ldr,
                               const float *norm_weight_dev, float eps, void *norm_out_dev, int64_t ldn,
                               uint32_t *arrive_dev, uint32_t *status_dev, void *stream);

/* cbq_linear_fixed_multi with CBQ_EPI_RESIDUAL for one matrix followed, in
 * the same launch, by cbq_rmsnorm of the updated rows: resid[t] +=
 * round(x[t] @ W^T (+ bias)) (resid [T, ldr], in place), then norm_out[t]
 * (stride ldn) = RMSNorm(resid[t]) with norm_weight_dev (may be NULL) and
 * eps, the values cbq_rmsnorm gives.  The CTA that finishes last (counted on
 * arrive_dev: 0 before the call, left 0) normalizes the rows.  T <= 2 and the
 * alignment rules of cbq_linear_fixed_multi, else CBQ_ERR_UNSUPPORTED before
 * launching. */
int cbq_linear_fixed_residual_norm(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                   const uint8_t *packed_dev, int64_t packed_bytes, const float *codebook_dev,
                                   int64_t C, int bits, int64_t M, int64_t K, const float *bias_dev,
                                   void *resid_dev, int64_t ldr, int out_dtype, const float *norm_weight_dev,
                                   float eps, void *norm_out_dev, int64_t ldn, uint32_t *arrive_dev,
                                   void *stream);

/* ---- host-resident streams (models whose packed indices exceed device memory) ----
 * The reference memory-maps flat .idx files (raw `indices` bytes) and runs its
 * CPU kernel on the mapping (src/compressed_matmul_cpu.py:23-63,
 * src/adaptive_compressor.py:1254-1316).  Here the stream stays in host
 * memory and is copied to the device in row chunks per call. */

/* Page-locks [host_ptr, host_ptr + bytes) for asynchronous copies
 * (cudaHostRegister; read_only != 0 for a read-only mapping such as a
 * memory-mapped .idx file, CBQ_ERR_UNSUPPORTED where the device cannot).
 * cbq_host_unregister undoes it. */
int cbq_host_register(void *host_ptr, int64_t bytes, int read_only);
int cbq_host_unregister(void *host_ptr);

/* Rows per chunk of cbq_linear_fixed_streamed for a staging buffer of
 * staging_bytes (two halves), or -1 (K % 128 != 0, or not one row fits). */
int64_t cbq_streamed_chunk_rows(int64_t M, int64_t K, int bits, int64_t staging_bytes);

/* cbq_linear_fixed with the packed stream in HOST memory (packed_host:
 * ceil(M*K*bits/8) bytes, pinned or registered for the copies to overlap).
 * Row chunks are copied into the two halves of staging_dev (device, 256-byte
 * aligned) on a copy stream of the library, each chunk's copy overlapping the
 * previous chunk's GEMV on `stream`; the GEMV of a chunk is cbq_linear_fixed
 * over its rows (workspace_dev as there, sized for one chunk's rows; may be
 * NULL).  Copies start after the work already queued on `stream`; calls on
 * one device are serialised by a lock.  K % 128 == 0, else
 * CBQ_ERR_UNSUPPORTED.  No counterpart on the reference's GPU path (its mmap
 * path runs on the CPU). */
int cbq_linear_fixed_streamed(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, const uint8_t *packed_host,
                              int64_t packed_bytes, const float *codebook_dev, int64_t C, int bits, int64_t M,
                              int64_t K, const float *bias_dev, void *out_dev, int out_dtype, int64_t ldo,
                              void *staging_dev, int64_t staging_bytes, void *workspace_dev,
                              int64_t workspace_bytes, void *stream);

/* Size of the device array built into the library that
 * cbq_linear_fixed_noalloc uses as its workspace (8 MiB on every GPU that
 * loads the library, until the process exits). */
#define CBQ_NOALLOC_SCRATCH_BYTES (8u << 20)

/* cbq_linear_fixed for callers that cannot allocate device memory (for
 * example a plugin inside a host framework that owns all device memory and
 * hands it only inputs and outputs).  No counterpart in the reference.
 * Same arguments and result as cbq_linear_fixed, but the workspace comes from
 * the built-in array above; no cudaMalloc/cudaFree is ever called.
 *   - Only the 3..63-token kernel (and fp32 activations at 64 tokens or
 *     more) uses the array.  On that path a matrix that needs more than
 *     CBQ_NOALLOC_SCRATCH_BYTES (cbq_linear_fixed_workspace_bytes(M, K, T))
 *     returns CBQ_ERR_ARG before anything is launched, and the bytes it uses
 *     are cleared on `stream` before the launch.  One or two tokens, and 64
 *     or more bf16 tokens, run without it (no size limit, no clearing).
 *   - The first call in a CUDA context looks the array's device address up
 *     (the address is cached per context); make that first call before any
 *     stream capture in that context.
 *   - All calls share the one array: calls that overlap on the GPU (different
 *     streams, or several host threads) race and give wrong results. */
int cbq_linear_fixed_noalloc(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                             const uint8_t *packed_dev, int64_t packed_bytes,
                             const float *codebook_dev, int64_t C, int bits,
                             int64_t M, int64_t K, const float *bias_dev,
                             void *out_dev, int out_dtype, int64_t ldo, void *stream);

/* out[t, h] = codebook[min(idx(ids[t]*H + h), C-1)] for a [vocab, H] table.
 * Replaces fused_compressed_embedding (src/gpu_accelerated_functions.py:276-307).
 * Token ids outside [0, vocab) are an argument error detected on the device:
 * their rows are zero-filled and CBQ_FLAG_CORRUPT is set in status_dev. */
int cbq_embedding_fixed(const int64_t *ids_dev, int64_t T,
                        const uint8_t *packed_dev, int64_t packed_bytes,
                        const float *codebook_dev, int64_t C, int bits,
                        int64_t vocab, int64_t H, void *out_dev, int out_dtype,
                        uint32_t *status_dev, void *stream);

/* idx[i] = field i (i < n) of a b-bit LSB-first stream on the device (the
 * inverse of cbq_pack_fixed; the reference's unpack_any_bits,
 * src/bitpack.py:97-156).  packed_bytes >= cbq_fixed_stream_bytes(1, n, bits). */
int cbq_unpack_fixed(const uint8_t *packed_dev, int64_t packed_bytes, int bits, int64_t n, uint16_t *idx_dev,
                     void *stream);

/* Write the LSB-first stream of n indices (the device twin of
 * pack_any_bits, src/bitpack.py:32-94).  out_bytes >= ceil(n*bits/8) rounded
 * up to 4; bytes past ceil(n*bits/8) are written as zero. */
int cbq_pack_fixed(const uint16_t *idx_dev, int64_t n, int bits,
                   uint8_t *out_dev, int64_t out_bytes, void *stream);

/* ======================================================================
 * Canonical-Huffman streams
 * ====================================================================== */

/* Decode tables derived from huff_lengths (uint8[alphabet]); the CUDA kernels
 * use these instead of the stored 12-bit tables, which carry the same codes
 * (src/huffman_codebook.py:353-423).  Build on the host, copy to the device
 * verbatim (the blob contains no pointers). */
int64_t cbq_huff_tables_bytes(int64_t alphabet);
int cbq_huff_tables_build(const uint8_t *huff_lengths, int64_t alphabet,
                          void *tables_host, int64_t tables_bytes);
/* Longest code length in a built table blob (0 = empty code). */
int cbq_huff_tables_max_len(const void *tables_host);

/* Device bytes to allocate for a Huffman stream whose on-disk `huff_stream`
 * has stream_len bytes (it already ends with 4 zero bytes). */
int64_t cbq_huff_stream_bytes(int64_t stream_len);

/* Symbols per entry of the chunk-entry table, its entry count
 * (M * ceil(K/64)), and the 32-bit words to allocate for the table. */
#define CBQ_HUFF_CHUNK 64
int64_t cbq_huff_chunk_count(int64_t M, int64_t K);
int64_t cbq_huff_chunk_table_words(int64_t M, int64_t K);

/* Load-time pass: decode every row once and record, for each row r and
 * chunk c (n = cbq_huff_chunk_count(M, K) entries, chunk_dev holding
 * cbq_huff_chunk_table_words(M, K) = 2n words):
 *   uint32_t chunk_dev[n]: bit offset of symbol c*64 relative to
 *     row_bit_starts[r];
 *   uint32_t quarter[n] (at chunk_dev + n): bits 0-9, 10-19 and 20-29 hold
 *     the bit lengths of the chunk's codes 0-15, 16-31 and 32-47 (each at
 *     most 16 * 32 = 512; 0 unless the row goes on past the group), so the
 *     one-token GEMV runs four independent decoders per chunk.
 * The reference format has only per-row entry points
 * (src/huffman_codebook.py:213); this table gives the GEMV its 64- and
 * 16-symbol entry points.  Records CBQ_FLAG_ROW_END when a row does not end
 * where the next one starts (the last row: when it does not end within the
 * final 16 bits of total_bits, which admits row shards cut from the tail of a
 * stream) and CBQ_FLAG_CORRUPT for undecodable codes, in status_dev. */
int cbq_huff_chunk_table(const uint8_t *stream_dev, int64_t stream_bytes,
                         const void *tables_dev, const int64_t *row_bit_starts_dev,
                         int64_t M, int64_t K, int64_t total_bits,
                         uint32_t *chunk_dev, uint32_t *status_dev, void *stream);

/* Load-time pass: the two-level decode table the fused GEMV reads.  For each
 * 14-bit prefix: the length of the code it starts with and either the
 * codebook value (bf16 bits, when every codebook value is exactly a bf16: all
 * lossless codebooks) or the symbol; prefixes of longer codes point into a
 * second-level table.  lut_dev holds cbq_huff_decode_lut_bytes() bytes,
 * 16-byte aligned. */
int64_t cbq_huff_decode_lut_bytes(void);
int cbq_huff_build_decode_lut(const void *tables_dev, const float *codebook_dev, int64_t C,
                              uint32_t *lut_dev, void *stream);

/* Workspace bytes cbq_linear_huff may use (same contract as
 * cbq_linear_fixed_workspace_bytes).  From 64 tokens this includes room for
 * the stream transcoded to fixed width (2 * M * K bytes at most): with it,
 * bf16 activations, M % 128 == 0, K % 128 == 0 and C <= 16384, the call
 * first rewrites the Huffman stream as a b-bit LSB-first stream (b =
 * ceil(log2 C), indices clamped to C - 1) in the workspace and then runs the
 * tensor-core GEMM of cbq_linear_fixed on it, so every symbol is
 * entropy-decoded once per call; without it the CUDA-core kernel runs. */
int64_t cbq_linear_huff_workspace_bytes(int64_t M, int64_t K, int64_t T);

/* Fused Huffman decode + GEMV: same result as cbq_linear_fixed on the
 * decoded indices.  Replaces huffman_decode_to_i32 + huffman_i32_linear
 * (src/gpu_huffman_functions.py:297-370), without the int32 [M,K] buffer.
 * total_bits = 8 * (stream_len - 4): the end of the last row.  workspace_dev
 * may be NULL (work is then balanced in whole rows). */
int cbq_linear_huff(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                    const uint8_t *stream_dev, int64_t stream_bytes,
                    const void *tables_dev, const uint32_t *lut_dev,
                    const int64_t *row_bit_starts_dev,
                    const uint32_t *chunk_dev, int64_t total_bits,
                    const float *codebook_dev, int64_t C,
                    int64_t M, int64_t K, const float *bias_dev,
                    void *out_dev, int out_dtype, int64_t ldo,
                    void *workspace_dev, int64_t workspace_bytes,
                    uint32_t *status_dev, void *stream);

/* Huffman embedding: decodes only the requested rows (the reference decodes
 * the whole table per call, src/gpu_huffman_functions.py:966-978). */
int cbq_embedding_huff(const int64_t *ids_dev, int64_t T,
                       const uint8_t *stream_dev, int64_t stream_bytes,
                       const void *tables_dev, const int64_t *row_bit_starts_dev,
                       const uint32_t *chunk_dev, const float *codebook_dev,
                       int64_t C, int64_t vocab, int64_t H,
                       void *out_dev, int out_dtype, uint32_t *status_dev,
                       void *stream);

/* Decode rows to uint16 indices (the device twin of
 * huffman_decode_indices, src/huffman_codebook.py:259-340; used to check
 * bit-exactness, not on the GEMV path). */
int cbq_huff_decode_indices(const uint8_t *stream_dev, int64_t stream_bytes,
                            const void *tables_dev, const int64_t *row_bit_starts_dev,
                            const uint32_t *chunk_dev, int64_t M, int64_t K,
                            uint16_t *idx_dev, uint32_t *status_dev, void *stream);

/* Encode n indices with canonical codes (code_dev uint32[alphabet],
 * len_dev uint8[alphabet]) at the given exclusive bit starts (int64[n]),
 * MSB-first (the device twin of src/huffman_codebook.py:167-201).  out_dev
 * must hold out_bytes >= ceil(total_bits/8) + 8 bytes; it is zeroed here. */
int cbq_huff_encode(const uint16_t *idx_dev, int64_t n, const uint32_t *code_dev,
                    const uint8_t *len_dev, const int64_t *bit_starts_dev,
                    uint8_t *out_dev, int64_t out_bytes, void *stream);

/* ======================================================================
 * Decode-step kernels around the compressed linear layers (one new token
 * per sequence).  The math of HF transformers' Qwen3 decoder layer
 * (models/qwen3); element-wise steps round to the activation dtype where the
 * unfused sequence of torch operations does, reductions run in fp32.  No
 * counterpart in the reference, which runs these steps through HF's torch
 * modules (src/model_loader.py builds the HF model around the compressed
 * linears).  dtype: CBQ_F32 or CBQ_BF16 for every activation and cache.
 * ====================================================================== */

/* Per row r of x [rows, n]: if add_dev, x[r] = round(x[r] + add[r]) (written
 * back: the residual-stream update); then
 * out[r] = round(w * round(x[r] * rsqrt(mean(x[r]^2) + eps))), w = weight_dev
 * (fp32 [n]) or 1. */
int cbq_rmsnorm(void *x_dev, const void *add_dev, int dtype, int64_t rows, int64_t n,
                const float *weight_dev, float eps, void *out_dev, void *stream);

/* The all-reduce consumer: waits (bounded, 2 s; CBQ_FLAG_TIMEOUT in
 * status_dev, nothing written, on expiry) until counts_dev[s] >=
 * (*epoch_dev) * expect for every rank s < world, then for each row r of x
 * [rows, n]: x[r] = round(x[r] + round(sum_s slots[s][r])) in rank order
 * (slots_dev: [world][rows][n], this rank's buffer that the peers wrote) and
 * out[r] = RMSNorm(x[r]) as cbq_rmsnorm.  *epoch_dev counts the steps (the
 * caller increments it once per step before the first producer). */
int cbq_rmsnorm_allreduce(void *x_dev, const void *slots_dev, const uint32_t *counts_dev,
                          const uint32_t *epoch_dev, int64_t expect, int world, int dtype, int64_t rows,
                          int64_t n, const float *weight_dev, float eps, void *out_dev,
                          uint32_t *status_dev, void *stream);

/* Greedy next token of B logits rows [B, ld] (this rank's V vocabulary
 * entries, ids rank*V .. rank*V + V - 1): the largest logit, the lowest id on
 * ties (torch's max), written to next_ids_dev[b] (int64).  world > 1: each
 * rank stores its (value, id) pair as two epoch-flagged 64-bit words into
 * slot `rank` of every rank's pick buffer (slot_dev[p]: rank p's buffer at
 * this rank's slot, [B][2] words; local_slots_dev: this rank's buffer,
 * [world][B][2] words) and takes the best of the world pairs it reads back
 * (bounded wait for *epoch_dev; on timeout CBQ_FLAG_TIMEOUT in status_dev and
 * the row keeps its previous id).  Replaces the all-gather of (max, index)
 * pairs and the torch reductions around it.  No counterpart in the reference
 * (HF's generate picks on the host framework's side). */
int cbq_greedy_pick(const void *logits_dev, int dtype, int64_t B, int64_t V, int64_t ld, int rank, int world,
                    void *const *slot_dev, const void *local_slots_dev, const uint32_t *epoch_dev,
                    int64_t *next_ids_dev, uint32_t *status_dev, void *stream);

/* The attention block's element-wise part for the token at position *pos_dev
 * (device int64): per-head RMSNorm of q [B, Hq*d] and k [B, Hkv*d] (weights
 * fp32 [d] or NULL = 1), rotary embedding with cos/sin tables (fp32
 * [cache_len, d], rotate_half form), q -> q_out [B, Hq, d], k and v [B, Hkv*d]
 * -> row *pos_dev of k_cache / v_cache [B, Hkv, cache_len, d].  head_dim 64,
 * 128 or 256.  Nothing is written when *pos_dev is outside [0, cache_len). */
int cbq_qk_norm_rope(const void *q_dev, const void *k_dev, const void *v_dev, int dtype, int64_t B,
                     int64_t Hq, int64_t Hkv, int64_t head_dim, float eps, const float *q_weight_dev,
                     const float *k_weight_dev, const float *cos_dev, const float *sin_dev,
                     const int64_t *pos_dev, void *q_out_dev, void *k_cache_dev, void *v_cache_dev,
                     int64_t cache_len, void *stream);

/* Grouped-query attention of q [B, Hq, d] over cache rows 0..*pos_dev of
 * k_cache / v_cache [B, Hkv, cache_len, d] (query head h reads kv head
 * h / (Hq / Hkv)), softmax(q k^T * scale) v in fp32 -> out [B, Hq*d].
 * Hq / Hkv <= 8; the scores of one kv head's query heads
 * (cache_len * Hq/Hkv * 4 bytes) are held in shared memory, so longer caches
 * return CBQ_ERR_UNSUPPORTED. */
int cbq_attn_decode(const void *q_dev, const void *k_cache_dev, const void *v_cache_dev, int dtype,
                    int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, int64_t cache_len,
                    const int64_t *pos_dev, float scale, void *out_dev, void *stream);

/* cbq_qk_norm_rope followed by cbq_attn_decode in one launch: q_dev, k_dev,
 * v_dev are this step's projections; each CTA normalizes and rotates its kv
 * head's query heads (kept on chip) and new k row, writes the new k and v
 * rows at *pos_dev into the caches, then attends over rows 0..*pos_dev.  A
 * position outside [0, cache_len) gives a zero output and writes nothing. */
int cbq_attn_decode_rope(const void *q_dev, const void *k_dev, const void *v_dev, int dtype, int64_t B,
                         int64_t Hq, int64_t Hkv, int64_t head_dim, float eps, const float *q_weight_dev,
                         const float *k_weight_dev, const float *cos_dev, const float *sin_dev,
                         const int64_t *pos_dev, void *k_cache_dev, void *v_cache_dev, int64_t cache_len,
                         float scale, void *out_dev, void *stream);

/* Workspace bytes of the split-key attention entry points below for this
 * shape (its arrival counters must be zero before the first call; every call
 * leaves them zero).  No counterpart in the reference. */
int64_t cbq_attn_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, int64_t cache_len);

/* out[i] = round(round(silu(g[i])) * u[i]) over n elements (fp32 or bf16;
 * out may alias g or u): SiLU * up when gate and up come from separate
 * launches (Huffman streams, more than two tokens), with the rounding of the
 * fused GEMV epilogue.  No counterpart in the reference (HF Qwen3MLP). */
int cbq_silu_mul(const void *g_dev, const void *u_dev, int dtype, int64_t n, void *out_dev, void *stream);

/* cbq_attn_decode_rope / cbq_attn_decode with the keys of every (row, kv
 * head) split over several CTAs (flash-decoding): each CTA attends over one
 * chunk of the keys and writes its partial softmax state (max, sum,
 * unnormalised weighted values) to the workspace, and the CTA that finishes
 * a (row, kv head) last combines the chunks in chunk order; with at most 16
 * chunks they run as one thread-block cluster and combine through
 * distributed shared memory instead (same arithmetic and order;
 * CBQ_ATTN_CLUSTER=0 in the environment selects the workspace form).  The
 * number of chunks depends only on B, Hkv, cache_len and the SM count, so a
 * call is deterministic.  Results equal the one-CTA forms up to the fp32 summation
 * order.  workspace_bytes >= cbq_attn_workspace_bytes(...), else CBQ_ERR_ARG.
 * Calls that share a workspace must not overlap on the GPU.  No counterpart
 * in the reference (HF attention on the host framework's side). */
int cbq_attn_decode_rope_split(const void *q_dev, const void *k_dev, const void *v_dev, int dtype, int64_t B,
                               int64_t Hq, int64_t Hkv, int64_t head_dim, float eps, const float *q_weight_dev,
                               const float *k_weight_dev, const float *cos_dev, const float *sin_dev,
                               const int64_t *pos_dev, void *k_cache_dev, void *v_cache_dev, int64_t cache_len,
                               float scale, void *out_dev, void *workspace_dev, int64_t workspace_bytes,
                               void *stream);
int cbq_attn_decode_split(const void *q_dev, const void *k_cache_dev, const void *v_cache_dev, int dtype,
                          int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, int64_t cache_len,
                          const int64_t *pos_dev, float scale, void *out_dev, void *workspace_dev,
                          int64_t workspace_bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* CBQ_H */
