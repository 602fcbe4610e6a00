/*
 * cbq_oracle.c -- CPU restatement of the reference's codebook decode-matmul
 * path (bigattichouse/Codebook-Quantization).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA product
 * path: tests, the smoke check and the bench's cpu_baseline leg may call it;
 * the product (the CUDA library and the Python package) never links or calls
 * it.  Every function cites the reference file:line whose behaviour it
 * restates.  Paths are relative to the reference project root.
 *
 * Formats restated here:
 *   - fixed width: element e of a row-major [M,K] index matrix occupies bits
 *     [e*b, (e+1)*b) of a little-endian LSB-first byte stream
 *     (src/bitpack.py:32-94, src/compressed_matmul.c:334-347);
 *   - canonical Huffman: MSB-first bit stream, rows concatenated without
 *     alignment, row r starts at row_bit_starts[r] (src/huffman_codebook.py:
 *     126-226), decoded with a 12-bit prefix table plus a per-length
 *     canonical slow path (src/compressed_matmul.c:121-186).
 *
 * Unlike the reference, reads beyond the supplied byte length return zero
 * bits, so the oracle needs no padding (the reference relies on 2 or 4 pad
 * bytes; src/compressed_matmul_cpu.py:303-305, 441-442).
 *
 * Arithmetic order matches the reference kernels: for each row r, k ascends
 * and each token t accumulates x[t,k]*w into an fp32 sum
 * (src/compressed_matmul.c:416-450).
 */
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_LUT_BITS 12

/* ---------------------------------------------------------------- helpers */

static inline uint32_t orc_byte(const uint8_t *s, int64_t len, int64_t i)
{
    return (i >= 0 && i < len) ? (uint32_t)s[i] : 0u;
}

/* Fixed-width index at element e (src/compressed_matmul.c:334-347): the
 * index is the b-bit field starting at bit e*b, bit 0 being the LSB of
 * byte 0.  A 32-bit little-endian window over 4 bytes covers any b <= 16
 * at any shift 0..7. */
static inline uint32_t orc_fixed_at(const uint8_t *packed, int64_t len,
                                    int64_t e, int bits)
{
    int64_t bit = e * (int64_t)bits;
    int64_t byte = bit >> 3;
    unsigned shift = (unsigned)(bit & 7);
    uint32_t win = orc_byte(packed, len, byte)
                 | (orc_byte(packed, len, byte + 1) << 8)
                 | (orc_byte(packed, len, byte + 2) << 16)
                 | (orc_byte(packed, len, byte + 3) << 24);
    uint32_t mask = (bits >= 32) ? 0xffffffffu : ((1u << bits) - 1u);
    return (win >> shift) & mask;
}

/* MSB-first peek of n <= 25 bits at absolute bit position pos
 * (src/compressed_matmul.c:121-131). */
static inline uint32_t orc_peek_msb(const uint8_t *s, int64_t len,
                                    int64_t pos, int n)
{
    int64_t byte = pos >> 3;
    unsigned off = (unsigned)(pos & 7);
    uint32_t w = (orc_byte(s, len, byte) << 24)
               | (orc_byte(s, len, byte + 1) << 16)
               | (orc_byte(s, len, byte + 2) << 8)
               |  orc_byte(s, len, byte + 3);
    return (w << off) >> (32 - n);
}

/* One canonical-Huffman symbol (src/compressed_matmul.c:148-186).
 * Fast path: the next 12 bits index lut_sym/lut_len; lut_len==0 means the
 * code is longer than 12 bits.  Slow path: grow the code one bit at a time
 * and test it against the first code / symbol count of each length.  A code
 * that matches no length consumes one bit and yields symbol 0 (the
 * reference's corrupt-stream guard). */
static inline int orc_decode_one(const uint8_t *s, int64_t len, int64_t *pos,
                                 const uint16_t *lut_sym, const uint8_t *lut_len,
                                 const int64_t *sl_first_code,
                                 const int32_t *sl_base_offset,
                                 const uint16_t *sl_sym, int sl_max_len)
{
    uint32_t key = orc_peek_msb(s, len, *pos, ORC_LUT_BITS);
    int l = lut_len[key];
    if (l > 0) {
        *pos += l;
        return lut_sym[key];
    }
    uint32_t code = key;
    for (int L = ORC_LUT_BITS + 1; L <= sl_max_len; ++L) {
        code = (code << 1) | orc_peek_msb(s, len, *pos + (L - 1), 1);
        int64_t first = sl_first_code[L];
        if (first < 0) continue;
        int64_t d = (int64_t)code - first;
        int64_t cnt = (int64_t)sl_base_offset[L + 1] - sl_base_offset[L];
        if (d >= 0 && d < cnt) {
            *pos += L;
            return sl_sym[sl_base_offset[L] + d];
        }
    }
    *pos += 1;
    return 0;
}

static inline int orc_clamp(int idx, int64_t C)
{
    return (idx >= C) ? (int)(C - 1) : idx;
}

/* ------------------------------------------------------------ fixed width */

/* Decode n indices starting at element `first`
 * (src/bitpack.py:97-156; element addressing of src/compressed_matmul.c:337). */
void orc_unpack_fixed(const uint8_t *packed, int64_t packed_len, int bits,
                      int64_t first, int64_t n, uint16_t *out)
{
    #pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        out[i] = (uint16_t)orc_fixed_at(packed, packed_len, first + i, bits);
}

/* out[t*M + r] += sum_k x[t*K+k] * cb[min(idx(r*K+k), C-1)] for rows
 * [r0, r1) (src/compressed_matmul.c:416-450).  out is accumulated into;
 * the caller zeroes it, as the reference requires. */
void orc_linear_fixed_f32(const float *x, const uint8_t *packed,
                          int64_t packed_len, const float *cb, int64_t C,
                          int bits, int64_t T, int64_t M, int64_t K,
                          float *out, int64_t r0, int64_t r1)
{
    if (r1 > M) r1 = M;
    #pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = r0; r < r1; ++r) {
        for (int64_t k = 0; k < K; ++k) {
            int idx = orc_clamp((int)orc_fixed_at(packed, packed_len, r * K + k, bits), C);
            float w = cb[idx];
            for (int64_t t = 0; t < T; ++t)
                out[t * M + r] += x[t * K + k] * w;
        }
    }
}

/* out[t, h] = cb[min(idx(id_t*H + h), C-1)]
 * (src/gpu_accelerated_functions.py:109-126). */
void orc_embedding_fixed_f32(const int64_t *ids, int64_t T, const uint8_t *packed,
                             int64_t packed_len, const float *cb, int64_t C,
                             int bits, int64_t H, float *out)
{
    #pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t)
        for (int64_t h = 0; h < H; ++h) {
            int idx = orc_clamp((int)orc_fixed_at(packed, packed_len, ids[t] * H + h, bits), C);
            out[t * H + h] = cb[idx];
        }
}

/* ---------------------------------------------------------------- Huffman */

/* Decode K symbols for each row r in [0, M), starting at row_bit_starts[r]
 * (the per-row decode of src/compressed_matmul.c:296-322, returning the raw
 * symbols instead of codebook values). */
void orc_huff_decode_rows(const uint8_t *stream, int64_t stream_len,
                          const uint16_t *lut_sym, const uint8_t *lut_len,
                          const int64_t *sl_first_code, const int32_t *sl_base_offset,
                          const uint16_t *sl_sym, int sl_max_len,
                          const int64_t *row_bit_starts, int64_t M, int64_t K,
                          uint16_t *out)
{
    #pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < M; ++r) {
        int64_t pos = row_bit_starts[r];
        for (int64_t k = 0; k < K; ++k)
            out[r * K + k] = (uint16_t)orc_decode_one(stream, stream_len, &pos, lut_sym, lut_len,
                                                      sl_first_code, sl_base_offset, sl_sym,
                                                      sl_max_len);
    }
}

/* Bit offset of every S-th symbol of every row, relative to the row start:
 * offs[r*nchunk + c] = bit position of symbol c*S of row r minus
 * row_bit_starts[r].  The reference has no such table; this is the oracle
 * for the chunk-entry table the CUDA path derives at load time. */
void orc_huff_chunk_offsets(const uint8_t *stream, int64_t stream_len,
                            const uint16_t *lut_sym, const uint8_t *lut_len,
                            const int64_t *sl_first_code, const int32_t *sl_base_offset,
                            const uint16_t *sl_sym, int sl_max_len,
                            const int64_t *row_bit_starts, int64_t M, int64_t K,
                            int64_t S, int64_t *offs)
{
    int64_t nchunk = (K + S - 1) / S;
    #pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = 0; r < M; ++r) {
        int64_t pos = row_bit_starts[r];
        for (int64_t k = 0; k < K; ++k) {
            if (k % S == 0) offs[r * nchunk + k / S] = pos - row_bit_starts[r];
            orc_decode_one(stream, stream_len, &pos, lut_sym, lut_len,
                           sl_first_code, sl_base_offset, sl_sym, sl_max_len);
        }
    }
}

/* out[t*M + r] += sum_k x[t*K+k] * cb[min(sym_k, C-1)] over rows [r0, r1)
 * (src/compressed_matmul.c:208-239).  out is accumulated into. */
void orc_huff_linear_f32(const float *x, const uint8_t *stream, int64_t stream_len,
                         const uint16_t *lut_sym, const uint8_t *lut_len,
                         const int64_t *sl_first_code, const int32_t *sl_base_offset,
                         const uint16_t *sl_sym, int sl_max_len,
                         const int64_t *row_bit_starts, const float *cb, int64_t C,
                         int64_t T, int64_t M, int64_t K, float *out,
                         int64_t r0, int64_t r1)
{
    if (r1 > M) r1 = M;
    #pragma omp parallel for schedule(dynamic, 64)
    for (int64_t r = r0; r < r1; ++r) {
        int64_t pos = row_bit_starts[r];
        for (int64_t k = 0; k < K; ++k) {
            int sym = orc_decode_one(stream, stream_len, &pos, lut_sym, lut_len,
                                     sl_first_code, sl_base_offset, sl_sym, sl_max_len);
            float w = cb[orc_clamp(sym, C)];
            for (int64_t t = 0; t < T; ++t)
                out[t * M + r] += x[t * K + k] * w;
        }
    }
}

/* out[t, h] = cb[min(sym, C-1)] for the H symbols of row ids[t]
 * (src/compressed_matmul.c:253-281).  out is overwritten. */
void orc_huff_embedding_f32(const int64_t *ids, int64_t T, const uint8_t *stream,
                            int64_t stream_len, const uint16_t *lut_sym,
                            const uint8_t *lut_len, const int64_t *sl_first_code,
                            const int32_t *sl_base_offset, const uint16_t *sl_sym,
                            int sl_max_len, const int64_t *row_bit_starts,
                            const float *cb, int64_t C, int64_t H, float *out)
{
    #pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
        int64_t pos = row_bit_starts[ids[t]];
        for (int64_t h = 0; h < H; ++h) {
            int sym = orc_decode_one(stream, stream_len, &pos, lut_sym, lut_len,
                                     sl_first_code, sl_base_offset, sl_sym, sl_max_len);
            out[t * H + h] = cb[orc_clamp(sym, C)];
        }
    }
}

/* Threads for the next parallel regions started by the calling thread (the
 * OpenMP runtime is shared with the reference's own object in the process, so
 * this also sets the threads of its kernels).  Overrides OMP_NUM_THREADS,
 * which launchers such as torchrun set to 1. */
void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* Threads OpenMP will use (for reporting the CPU baseline's core count). */
int orc_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
