// cbq_huff.cu -- canonical-Huffman codebook decode-GEMV, embedding, decode and
// encoder (sm_100a).
//
// Stream format: canonical codes written MSB-first, rows concatenated with no
// alignment, row r starting at bit row_bit_starts[r]
// (reference src/huffman_codebook.py:126-226).  A symbol decodes through a
// 12-bit prefix table, or, for longer codes, by finding the smallest length L
// whose canonical range contains the next L bits -- the same result as the
// reference's bit-by-bit slow path (src/compressed_matmul.c:148-186); a
// prefix that matches no code yields symbol 0 and consumes one bit, as the
// reference does, and is recorded in the caller's status word.
//
// GEMV (cbq_linear_huff): the reference format can only be entered at row
// starts, so a load-time pass (cbq_huff_chunk_table) records the bit offset of
// every 64th symbol of every row; a second load-time pass
// (cbq_huff_build_decode_lut) folds the codebook into a two-level decode
// table.  The fused kernel itself is in cbq_huff_kernel.cuh.
#include <algorithm>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <numeric>

#include "cbq_hgemv_kernel.cuh"
#include "cbq_huff_kernel.cuh"

namespace cbq {
int gemm_fixed(const void *x, int64_t T, int64_t ldx, const uint8_t *packed, const float *cb, int64_t C,
               int bits, int64_t M, int64_t K, const float *bias, void *out, int out_dtype, int64_t ldo,
               cudaStream_t s);
}

namespace {

using namespace cbq;

constexpr uint32_t kMagic = 0x48514243u;  // "CBQH"
constexpr int kLutBits = 12;
constexpr int kLutSize = 1 << kLutBits;
constexpr int kMaxLen = 32;
constexpr int S = CBQ_HUFF_CHUNK;          // symbols per chunk entry

static_assert(offsetof(HuffTables, lut) % 16 == 0, "lut must be 16-byte aligned for uint4 loads");
static_assert(offsetof(HuffTables, lut) == 688, "blob layout is part of the ABI (tests decode it)");
static_assert(sizeof(HuffTables) % 16 == 0, "blob alignment");

// Shared-memory copy of the parts of the tables every symbol may touch.
// 16-byte aligned: load_tables() fills lut with 16-byte stores.
struct alignas(16) SmemTables {
    uint32_t lut[kLutSize];
    uint64_t limit[kMaxLen + 1];
    uint64_t first[kMaxLen + 1];
    int32_t offset[kMaxLen + 1];
    int32_t max_len;
};

__device__ void load_tables(SmemTables *st, const HuffTables *g) {
    const uint4 *src = reinterpret_cast<const uint4 *>(g->lut);
    uint4 *dst = reinterpret_cast<uint4 *>(st->lut);
    for (int i = threadIdx.x; i < kLutSize / 4; i += blockDim.x) dst[i] = src[i];
    for (int i = threadIdx.x; i <= kMaxLen; i += blockDim.x) {
        st->limit[i] = g->limit[i];
        st->first[i] = g->first[i];
        st->offset[i] = g->offset[i];
    }
    if (threadIdx.x == 0) st->max_len = g->max_len;
}

// Decode the symbol at the top of `buf`; len = 0 means no code matched.
__device__ __forceinline__ uint32_t decode_sym(uint64_t buf, const SmemTables *st,
                                               const uint16_t *gsyms, int &len) {
    const uint32_t e = st->lut[buf >> (64 - kLutBits)];
    len = (int)(e >> 16);
    if (len) return e & 0xffffu;
    const uint32_t w32 = (uint32_t)(buf >> 32);
    const int ml = st->max_len;
    for (int L = kLutBits + 1; L <= ml; ++L) {
        const uint64_t v = (uint64_t)(w32 >> (32 - L));
        if (v < st->limit[L]) {
            len = L;
            return gsyms[st->offset[L] + (uint32_t)(v - st->first[L])];
        }
    }
    len = 0;
    return 0u;
}

// ---------------------------------------------------------------- chunk table

__global__ void __launch_bounds__(128) k_huff_chunks(const uint8_t *stream, uint64_t nwords,
                                                     const HuffTables *tab,
                                                     const int64_t *rbs, int64_t M, int64_t K,
                                                     int64_t total_bits, uint32_t *chunk,
                                                     uint32_t *status) {
    __shared__ SmemTables st;
    load_tables(&st, tab);
    __syncthreads();
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= M) return;
    const uint16_t *gsyms = blob_syms(tab);
    const int64_t nch = (K + S - 1) / S;
    const int64_t start = rbs[r];
    BitBuf bb;
    bb.init(reinterpret_cast<const uint32_t *>(stream), nwords, (uint64_t)start);
    int64_t pos = start, q0 = start;
    uint32_t bad = 0, quarters = 0;
    bool overflow = false;
    uint32_t *quarter = chunk + M * nch;
    static_assert(S == 64, "three 10-bit quarter lengths per 64-symbol chunk");
    for (int64_t k = 0; k < K; ++k) {
        if ((k % S) == 0) {
            const int64_t rel = pos - start;
            overflow |= rel > 0xffffffffll;
            chunk[r * nch + k / S] = (uint32_t)rel;
            if (k) quarter[r * nch + k / S - 1] = quarters;
            quarters = 0;
            q0 = pos;
        } else if ((k % 16) == 0) {                               // at most 16 codes of at most 32 bits
            quarters |= (uint32_t)(pos - q0) << (10 * (int)((k % S) / 16 - 1));
            q0 = pos;
        }
        int len;
        decode_sym(bb.buf, &st, gsyms, len);
        if (len == 0) { len = 1; ++bad; }
        bb.consume(len);
        pos += len;
    }
    if (K) quarter[r * nch + nch - 1] = quarters;
    if (bad) report(status, CBQ_FLAG_CORRUPT, (uint32_t)r);
    // The last row ends inside the stream's final bytes: within 8 bits of the
    // end for a stream as the encoder writes it, within 16 for a row shard
    // cut from the tail of one (the source's up to 7 padding bits, plus up to
    // 7 more from the shard's own byte rounding).
    const bool last = (r + 1 == M);
    const bool end_ok = last ? (pos <= total_bits && pos > total_bits - 16) || (K == 0)
                             : (pos == rbs[r + 1]);
    if (!end_ok || overflow) report(status, CBQ_FLAG_ROW_END, (uint32_t)r);
}

// ---------------------------------------------------------------- decode table

// Length of the canonical code that starts the 32-bit window w (0: none).
__device__ __forceinline__ int code_len_at(const HuffTables *t, uint32_t w, uint32_t &sym) {
    for (int L = 1; L <= t->max_len; ++L) {
        const uint64_t v = (uint64_t)(w >> (32 - L));
        if (v < t->limit[L]) {
            sym = blob_syms(t)[t->offset[L] + (uint32_t)(v - t->first[L])];
            return L;
        }
    }
    sym = 0;
    return 0;
}

// One block of 1024 threads builds the two-level decode table
// (layout in cbq_huff_kernel.cuh).  Thread i owns the 16 consecutive 14-bit
// prefixes [16i, 16i+16); second-level tables are laid out in prefix order by
// a block-wide exclusive scan and dropped (canonical search) once they would
// exceed kHfSubMax entries.
__global__ void __launch_bounds__(1024) k_huff_build_lut(const HuffTables *tab, const float *cb, int C,
                                                         uint32_t *lut) {
    __shared__ uint32_t warp_tot[32];
    int exact = 1;
    for (int c = threadIdx.x; c < C; c += blockDim.x) exact &= (__float_as_uint(cb[c]) & 0xffffu) == 0;
    exact = __syncthreads_and(exact);
    auto payload = [&](uint32_t sym) -> uint32_t {
        return exact ? (__float_as_uint(cb[min((int)sym, C - 1)]) >> 16) : sym;
    };
    constexpr int kPer = kHfLutSize / 1024;
    const int p0 = threadIdx.x * kPer;
    uint8_t depth[kPer];
    uint32_t mine = 0;
    for (int j = 0; j < kPer; ++j) {
        const uint32_t p = (uint32_t)(p0 + j);
        uint32_t sym;
        const int L0 = code_len_at(tab, p << (32 - kHfLutBits), sym);
        depth[j] = 0;
        if (L0 >= 1 && L0 <= kHfLutBits) {
            lut[p] = (payload(sym) << 16) | (uint32_t)L0;
        } else if (L0 == 0 && code_len_at(tab, (p << (32 - kHfLutBits)) | ((1u << (32 - kHfLutBits)) - 1u),
                                          sym) == 0) {
            lut[p] = (payload(0) << 16) | 1u;           // no code starts here: guard
        } else if (L0 > kHfLutBits || L0 == 0) {
            uint32_t s2;
            int L1 = code_len_at(tab, (p << (32 - kHfLutBits)) | ((1u << (32 - kHfLutBits)) - 1u), s2);
            if (L1 == 0) L1 = 32;                           // incomplete code: cover every bit
            depth[j] = (uint8_t)(L1 - kHfLutBits);
            mine += 1u << depth[j];
            lut[p] = 0;
        } else {
            lut[p] = 0;
        }
    }
    // block exclusive scan of `mine`
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = mine;
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const uint32_t v = warp_tot[lane];
        uint32_t iv = v;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t u = __shfl_up_sync(0xffffffffu, iv, o);
            if (lane >= o) iv += u;
        }
        warp_tot[lane] = iv - v;                             // exclusive per warp
    }
    __syncthreads();
    uint32_t off = warp_tot[warp] + incl - mine;
    uint32_t *sub = lut + kHfLutSize + 4;
    uint32_t used_max = 0;
    int dropped = 0;
    for (int j = 0; j < kPer; ++j) {
        if (!depth[j]) continue;
        const uint32_t p = (uint32_t)(p0 + j);
        const uint32_t d = depth[j], n = 1u << d;
        if (off + n <= (uint32_t)kHfSubMax) {
            lut[p] = (off << 16) | 0x80u | (32u - d);
            for (uint32_t k = 0; k < n; ++k) {
                const uint32_t w = (p << (32 - kHfLutBits)) | (k << (32 - kHfLutBits - d));
                uint32_t sym;
                const int L = code_len_at(tab, w, sym);
                sub[off + k] = (L > kHfLutBits) ? ((payload(sym) << 16) | (uint32_t)L)
                                                : ((payload(0) << 16) | 1u);
            }
            used_max = max(used_max, off + n);
        } else {
            dropped = 1;
        }
        off += n;
    }
    used_max = __reduce_max_sync(0xffffffffu, used_max);
    if (lane == 0) atomicMax(&lut[kHfLutSize + 1], used_max);
    dropped = __syncthreads_or(dropped);
    if (threadIdx.x == 0) {
        lut[kHfLutSize] = exact ? 1u : 0u;
        lut[kHfLutSize + 2] = dropped ? 0u : 1u;
    }
}

// ---------------------------------------------------------------- decode / embedding

__global__ void __launch_bounds__(256) k_huff_decode(const uint8_t *stream, uint64_t nwords,
                                                     const HuffTables *tab,
                                                     const int64_t *rbs, const uint32_t *chunk,
                                                     int64_t M, int64_t K, uint16_t *idx,
                                                     uint32_t *status) {
    __shared__ SmemTables st;
    load_tables(&st, tab);
    __syncthreads();
    const int64_t nch = (K + S - 1) / S;
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= M * nch) return;
    const int64_t r = g / nch, q = g - r * nch;
    const uint16_t *gsyms = blob_syms(tab);
    BitBuf bb;
    bb.init(reinterpret_cast<const uint32_t *>(stream), nwords, (uint64_t)(rbs[r] + chunk[g]));
    const int nsym = (int)min((int64_t)S, K - q * S);
    uint32_t bad = 0;
    for (int i = 0; i < nsym; ++i) {
        int len;
        const uint32_t sym = decode_sym(bb.buf, &st, gsyms, len);
        if (len == 0) { len = 1; ++bad; }
        bb.consume(len);
        idx[r * K + q * S + i] = (uint16_t)sym;
    }
    if (bad) report(status, CBQ_FLAG_CORRUPT, (uint32_t)r);
}

// Huffman -> fixed-width transcode for the tensor-core prefill: thread g
// decodes 64-symbol chunk q of row r (entered through the chunk table) and
// writes its fields at BITS bits each, LSB-first: the chunk's 64 * BITS bits
// are exactly the 2 * BITS words at word (r * K / 64 + q) * 2 * BITS of the
// fixed-width stream (K % 64 == 0), so threads never share a word.  Symbols
// are clamped to C - 1 as they are written (the reference's clamp), which
// the GEMM would otherwise apply.
template <int BITS>
__global__ void __launch_bounds__(256) k_huff_transcode(const uint8_t *stream, uint64_t nwords,
                                                        const HuffTables *tab, const int64_t *rbs,
                                                        const uint32_t *chunk, int64_t M, int64_t K, int C,
                                                        uint32_t *packed, uint32_t *status) {
    __shared__ SmemTables st;
    load_tables(&st, tab);
    __syncthreads();
    const int64_t nch = K / S;
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= M * nch) return;
    const int64_t r = g / nch;
    const uint16_t *gsyms = blob_syms(tab);
    BitBuf bb;
    bb.init(reinterpret_cast<const uint32_t *>(stream), nwords, (uint64_t)(rbs[r] + chunk[g]));
    constexpr int NW = 2 * BITS;
    constexpr uint32_t mask = (1u << BITS) - 1u;
    uint32_t w[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = 0u;
    uint32_t bad = 0;
#pragma unroll
    for (int i = 0; i < S; ++i) {
        int len;
        // clamp (idx >= C -> C-1) here: the field then fits BITS = bits_for(C)
        const uint32_t sym = min(decode_sym(bb.buf, &st, gsyms, len), (uint32_t)(C - 1)) & mask;
        if (len == 0) { len = 1; ++bad; }
        bb.consume(len);
        const int bit = i * BITS, wi = bit >> 5, sh = bit & 31;
        w[wi] |= sym << sh;
        if (sh + BITS > 32) w[wi + 1] |= sym >> (32 - sh);
    }
    uint2 *dst = reinterpret_cast<uint2 *>(packed + g * NW);
#pragma unroll
    for (int i = 0; i < NW / 2; ++i) dst[i] = make_uint2(w[2 * i], w[2 * i + 1]);
    if (bad) report(status, CBQ_FLAG_CORRUPT, (uint32_t)r);
}

template <typename OT>
__global__ void __launch_bounds__(256) k_huff_embedding(const int64_t *ids, const uint8_t *stream,
                                                        uint64_t nwords,
                                                        const HuffTables *tab, const int64_t *rbs,
                                                        const uint32_t *chunk, const float *cb,
                                                        int C, int64_t vocab, int64_t H, OT *out,
                                                        uint32_t *status) {
    __shared__ SmemTables st;
    load_tables(&st, tab);
    __syncthreads();
    const int64_t t = blockIdx.x;
    const int64_t id = ids[t];
    const int64_t nch = (H + S - 1) / S;
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) report(status, CBQ_FLAG_CORRUPT, (uint32_t)t);
        for (int64_t h = threadIdx.x; h < H; h += blockDim.x) out[t * H + h] = from_f32<OT>(0.f);
        return;
    }
    const uint16_t *gsyms = blob_syms(tab);
    const uint32_t cmax = (uint32_t)(C - 1);
    for (int64_t q = threadIdx.x; q < nch; q += blockDim.x) {
        BitBuf bb;
        bb.init(reinterpret_cast<const uint32_t *>(stream), nwords,
                (uint64_t)(rbs[id] + chunk[id * nch + q]));
        const int nsym = (int)min((int64_t)S, H - q * S);
        uint32_t bad = 0;
        for (int i = 0; i < nsym; ++i) {
            int len;
            const uint32_t sym = decode_sym(bb.buf, &st, gsyms, len);
            if (len == 0) { len = 1; ++bad; }
            bb.consume(len);
            out[t * H + q * S + i] = from_f32<OT>(__ldg(cb + min(sym, cmax)));
        }
        if (bad) report(status, CBQ_FLAG_CORRUPT, (uint32_t)id);
    }
}

// One thread per symbol: OR its code into the (byte-swapped) big-endian words.
__global__ void k_huff_encode(const uint16_t *idx, int64_t n, const uint32_t *code,
                              const uint8_t *len, const int64_t *starts, uint32_t *out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t s = idx[i];
    const int L = len[s];
    if (L == 0) return;
    const int64_t p = starts[i];
    const int o = (int)(p & 31);
    const uint64_t v = (uint64_t)code[s] << (64 - L - o);
    const uint32_t hi = (uint32_t)(v >> 32), lo = (uint32_t)v;
    atomicOr(out + (p >> 5), bswap32(hi));
    if (lo) atomicOr(out + (p >> 5) + 1, bswap32(lo));
}

// ---------------------------------------------------------------- planning

struct HuffPlan {
    int TB = 0, grid = 0;
    uint32_t cap = 0;
    size_t smem = 0;
};

bool plan_huff(int64_t M, int64_t K, int64_t T, int64_t total_bits, int xbytes, HuffPlan &p) {
    if (M <= 0 || K <= 0 || M >= (1ll << 31) || K > (1 << 18)) return false;
    const double avg = std::max(1.0, (double)total_bits / ((double)M * (double)K));
    const int64_t seg = std::min<int64_t>(K, kHfSeg);
    p.cap = (uint32_t)std::max<int64_t>(512, cbq_host::align_up((int64_t)(seg * avg / 8.0 * 1.15) + 96, 128));
    const size_t budget = (size_t)cbq_host::max_smem_optin() - 256;
    const size_t ring = (size_t)kHfWarps * kHfSlots * p.cap;
    int TB = 8;
    while (TB > 1 && TB > T) TB /= 2;
    while (TB > 1 && huff_prefix_bytes((int)K, TB, xbytes) + ring > budget) TB /= 2;
    if (huff_prefix_bytes((int)K, TB, xbytes) + ring > budget) return false;
    p.TB = TB;
    p.smem = huff_prefix_bytes((int)K, TB, xbytes) + ring;
    p.grid = cbq_host::sm_count();
    return true;
}

// One-token kernel (k_gemv_huff): rows per CTA and the ring slot size.
struct HgPlan {
    int grid = 0, rows_per_cta = 0, nseg = 0;
    uint32_t cap = 0;
    size_t smem = 0;
};

bool plan_hgemv(int64_t M, int64_t K, int64_t total_bits, HgPlan &p) {
    if (M <= 0 || K <= 0 || M >= (1ll << 31) || K > (1 << 20)) return false;
    const int64_t sms = cbq_host::sm_count();
    const int64_t rows = (M + sms - 1) / sms;
    const int64_t nch = (K + S - 1) / S;
    const int nseg = (int)((nch + 31) / 32);
    const size_t budget = (size_t)cbq_host::max_smem_optin();
    const size_t prefix = hg_prefix_bytes((int)rows, nseg);
    if (prefix >= budget) return false;
    // room for a unit of 1.25x the average code length, capped by shared memory
    const double avg = std::max(1.0, (double)total_bits / ((double)M * (double)K));
    const int64_t want = cbq_host::align_up((int64_t)(std::min<int64_t>(K, kHgSeg) * avg / 8.0 * 1.25) + 96, 128);
    const int64_t room = (int64_t)((budget - prefix) / (kHgWarps * kHgSlots)) & ~(int64_t)127;
    const int64_t cap = std::min<int64_t>(std::max<int64_t>(want, 1024), room);
    if (cap < 1024) return false;
    p.grid = (int)((M + rows - 1) / rows);
    p.rows_per_cta = (int)rows;
    p.nseg = nseg;
    p.cap = (uint32_t)cap;
    p.smem = prefix + (size_t)kHgWarps * kHgSlots * (size_t)cap;
    return true;
}

template <typename XT>
int launch_hgemv(const HgArgs &a, const HgPlan &p, cudaStream_t s) {
    auto kern = k_gemv_huff<XT>;
    static std::mutex mu;
    static size_t configured[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CBQ_ERR_CUDA;
    {
        std::lock_guard<std::mutex> g(mu);
        if (configured[dev & 63] < p.smem) {
            CBQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
            configured[dev & 63] = p.smem;
        }
    }
    CBQ_CUDA_TRY(cbq_host::launch_pdl(kern, dim3(p.grid), dim3(kHgWarps * 32), p.smem, s, a));
    return CBQ_OK;
}

// Token count from which cbq_linear_huff transcodes to fixed width and runs
// the tensor-core GEMM (bf16 activations).
constexpr int64_t kHuffGemmMinTokens = 64;

int64_t huff_split_bytes(int64_t M, int64_t K, int64_t T) {
    const int64_t nseg = ((K + S - 1) / S + 31) / 32;
    const int64_t TB = T >= 8 ? 8 : T >= 4 ? 4 : T >= 2 ? 2 : 1;
    return cbq_host::align_up(M * nseg * TB * 4, 256) + cbq_host::align_up(M * 4, 256);
}

// Fixed-width stream of the transcode at the widest supported width (16
// bits), after the split-row workspace.
int64_t huff_transcode_bytes(int64_t M, int64_t K) { return cbq_host::align_up(M * K * 2 + 64, 256); }

int64_t huff_workspace_bytes(int64_t M, int64_t K, int64_t T) {
    return huff_split_bytes(M, K, T) + (T >= kHuffGemmMinTokens ? huff_transcode_bytes(M, K) : 0);
}

int bits_for_entries(int64_t n) {
    int b = 1;
    while (b < 16 && (1ll << b) < n) ++b;
    return b;
}

template <int BITS>
int launch_transcode(const uint8_t *stream, int64_t stream_bytes, const HuffTables *tab, const int64_t *rbs,
                     const uint32_t *chunk, int64_t M, int64_t K, int C, uint32_t *packed, uint32_t *status,
                     cudaStream_t s) {
    const int64_t n = M * (K / S);
    k_huff_transcode<BITS><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(stream, (uint64_t)stream_bytes / 4, tab, rbs,
                                                                      chunk, M, K, C, packed, status);
    return cudaGetLastError() == cudaSuccess ? CBQ_OK : CBQ_ERR_CUDA;
}

template <int TB, typename XT>
int launch_huff_t(const HuffArgs &a, const HuffPlan &p, cudaStream_t s) {
    auto kern = k_linear_huff<TB, XT>;
    static std::mutex mu;
    static size_t configured[64] = {0};
    int dev = 0;
    CBQ_CUDA_TRY(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> g(mu);
        if (configured[dev & 63] < p.smem) {
            CBQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)p.smem));
            configured[dev & 63] = p.smem;
        }
    }
    kern<<<p.grid, kHfWarps * 32, p.smem, s>>>(a);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

template <typename XT>
int linear_huff_impl(HuffArgs a, int64_t T, const HuffPlan &p, cudaStream_t s) {
    for (int64_t t0 = 0; t0 < T; t0 += p.TB) {
        a.t0 = t0;
        a.ntok = (int)std::min<int64_t>(p.TB, T - t0);
        int rc = CBQ_ERR_UNSUPPORTED;
        switch (p.TB) {
            case 1: rc = launch_huff_t<1, XT>(a, p, s); break;
            case 2: rc = launch_huff_t<2, XT>(a, p, s); break;
            case 4: rc = launch_huff_t<4, XT>(a, p, s); break;
            case 8: rc = launch_huff_t<8, XT>(a, p, s); break;
        }
        if (rc != CBQ_OK) return rc;
    }
    return CBQ_OK;
}

bool tables_ok(const void *t) { return t != nullptr; }

}  // namespace

// ------------------------------------------------------------------- C ABI

extern "C" int64_t cbq_huff_tables_bytes(int64_t alphabet) {
    if (alphabet < 1 || alphabet > 65536) return -1;
    return (int64_t)sizeof(HuffTables) + cbq_host::align_up(alphabet * 2, 16);
}

extern "C" int cbq_huff_tables_build(const uint8_t *lengths, int64_t A, void *out, int64_t bytes) {
    if (!lengths || !out || A < 1 || A > 65536 || bytes < cbq_huff_tables_bytes(A)) return CBQ_ERR_ARG;
    std::memset(out, 0, (size_t)bytes);
    HuffTables *t = static_cast<HuffTables *>(out);
    uint16_t *syms = reinterpret_cast<uint16_t *>(t + 1);
    int64_t count[kMaxLen + 1] = {0};
    for (int64_t s = 0; s < A; ++s) {
        if (lengths[s] > kMaxLen) return CBQ_ERR_ARG;
        if (lengths[s]) ++count[lengths[s]];
    }
    // canonical first codes (RFC 1951 3.2.2) and the Kraft check
    uint64_t code = 0;
    int max_len = 0;
    int64_t used = 0;
    for (int L = 1; L <= kMaxLen; ++L) {
        code = (code + (uint64_t)count[L - 1]) << 1;
        t->first[L] = code;
        t->limit[L] = code + (uint64_t)count[L];
        if (t->limit[L] > (1ull << L)) return CBQ_ERR_ARG;  // over-subscribed code
        t->offset[L] = (int32_t)used;
        used += count[L];
        if (count[L]) max_len = L;
    }
    int64_t pos = 0;
    for (int L = 1; L <= kMaxLen; ++L)
        for (int64_t s = 0; s < A; ++s)
            if (lengths[s] == L) syms[pos++] = (uint16_t)s;
    for (int L = 1; L <= kLutBits; ++L)
        for (int64_t i = 0; i < count[L]; ++i) {
            const uint64_t c = t->first[L] + (uint64_t)i;
            const uint32_t sym = syms[t->offset[L] + i];
            const uint64_t base = c << (kLutBits - L), span = 1ull << (kLutBits - L);
            for (uint64_t k = 0; k < span; ++k) t->lut[base + k] = ((uint32_t)L << 16) | sym;
        }
    t->magic = kMagic;
    t->alphabet = (int32_t)A;
    t->max_len = max_len;
    t->n_used = (int32_t)used;
    return CBQ_OK;
}

extern "C" int cbq_huff_tables_max_len(const void *tables_host) {
    const HuffTables *t = static_cast<const HuffTables *>(tables_host);
    return (t && t->magic == kMagic) ? t->max_len : -1;
}

extern "C" int64_t cbq_huff_stream_bytes(int64_t stream_len) {
    if (stream_len < 0) return -1;
    return cbq_host::align_up(stream_len, 16) + 64;
}

extern "C" int64_t cbq_huff_chunk_count(int64_t M, int64_t K) {
    if (M < 0 || K < 0) return -1;
    return M * ((K + S - 1) / S);
}

extern "C" int64_t cbq_huff_chunk_table_words(int64_t M, int64_t K) {
    const int64_t n = cbq_huff_chunk_count(M, K);
    return n < 0 ? -1 : 2 * n;
}

extern "C" int cbq_huff_chunk_table(const uint8_t *stream_dev, int64_t stream_bytes,
                                    const void *tables_dev, const int64_t *rbs_dev, int64_t M,
                                    int64_t K, int64_t total_bits, uint32_t *chunk_dev,
                                    uint32_t *status_dev, void *stream) {
    if (M < 0 || K < 0 || total_bits < 0 || stream_bytes < cbq_huff_stream_bytes((total_bits + 7) / 8))
        return CBQ_ERR_ARG;
    if (M == 0 || K == 0) return CBQ_OK;
    if (!stream_dev || !tables_ok(tables_dev) || !rbs_dev || !chunk_dev) return CBQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(stream_dev) & 15) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    k_huff_chunks<<<(unsigned)((M + 127) / 128), 128, 0, s>>>(
        stream_dev, (uint64_t)stream_bytes / 4, static_cast<const HuffTables *>(tables_dev), rbs_dev, M, K, total_bits,
        chunk_dev, status_dev);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

extern "C" int64_t cbq_huff_decode_lut_bytes(void) { return (int64_t)kHfLutWords * 4; }

extern "C" int cbq_huff_build_decode_lut(const void *tables_dev, const float *codebook_dev, int64_t C,
                                         uint32_t *lut_dev, void *stream) {
    if (!tables_dev || !codebook_dev || !lut_dev || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(lut_dev) & 15) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CBQ_CUDA_TRY(cudaMemsetAsync(lut_dev, 0, (size_t)kHfLutWords * 4, s));
    k_huff_build_lut<<<1, 1024, 0, s>>>(static_cast<const HuffTables *>(tables_dev), codebook_dev, (int)C,
                                        lut_dev);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

extern "C" int64_t cbq_linear_huff_workspace_bytes(int64_t M, int64_t K, int64_t T) {
    if (M < 0 || K < 0 || T < 0) return -1;
    return huff_workspace_bytes(M, K, T);
}

extern "C" int cbq_linear_huff(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                               const uint8_t *stream_dev, int64_t stream_bytes,
                               const void *tables_dev, const uint32_t *lut_dev,
                               const int64_t *rbs_dev, const uint32_t *chunk_dev, int64_t total_bits,
                               const float *codebook_dev, int64_t C, int64_t M, int64_t K,
                               const float *bias_dev, void *out_dev, int out_dtype, int64_t ldo,
                               void *workspace_dev, int64_t workspace_bytes, uint32_t *status_dev,
                               void *stream) {
    if (T < 0 || M < 0 || K < 0 || C < 1 || C > 65536 || total_bits < 0) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (T == 0 || M == 0) return CBQ_OK;
    if (!out_dev || !codebook_dev || !x_dev || !stream_dev || !tables_ok(tables_dev) || !lut_dev ||
        !rbs_dev || !chunk_dev)
        return CBQ_ERR_ARG;
    if (ldx < K || ldo < M) return CBQ_ERR_ARG;
    if (stream_bytes < cbq_huff_stream_bytes((total_bits + 7) / 8)) return CBQ_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(stream_dev) & 15) || (reinterpret_cast<uintptr_t>(lut_dev) & 15))
        return CBQ_ERR_ARG;
    if (workspace_dev && workspace_bytes < huff_workspace_bytes(M, K, T)) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    HgPlan g;
    if (T == 1 && (reinterpret_cast<uintptr_t>(x_dev) & 15) == 0 && plan_hgemv(M, K, total_bits, g)) {
        HgArgs h{};
        h.x = x_dev; h.ldx = ldx; h.stream = stream_dev; h.stream_bytes = stream_bytes;
        h.tables = static_cast<const HuffTables *>(tables_dev); h.lut = lut_dev; h.rbs = rbs_dev;
        h.chunk = chunk_dev; h.total_bits = total_bits; h.codebook = codebook_dev; h.C = (int)C;
        h.M = (int)M; h.K = (int)K; h.nch = (int)((K + S - 1) / S); h.nseg = g.nseg;
        h.rows_per_cta = g.rows_per_cta; h.bias = bias_dev; h.out = out_dev; h.ldo = ldo;
        h.out_bf16 = out_dtype == CBQ_BF16; h.cap = g.cap; h.status = status_dev;
        h.m4 = 4u; h.m16 = 1u << 16;
        return x_dtype == CBQ_BF16 ? launch_hgemv<__nv_bfloat16>(h, g, s) : launch_hgemv<float>(h, g, s);
    }
    // Many bf16 tokens: transcode the stream once to fixed width (in the
    // workspace, after the split-row part) and run the tensor-core GEMM on
    // it, so each symbol is entropy-decoded once per call instead of once per
    // output tile.
    if (T >= kHuffGemmMinTokens && x_dtype == CBQ_BF16 && workspace_dev &&
        workspace_bytes >= huff_workspace_bytes(M, K, T) && K % (2 * S) == 0 && M % 128 == 0) {
        const HuffTables *tab = static_cast<const HuffTables *>(tables_dev);
        const int bits = bits_for_entries(std::max<int64_t>(C, 2));
        if (bits <= 14) {
            uint8_t *pk = static_cast<uint8_t *>(workspace_dev) + huff_split_bytes(M, K, T);
            uint32_t *pw = reinterpret_cast<uint32_t *>(pk);
            int rc = CBQ_ERR_ARG;
            switch (bits) {
#define CBQ_T(n) case n: rc = launch_transcode<n>(stream_dev, stream_bytes, tab, rbs_dev, chunk_dev, M, K, (int)C, \
                                                   pw, status_dev, s); break;
                CBQ_T(1) CBQ_T(2) CBQ_T(3) CBQ_T(4) CBQ_T(5) CBQ_T(6) CBQ_T(7)
                CBQ_T(8) CBQ_T(9) CBQ_T(10) CBQ_T(11) CBQ_T(12) CBQ_T(13) CBQ_T(14)
#undef CBQ_T
            }
            if (rc != CBQ_OK) return rc;
            rc = gemm_fixed(x_dev, T, ldx, pk, codebook_dev, C, bits, M, K, bias_dev, out_dev, out_dtype, ldo, s);
            if (rc != CBQ_ERR_UNSUPPORTED) return rc;
        }
    }
    HuffPlan p;
    if (!plan_huff(M, K, T, total_bits, x_dtype == CBQ_BF16 ? 2 : 4, p)) return CBQ_ERR_UNSUPPORTED;
    HuffArgs a{};
    a.x = x_dev; a.ldx = ldx; a.stream = stream_dev; a.stream_bytes = stream_bytes;
    a.tables = static_cast<const HuffTables *>(tables_dev); a.lut = lut_dev; a.rbs = rbs_dev;
    a.chunk = chunk_dev; a.total_bits = total_bits; a.codebook = codebook_dev; a.C = (int)C;
    a.M = (int)M; a.K = (int)K; a.nch = (int)((K + S - 1) / S); a.nseg = (a.nch + 31) / 32;
    a.bias = bias_dev; a.out = out_dev; a.ldo = ldo; a.out_bf16 = out_dtype == CBQ_BF16;
    a.cap = p.cap; a.status = status_dev;
    if (workspace_dev) {
        const int64_t pb = cbq_host::align_up(M * (int64_t)a.nseg * p.TB * 4, 256);
        a.part = static_cast<float *>(workspace_dev);
        a.cnt = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(workspace_dev) + pb);
    }
    if (x_dtype == CBQ_BF16) return linear_huff_impl<__nv_bfloat16>(a, T, p, s);
    return linear_huff_impl<float>(a, T, p, s);
}

extern "C" int cbq_embedding_huff(const int64_t *ids_dev, int64_t T, const uint8_t *stream_dev,
                                  int64_t stream_bytes, const void *tables_dev,
                                  const int64_t *rbs_dev, const uint32_t *chunk_dev,
                                  const float *codebook_dev, int64_t C, int64_t vocab, int64_t H,
                                  void *out_dev, int out_dtype, uint32_t *status_dev, void *stream) {
    if (T < 0 || vocab < 0 || H < 0 || C < 1 || C > 65536 || stream_bytes < 0) return CBQ_ERR_ARG;
    if (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16) return CBQ_ERR_ARG;
    if (T == 0 || H == 0) return CBQ_OK;
    if (!ids_dev || !stream_dev || !tables_ok(tables_dev) || !rbs_dev || !chunk_dev ||
        !codebook_dev || !out_dev)
        return CBQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(stream_dev) & 15) return CBQ_ERR_ARG;
    if (T > 0x7fffffff) return CBQ_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const HuffTables *tab = static_cast<const HuffTables *>(tables_dev);
    if (out_dtype == CBQ_F32)
        k_huff_embedding<float><<<(unsigned)T, 256, 0, s>>>(ids_dev, stream_dev,
                                                           (uint64_t)stream_bytes / 4, tab, rbs_dev,
                                                           chunk_dev, codebook_dev, (int)C, vocab,
                                                           H, static_cast<float *>(out_dev),
                                                           status_dev);
    else
        k_huff_embedding<__nv_bfloat16><<<(unsigned)T, 256, 0, s>>>(
            ids_dev, stream_dev, (uint64_t)stream_bytes / 4, tab, rbs_dev, chunk_dev, codebook_dev, (int)C, vocab, H,
            static_cast<__nv_bfloat16 *>(out_dev), status_dev);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

extern "C" int cbq_huff_decode_indices(const uint8_t *stream_dev, int64_t stream_bytes,
                                       const void *tables_dev, const int64_t *rbs_dev,
                                       const uint32_t *chunk_dev, int64_t M, int64_t K,
                                       uint16_t *idx_dev, uint32_t *status_dev, void *stream) {
    if (M < 0 || K < 0 || stream_bytes < 0) return CBQ_ERR_ARG;
    if (M == 0 || K == 0) return CBQ_OK;
    if (!stream_dev || !tables_ok(tables_dev) || !rbs_dev || !chunk_dev || !idx_dev) return CBQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(stream_dev) & 15) return CBQ_ERR_ARG;
    const int64_t n = M * ((K + S - 1) / S);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    k_huff_decode<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        stream_dev, (uint64_t)stream_bytes / 4, static_cast<const HuffTables *>(tables_dev), rbs_dev, chunk_dev, M, K, idx_dev,
        status_dev);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

extern "C" int cbq_huff_encode(const uint16_t *idx_dev, int64_t n, const uint32_t *code_dev,
                               const uint8_t *len_dev, const int64_t *starts_dev, uint8_t *out_dev,
                               int64_t out_bytes, void *stream) {
    if (n < 0 || out_bytes < 8 || (out_bytes & 3)) return CBQ_ERR_ARG;
    if (!out_dev || (reinterpret_cast<uintptr_t>(out_dev) & 3)) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CBQ_CUDA_TRY(cudaMemsetAsync(out_dev, 0, (size_t)out_bytes, s));
    if (n == 0) return CBQ_OK;
    if (!idx_dev || !code_dev || !len_dev || !starts_dev) return CBQ_ERR_ARG;
    k_huff_encode<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        idx_dev, n, code_dev, len_dev, starts_dev, reinterpret_cast<uint32_t *>(out_dev));
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}
