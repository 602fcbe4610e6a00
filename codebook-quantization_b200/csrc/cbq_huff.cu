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
// every 64th symbol of every row.  The GEMV then gives each thread one
// 64-symbol chunk: a persistent CTA stages a tile of RB rows (one contiguous
// bit range) into shared memory with cp.async.bulk, every thread decodes its
// chunk from a 64-bit MSB-first bit buffer fed by 32-bit shared loads, looks
// each code up in a shared 4096-entry table, gathers the fp32 codebook value
// from shared memory and accumulates against x (fp32 in shared memory, one
// padding word per 64 so that neighbouring chunks hit distinct banks).  Chunk
// sums are reduced per row by one warp in fixed order (deterministic).
#include <algorithm>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <numeric>

#include "cbq_common.cuh"

namespace {

using namespace cbq;

constexpr uint32_t kMagic = 0x48514243u;  // "CBQH"
constexpr int kLutBits = 12;
constexpr int kLutSize = 1 << kLutBits;
constexpr int kMaxLen = 32;
constexpr int S = CBQ_HUFF_CHUNK;          // symbols per chunk entry
constexpr int kMaxCbSmem = 16384;
constexpr int kMaxStages = 8;

// Host/device table blob (no pointers; copied verbatim to the device).
struct HuffTables {
    uint32_t magic;
    int32_t alphabet;
    int32_t max_len;
    int32_t n_used;
    uint64_t limit[kMaxLen + 1];   // first[L] + count[L]: one past the last length-L code
    uint64_t first[kMaxLen + 1];   // first canonical code of length L
    int32_t offset[kMaxLen + 1];   // index in syms[] of the first length-L symbol
    int32_t pad_[3];               // puts lut on a 16-byte boundary (read with 16-byte loads)
    uint32_t lut[kLutSize];        // (len << 16) | sym for codes <= 12 bits; 0 otherwise
    // uint16_t syms[n_used] follows: symbols in (length, code) order
};
static_assert(offsetof(HuffTables, lut) % 16 == 0, "lut must be 16-byte aligned for uint4 loads");
static_assert(offsetof(HuffTables, lut) == 688, "blob layout is part of the ABI (tests decode it)");
static_assert(sizeof(HuffTables) % 16 == 0, "blob alignment");

__host__ __device__ inline const uint16_t *blob_syms(const HuffTables *t) {
    return reinterpret_cast<const uint16_t *>(t + 1);
}

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

__device__ __forceinline__ uint32_t bswap32(uint32_t v) { return __byte_perm(v, 0, 0x0123); }

// 64-bit MSB-first bit buffer over 32-bit words of a byte stream.
// Invariant before each decode: nb >= 32 valid bits at the top of buf.
// Words at index >= nw read as zero, so a corrupt offset or stream can never
// read outside the buffer it was given.
struct BitBuf {
    const uint32_t *w;
    uint64_t wp;
    uint64_t nw;
    uint64_t buf;
    int nb;
    __device__ __forceinline__ uint32_t word(uint64_t i) const {
        return (i < nw) ? bswap32(w[i]) : 0u;
    }
    __device__ __forceinline__ void init(const uint32_t *base, uint64_t nwords, uint64_t pos) {
        w = base;
        nw = nwords;
        wp = pos >> 5;
        const int sk = (int)(pos & 31);
        const uint64_t v = ((uint64_t)word(wp) << 32) | word(wp + 1);
        buf = v << sk;
        nb = 64 - sk;
        wp += 2;
    }
    __device__ __forceinline__ void consume(int n) {
        buf <<= n;
        nb -= n;
        if (nb < 32) {
            buf |= (uint64_t)word(wp++) << (32 - nb);
            nb += 32;
        }
    }
};

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
    int64_t pos = start;
    uint32_t bad = 0;
    bool overflow = false;
    for (int64_t k = 0; k < K; ++k) {
        if ((k % S) == 0) {
            const int64_t rel = pos - start;
            overflow |= rel > 0xffffffffll;
            chunk[r * nch + k / S] = (uint32_t)rel;
        }
        int len;
        decode_sym(bb.buf, &st, gsyms, len);
        if (len == 0) { len = 1; ++bad; }
        bb.consume(len);
        pos += len;
    }
    if (bad) report(status, CBQ_FLAG_CORRUPT, (uint32_t)r);
    const bool last = (r + 1 == M);
    const bool end_ok = last ? (pos <= total_bits && pos > total_bits - 8) || (K == 0)
                             : (pos == rbs[r + 1]);
    if (!end_ok || overflow) report(status, CBQ_FLAG_ROW_END, (uint32_t)r);
}

// ---------------------------------------------------------------- fused GEMV

struct HuffArgs {
    const void *x;
    int64_t ldx;
    int64_t t0;
    int ntok;
    const uint8_t *stream;
    int64_t stream_bytes;
    const HuffTables *tables;
    const int64_t *rbs;
    const uint32_t *chunk;
    int64_t total_bits;
    const float *codebook;
    int C;
    int M, K;
    const float *bias;
    void *out;
    int64_t ldo;
    int RB, ntiles, nst;
    uint32_t stage_cap;
    uint32_t *status;
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <int TB, bool CBS>
__device__ __forceinline__ void huff_chunk_dot(const uint32_t *words, uint64_t nwords, uint64_t pos,
                                               int nsym,
                                               const SmemTables *st, const uint16_t *gsyms,
                                               const float *cb, uint32_t cmax, const float *xq,
                                               int XSH, float (&acc)[TB], uint32_t &bad) {
    BitBuf bb;
    bb.init(words, nwords, pos);
#pragma unroll 4
    for (int i = 0; i < nsym; ++i) {
        int len;
        uint32_t sym = decode_sym(bb.buf, st, gsyms, len);
        if (len == 0) { len = 1; ++bad; }
        bb.consume(len);
        const float wt = CBS ? cb[min(sym, cmax)] : __ldg(cb + min(sym, cmax));
#pragma unroll
        for (int t = 0; t < TB; ++t) acc[t] = fmaf(xq[t * XSH + i], wt, acc[t]);
    }
}

template <int TB, bool CBS, typename XT, typename OT>
__global__ void __launch_bounds__(kThreads, 1) k_linear_huff(const HuffArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int K = a.K;
    const int nch = (K + S - 1) / S;
    const int XSH = nch * (S + 1);
    const int RB = a.RB, nst = a.nst;
    const int tile_chunks = RB * nch;

    // Every region starts on a 128-byte boundary (the bulk-copy destination
    // needs 16); huff_smem() on the host mirrors this carve-up exactly.
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    int64_t *b0s = reinterpret_cast<int64_t *>(smem + 128);
    size_t off = 256;
    SmemTables *st = reinterpret_cast<SmemTables *>(smem + off);
    off += a128(sizeof(SmemTables));
    float *cb_s = reinterpret_cast<float *>(smem + off);
    if (CBS) off += a128((size_t)a.C * 4);
    float *xs = reinterpret_cast<float *>(smem + off);
    off += a128((size_t)TB * XSH * 4);
    float *P = reinterpret_cast<float *>(smem + off);
    off += a128((size_t)TB * tile_chunks * 4);
    uint8_t *stg = smem + off;

    if (tid == 0) {
        for (int s = 0; s < nst; ++s) mbar_init(&bar[s], 1);
        mbar_fence_init();
    }
    load_tables(st, a.tables);
    if (CBS)
        for (int i = tid; i < a.C; i += kThreads) cb_s[i] = a.codebook[i];
    const XT *x = static_cast<const XT *>(a.x);
    for (int i = tid; i < TB * K; i += kThreads) {
        const int t = i / K, k = i - t * K;
        const float v = (t < a.ntok) ? to_f32<XT>(x[(a.t0 + t) * a.ldx + k]) : 0.f;
        xs[t * XSH + (k / S) * (S + 1) + (k % S)] = v;
    }
    __syncthreads();

    const int my_tiles =
        (blockIdx.x < (unsigned)a.ntiles) ? (a.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    auto issue = [&](int j) {
        const int tile = blockIdx.x + j * gridDim.x;
        const int s = j % nst;
        const int r0 = tile * RB;
        const int rows = min(RB, a.M - r0);
        const int64_t sb = a.rbs[r0];
        const int64_t eb = (r0 + rows < a.M) ? a.rbs[r0 + rows] : a.total_bits;
        const int64_t b0 = (sb >> 3) & ~(int64_t)15;
        const int64_t b1 = (((eb + 7) >> 3) + 15 & ~(int64_t)15) + 32;
        if (b1 - b0 <= (int64_t)a.stage_cap && b1 <= a.stream_bytes && b0 >= 0) {
            b0s[s] = b0;
            mbar_arrive_expect_tx(&bar[s], (uint32_t)(b1 - b0));
            bulk_g2s(stg + (size_t)s * a.stage_cap, a.stream + b0, (uint32_t)(b1 - b0), &bar[s]);
        } else {
            b0s[s] = -1;  // tile too wide for a stage: decode it from global memory
            mbar_arrive(&bar[s]);
        }
    };
    if (tid == 0)
        for (int j = 0; j < min(nst, my_tiles); ++j) issue(j);

    const uint16_t *gsyms = blob_syms(a.tables);
    const float *cb = CBS ? cb_s : a.codebook;
    const uint32_t cmax = (uint32_t)(a.C - 1);
    OT *out = static_cast<OT *>(a.out);
    const int warp = tid >> 5, lane = tid & 31;
    int j = 0;
    for (; j < my_tiles; ++j) {
        const int s = j % nst;
        const bool ok = mbar_wait_bounded(&bar[s], (uint32_t)(j / nst) & 1u);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) report(a.status, CBQ_FLAG_TIMEOUT, 0u);
            break;
        }
        const int tile = blockIdx.x + j * gridDim.x;
        const int r0 = tile * RB;
        const int rows = min(RB, a.M - r0);
        const int nc = rows * nch;
        const int64_t b0 = b0s[s];
        const uint32_t *sw = reinterpret_cast<const uint32_t *>(stg + (size_t)s * a.stage_cap);
        for (int c = tid; c < nc; c += kThreads) {
            const int rho = c / nch, q = c - rho * nch;
            const int64_t r = r0 + rho;
            const int64_t abs_bit = a.rbs[r] + (int64_t)a.chunk[r * nch + q];
            const int nsym = min(S, K - q * S);
            float acc[TB];
#pragma unroll
            for (int t = 0; t < TB; ++t) acc[t] = 0.f;
            uint32_t bad = 0;
            const float *xq = xs + q * (S + 1);
            if (b0 >= 0)
                huff_chunk_dot<TB, CBS>(sw, a.stage_cap / 4, (uint64_t)(abs_bit - b0 * 8), nsym, st,
                                        gsyms, cb, cmax, xq, XSH, acc, bad);
            else
                huff_chunk_dot<TB, CBS>(reinterpret_cast<const uint32_t *>(a.stream),
                                        (uint64_t)a.stream_bytes / 4, (uint64_t)abs_bit, nsym, st,
                                        gsyms, cb, cmax, xq, XSH, acc, bad);
            if (bad) report(a.status, CBQ_FLAG_CORRUPT, (uint32_t)r);
#pragma unroll
            for (int t = 0; t < TB; ++t) P[t * tile_chunks + c] = acc[t];
        }
        __syncthreads();
        if (tid == 0 && j + nst < my_tiles) issue(j + nst);
        for (int p = warp; p < rows * TB; p += kThreads / 32) {
            const int rho = p / TB, t = p - rho * TB;
            if (t >= a.ntok) continue;
            const float *pp = P + t * tile_chunks + rho * nch;
            float sum = 0.f;
            for (int q = lane; q < nch; q += 32) sum += pp[q];
            sum = warp_sum(sum);
            if (lane == 0) {
                const int r = r0 + rho;
                if (a.bias) sum += a.bias[r];
                out[(a.t0 + t) * a.ldo + r] = from_f32<OT>(sum);
            }
        }
        __syncthreads();
    }
    if (j < my_tiles && tid == 0) {
        for (int jj = j; jj < min(j + nst, my_tiles); ++jj)
            mbar_wait_bounded(&bar[jj % nst], (uint32_t)(jj / nst) & 1u);
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
    int RB = 0, nst = 0, TB = 0, ntiles = 0, grid = 0;
    uint32_t stage_cap = 0;
    size_t smem = 0;
    bool cbs = true;
};

size_t huff_smem(int C, bool cbs, int K, int RB, int TB, int nst, uint32_t cap) {
    const int nch = (K + S - 1) / S;
    size_t s = 256 + a128(sizeof(SmemTables));
    if (cbs) s += a128((size_t)C * 4);
    s += a128((size_t)TB * nch * (S + 1) * 4);
    s += a128((size_t)TB * RB * nch * 4);
    s += (size_t)nst * cap;
    return s;
}

bool plan_huff(int64_t M, int64_t K, int64_t C, int64_t T, int64_t total_bits, HuffPlan &p) {
    if (M <= 0 || K <= 0 || M >= (1ll << 31) || K > (1 << 18)) return false;
    const int nch = (int)((K + S - 1) / S);
    const double avg = std::max(1.0, (double)total_bits / ((double)M * (double)K));
    int RB = std::min(64, 256 / std::gcd(nch, 256));
    auto cap_of = [&](int rb) {
        return (uint32_t)cbq_host::align_up((int64_t)(rb * (double)K * avg / 8.0 * 1.3) + 128, 128);
    };
    while (RB > 1 && cap_of(RB) > 48 * 1024) RB /= 2;
    const uint32_t cap = cap_of(RB);
    const bool cbs = C <= kMaxCbSmem;
    const size_t budget = (size_t)cbq_host::max_smem_optin() - 1024;
    int TB = 8;
    while (TB > 1 && TB > T) TB /= 2;
    while (TB > 1 && huff_smem((int)C, cbs, (int)K, RB, TB, 2, cap) > budget) TB /= 2;
    if (huff_smem((int)C, cbs, (int)K, RB, TB, 2, cap) > budget) return false;
    int nst = 2;
    while (nst < kMaxStages && huff_smem((int)C, cbs, (int)K, RB, TB, nst + 1, cap) <= budget) ++nst;
    p.RB = RB; p.TB = TB; p.nst = nst; p.stage_cap = cap; p.cbs = cbs;
    p.smem = huff_smem((int)C, cbs, (int)K, RB, TB, nst, cap);
    p.ntiles = (int)((M + RB - 1) / RB);
    p.grid = std::min(p.ntiles, cbq_host::sm_count());
    return true;
}

template <int TB, bool CBS, typename XT, typename OT>
int launch_huff_t(const HuffArgs &a, const HuffPlan &p, cudaStream_t s) {
    auto kern = k_linear_huff<TB, CBS, XT, OT>;
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
    kern<<<p.grid, kThreads, p.smem, s>>>(a);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

template <bool CBS, typename XT, typename OT>
int launch_huff_tb(const HuffArgs &a, const HuffPlan &p, cudaStream_t s) {
    switch (p.TB) {
        case 1: return launch_huff_t<1, CBS, XT, OT>(a, p, s);
        case 2: return launch_huff_t<2, CBS, XT, OT>(a, p, s);
        case 4: return launch_huff_t<4, CBS, XT, OT>(a, p, s);
        case 8: return launch_huff_t<8, CBS, XT, OT>(a, p, s);
    }
    return CBQ_ERR_UNSUPPORTED;
}

template <typename XT, typename OT>
int linear_huff_impl(HuffArgs a, int64_t T, const HuffPlan &p, cudaStream_t s) {
    for (int64_t t0 = 0; t0 < T; t0 += p.TB) {
        a.t0 = t0;
        a.ntok = (int)std::min<int64_t>(p.TB, T - t0);
        const int rc = p.cbs ? launch_huff_tb<true, XT, OT>(a, p, s)
                             : launch_huff_tb<false, XT, OT>(a, p, s);
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

extern "C" int cbq_linear_huff(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                               const uint8_t *stream_dev, int64_t stream_bytes,
                               const void *tables_dev, const int64_t *rbs_dev,
                               const uint32_t *chunk_dev, int64_t total_bits,
                               const float *codebook_dev, int64_t C, int64_t M, int64_t K,
                               const float *bias_dev, void *out_dev, int out_dtype, int64_t ldo,
                               uint32_t *status_dev, void *stream) {
    if (T < 0 || M < 0 || K < 0 || C < 1 || C > 65536 || total_bits < 0) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (T == 0 || M == 0) return CBQ_OK;
    if (!out_dev || !codebook_dev || !x_dev || !stream_dev || !tables_ok(tables_dev) || !rbs_dev ||
        !chunk_dev)
        return CBQ_ERR_ARG;
    if (ldx < K || ldo < M) return CBQ_ERR_ARG;
    if (stream_bytes < cbq_huff_stream_bytes((total_bits + 7) / 8)) return CBQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(stream_dev) & 15) return CBQ_ERR_ARG;
    HuffPlan p;
    if (!plan_huff(M, K, C, T, total_bits, p)) return CBQ_ERR_UNSUPPORTED;
    HuffArgs a{};
    a.x = x_dev; a.ldx = ldx; a.stream = stream_dev; a.stream_bytes = stream_bytes;
    a.tables = static_cast<const HuffTables *>(tables_dev); a.rbs = rbs_dev; a.chunk = chunk_dev;
    a.total_bits = total_bits; a.codebook = codebook_dev; a.C = (int)C; a.M = (int)M; a.K = (int)K;
    a.bias = bias_dev; a.out = out_dev; a.ldo = ldo; a.RB = p.RB; a.ntiles = p.ntiles;
    a.nst = p.nst; a.stage_cap = p.stage_cap; a.status = status_dev;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (x_dtype == CBQ_F32 && out_dtype == CBQ_F32) return linear_huff_impl<float, float>(a, T, p, s);
    if (x_dtype == CBQ_BF16 && out_dtype == CBQ_BF16)
        return linear_huff_impl<__nv_bfloat16, __nv_bfloat16>(a, T, p, s);
    if (x_dtype == CBQ_BF16 && out_dtype == CBQ_F32)
        return linear_huff_impl<__nv_bfloat16, float>(a, T, p, s);
    return linear_huff_impl<float, __nv_bfloat16>(a, T, p, s);
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
