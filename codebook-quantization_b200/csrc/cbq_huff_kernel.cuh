// cbq_huff_kernel.cuh -- fused canonical-Huffman decode-GEMV kernel (sm_100a).
//
// Work decomposition mirrors the fixed-width kernel (cbq_fixed_kernel.cuh): a
// unit is one 2048-symbol segment of one row = 32 chunks of 64 symbols, whose
// start bits come from the load-time chunk-entry table; every warp of the
// persistent grid owns a balanced contiguous range of units and streams each
// unit's bit range into a private shared-memory ring with cp.async.bulk (a unit
// wider than a slot is decoded straight from global memory instead); lane j
// decodes chunk j of the unit.
//
// Decoding: a 16384-entry first-level table indexed by the next 14 bits gives,
// for every code of length <= 14, the code length and -- when every codebook
// value is an exact bf16 (all lossless codebooks) -- the bf16 codebook value
// itself, so one shared-memory load yields the weight.  A 14-bit prefix of
// longer codes points into a second-level table indexed by the following
// `depth` bits (one more load; about 2% of symbols for bf16 N(0, 0.02)
// weights).  Prefixes whose second level would not fit, and bit patterns that
// match no code, fall to the canonical search: the smallest length L whose
// canonical range contains the next L bits, which gives the reference's
// result (src/compressed_matmul.c:148-186); a pattern matching no code yields
// symbol 0 and consumes one bit (the reference's guard, :183-185) and is
// counted in the status word.  The bit buffer is two 32-bit registers,
// refilled once per pair of symbols.
#pragma once
#include "cbq_common.cuh"

namespace cbq {

constexpr int kHfWarps = 16;
constexpr int kHfChunk = CBQ_HUFF_CHUNK;         // symbols per chunk (64)
constexpr int kHfSeg = 32 * kHfChunk;            // symbols per unit (2048)
constexpr int kHfSlots = 2;
static_assert((kHfWarps * kHfSlots + 1) * 8 <= 512 && kHfWarps * kHfSlots * 8 <= 512,
              "barriers and slot bases each occupy a 512-byte region of shared memory");
constexpr int kHfLutBits = 14;
constexpr int kHfLutSize = 1 << kHfLutBits;
constexpr int kHfSubMax = 6144;                  // second-level entries kept in shared memory
constexpr int kHfLutWords = kHfLutSize + 4 + kHfSubMax;   // device table: level 1, header, level 2
constexpr int kHfMaxLen = 32;

// Host/device table blob built from huff_lengths (layout is part of the ABI).
struct HuffTables {
    uint32_t magic;
    int32_t alphabet;
    int32_t max_len;
    int32_t n_used;
    uint64_t limit[kHfMaxLen + 1];   // first[L] + count[L]: one past the last length-L code
    uint64_t first[kHfMaxLen + 1];   // first canonical code of length L
    int32_t offset[kHfMaxLen + 1];   // index in syms[] of the first length-L symbol
    int32_t pad_[3];
    uint32_t lut[4096];              // (len << 16) | sym for codes <= 12 bits; 0 otherwise
    // uint16_t syms[n_used] follows: symbols in (length, code) order
};

__host__ __device__ inline const uint16_t *blob_syms(const HuffTables *t) {
    return reinterpret_cast<const uint16_t *>(t + 1);
}

// The decode table (device buffer built by cbq_huff_build_decode_lut):
//   words [0, 16384): first level, indexed by the next 14 bits.
//     (payload << 16) | len for a code of length 1..14;
//     (payload(0) << 16) | 1 where no code starts with the prefix (an
//       incomplete code): the reference's guard, symbol 0 consuming one bit;
//     (so the low 16 bits of every resolved entry are exactly its length);
//     (offset << 16) | 0x80 | (32 - depth) for a prefix of longer codes: the
//       code's entry is second-level word offset + (the depth bits after the
//       prefix), i.e. sub[offset + ((window << 14) >> (32 - depth))];
//     0 when that prefix's second-level table did not fit (canonical search).
//   word 16384: mode (1 = payload is the bf16 value, 0 = payload is the
//     symbol); word 16385: second-level entries used; word 16386: 1 when the
//     two levels decode every 32-bit window (no 0 entries).
//   words [16388, 16388 + 6144): second level, (payload << 16) | len
//     (len 15..32), or the guard entry above for bit patterns that match no
//     code.
struct HuffSlow {                     // shared copy of the canonical tables
    uint64_t limit[kHfMaxLen + 1];
    uint64_t first[kHfMaxLen + 1];
    int32_t offset[kHfMaxLen + 1];
    int32_t max_len;
};

__device__ __forceinline__ uint32_t bswap32(uint32_t v) { return __byte_perm(v, 0, 0x0123); }

// 64-bit MSB-first bit buffer (used by the table, decode and embedding
// kernels); words at index >= nw read as zero so a corrupt offset or stream
// never reads outside the buffer it was given.
struct BitBuf {
    const uint32_t *w;
    uint32_t wp;
    uint32_t nw;
    uint64_t buf;
    int nb;
    __device__ __forceinline__ uint32_t word(uint32_t i) const { return (i < nw) ? bswap32(w[i]) : 0u; }
    __device__ __forceinline__ void init(const uint32_t *base, uint32_t nwords, uint64_t pos) {
        w = base;
        nw = nwords;
        const uint64_t wq = pos >> 5;
        wp = (wq < nwords) ? (uint32_t)wq : nwords;
        const int sk = (int)(pos & 31);
        buf = (((uint64_t)word(wp) << 32) | word(wp + 1)) << sk;
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

// Two-register MSB-first bit buffer for the fused GEMV: `hi` holds the next
// 32 bits of the stream, nb >= 14 valid bits at every fast-path decode.
struct Bits32 {
    const uint32_t *w;
    uint32_t wp, nw;
    uint32_t hi, lo;
    int nb;
    __device__ __forceinline__ uint32_t word(uint32_t i) const { return (i < nw) ? bswap32(w[i]) : 0u; }
    __device__ __forceinline__ void init(const uint32_t *base, uint32_t nwords, uint64_t pos) {
        w = base;
        nw = nwords;
        const uint64_t wq = pos >> 5;
        wp = (wq < nwords) ? (uint32_t)wq : nwords;
        const uint32_t sk = (uint32_t)(pos & 31);
        const uint32_t w0 = word(wp), w1 = word(wp + 1);
        hi = __funnelshift_lc(w1, w0, sk);
        lo = w1 << sk;
        nb = 64 - (int)sk;
        wp += 2;
    }
    // Append one word below the valid bits (nb < 32 on entry).
    __device__ __forceinline__ void refill() {
        const uint32_t W = word(wp++);
        const uint64_t v = (((uint64_t)hi << 32) | lo) | ((uint64_t)W << (32 - nb));
        hi = (uint32_t)(v >> 32);
        lo = (uint32_t)v;
        nb += 32;
    }
    __device__ __forceinline__ void consume_short(int n) {   // n <= 31
        hi = __funnelshift_l(lo, hi, n);
        lo <<= n;
        nb -= n;
    }
    __device__ __forceinline__ void consume_any(int n) {     // n <= 32
        hi = __funnelshift_lc(lo, hi, n);
        lo = (n < 32) ? (lo << n) : 0u;
        nb -= n;
    }
};

// Canonical search on a 32-bit window: (symbol, length), length 0 if none.
__device__ __forceinline__ uint32_t huff_canonical(uint32_t w32, const HuffSlow *hs, const uint16_t *gsyms,
                                                   int from, int &len) {
    for (int L = from; L <= hs->max_len; ++L) {
        const uint64_t v = (uint64_t)(w32 >> (32 - L));
        if (v < hs->limit[L]) {
            len = L;
            return gsyms[hs->offset[L] + (uint32_t)(v - hs->first[L])];
        }
    }
    len = 0;
    return 0u;
}

struct HuffArgs {
    const void *x;
    int64_t ldx;
    int64_t t0;
    int ntok;
    const uint8_t *stream;
    int64_t stream_bytes;
    const HuffTables *tables;
    const uint32_t *lut;              // two-level decode table (+ header words)
    const int64_t *rbs;
    const uint32_t *chunk;
    int64_t total_bits;
    const float *codebook;
    int C;
    int M, K, nch, nseg;
    const float *bias;
    void *out;
    int64_t ldo;
    int out_bf16;
    float *part;
    uint32_t *cnt;
    uint32_t cap;                     // bytes per ring slot
    uint32_t *status;
};

template <typename XT> struct XLayoutH;
template <> struct XLayoutH<float> {          // 64 floats + 4 pad: lane stride 68 words
    static constexpr int kStride = 68;
    __device__ static int elem(int k) { return (k >> 6) * 68 + (k & 63); }
};
template <> struct XLayoutH<__nv_bfloat16> {  // 64 halves + 8 pad: lane stride 36 words
    static constexpr int kStride = 72;
    __device__ static int elem(int k) { return (k >> 6) * 72 + (k & 63); }
};

__device__ __forceinline__ void hload_x8(const float *xr, int e, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(xr + e);
    const float4 b = *reinterpret_cast<const float4 *>(xr + e + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void hload_x8(const __nv_bfloat16 *xr, int e, float (&v)[8]) {
    const uint4 a = *reinterpret_cast<const uint4 *>(xr + e);
    const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        v[2 * q] = __uint_as_float(u[q] << 16);
        v[2 * q + 1] = __uint_as_float(u[q] & 0xffff0000u);
    }
}

// A code whose 14-bit prefix has no first-level entry: second level, else the
// canonical search.  Consumes the code and leaves >= 32 valid bits.
template <bool VALUE>
__device__ __forceinline__ float huff_long(Bits32 &bb, uint32_t e, const uint32_t *sub, const HuffSlow *hs,
                                           const uint16_t *gsyms, const float *gcb, uint32_t cmax,
                                           uint32_t &bad, bool count) {
    if (bb.nb < 32) bb.refill();
    uint32_t e2 = 0;
    if (e & 0x80u) e2 = sub[(e >> 16) + ((bb.hi << kHfLutBits) >> (e & 0x3fu))];
    float wt;
    int len = (int)(e2 & 0x3fu);
    if (len) {
        wt = VALUE ? __uint_as_float(e2 & 0xffff0000u) : __ldg(gcb + min(e2 >> 16, cmax));
    } else {
        const uint32_t sym = huff_canonical(bb.hi, hs, gsyms, 1, len);
        if (len == 0) { len = 1; bad += count ? 1u : 0u; }
        wt = __ldg(gcb + min(sym, cmax));
    }
    bb.consume_any(len);
    if (bb.nb < 32) bb.refill();
    return wt;
}

// Decode up to 64 symbols of one chunk and accumulate against x.
template <int TB, typename XT, bool VALUE>
__device__ __forceinline__ void huff_chunk(const uint32_t *words, uint32_t nw, uint64_t pos, int nsym,
                                           const uint32_t *lut, const uint32_t *sub, const HuffSlow *hs,
                                           const uint16_t *gsyms, const float *gcb, uint32_t cmax,
                                           const XT *xs, int XS, int e0, float (&acc)[TB],
                                           uint32_t &bad) {
    Bits32 bb;
    bb.init(words, nw, pos);
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
        if (8 * g >= nsym) break;
        float xv[TB][8];
#pragma unroll
        for (int t = 0; t < TB; ++t) hload_x8(xs + t * XS, e0 + 8 * g, xv[t]);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if ((q & 1) == 0 && bb.nb < 32) bb.refill();   // >= 32 bits for every pair of symbols
            const uint32_t e = lut[bb.hi >> (32 - kHfLutBits)];
            const int len = (e & 0x80u) ? 0 : (int)(e & 0x3fu);
            float wt;
            if (len) {
                wt = VALUE ? __uint_as_float(e & 0xffff0000u) : __ldg(gcb + min(e >> 16, cmax));
                bb.consume_short(len);
            } else {
                wt = huff_long<VALUE>(bb, e, sub, hs, gsyms, gcb, cmax, bad, 8 * g + q < nsym);
            }
            if (8 * g + q < nsym) {
#pragma unroll
                for (int t = 0; t < TB; ++t) acc[t] = fmaf(xv[t][q], wt, acc[t]);
            }
        }
    }
}

// Write (or combine) the sum of one warp's piece [s_first, s] of row r.
template <int TB>
__device__ __forceinline__ void huff_finish_piece(const HuffArgs &a, const float (&tot)[TB], int64_t r,
                                                  int s_first, int s) {
    const int nseg = a.nseg;
    const float b = a.bias ? a.bias[r] : 0.f;
    auto store = [&](int64_t o, float v) {
        if (a.out_bf16) static_cast<__nv_bfloat16 *>(a.out)[o] = __float2bfloat16_rn(v);
        else static_cast<float *>(a.out)[o] = v;
    };
    if (s_first == 0 && s == nseg - 1) {
        for (int t = 0; t < a.ntok; ++t) store((a.t0 + t) * a.ldo + r, tot[t] + b);
        return;
    }
    float *pr = a.part + (size_t)r * nseg * TB;
    for (int t = 0; t < TB; ++t) {
        pr[s_first * TB + t] = tot[t];
        for (int s2 = s_first + 1; s2 <= s; ++s2) pr[s2 * TB + t] = 0.f;
    }
    __threadfence();
    const uint32_t add = (uint32_t)(s - s_first + 1);
    const uint32_t old = atomicAdd(&a.cnt[r], add);
    if (old + add == (uint32_t)nseg) {
        __threadfence();
        for (int t = 0; t < a.ntok; ++t) {
            float sum = 0.f;
            for (int s2 = 0; s2 < nseg; ++s2) sum += __ldcg(pr + s2 * TB + t);
            store((a.t0 + t) * a.ldo + r, sum + b);
        }
        // leave the row's pieces and its counter zero, so the workspace stays
        // zero-filled for the next call whatever its shape
        for (int i = 0; i < nseg * TB; ++i) pr[i] = 0.f;
        atomicExch(&a.cnt[r], 0u);
    }
}

template <int TB, typename XT, bool VALUE>
__device__ void huff_warp_loop(const HuffArgs &a, const XT *xs, int XS, const uint32_t *lut,
                               const uint32_t *sub, const HuffSlow *hs, uint8_t *ring, uint64_t *bars,
                               int64_t *b0s, int64_t u0, int64_t u1) {
    const int lane = threadIdx.x & 31;
    const int64_t n = u1 - u0;
    const int nseg = a.nseg, nch = a.nch, K = a.K;
    const uint32_t cmax = (uint32_t)(a.C - 1);
    const uint16_t *gsyms = blob_syms(a.tables);

    // Per unit, lane j needs the start bit of chunk 32s+j, and lane 0 also the
    // end of the unit (start of chunk 32s+32, or the row end).  Both are loaded
    // kHfSlots units ahead so their latency hides behind the decode.  Row and
    // segment are tracked with cursors (no divisions in the loop).
    auto lane_start = [&](int64_t r, int s) -> int64_t {
        const int q = 32 * s + lane;
        return (q < nch) ? a.rbs[r] + (int64_t)a.chunk[r * nch + q] : -1;
    };
    auto unit_end = [&](int64_t r, int s) -> int64_t {
        if (32 * s + 32 < nch) return a.rbs[r] + (int64_t)a.chunk[r * nch + 32 * s + 32];
        return (r + 1 < a.M) ? a.rbs[r + 1] : a.total_bits;
    };
    auto issue = [&](int slot, int64_t sb, int64_t eb) {     // lane 0 only
        const int64_t b0 = (sb >> 3) & ~(int64_t)15;
        const int64_t b1 = ((((eb + 7) >> 3) + 15) & ~(int64_t)15) + 32;
        if (sb >= 0 && eb >= sb && b1 - b0 <= (int64_t)a.cap && b1 <= a.stream_bytes) {
            b0s[slot] = b0;
            mbar_arrive_expect_tx(&bars[slot], (uint32_t)(b1 - b0));
            bulk_g2s(ring + (size_t)slot * a.cap, a.stream + b0, (uint32_t)(b1 - b0), &bars[slot]);
        } else {
            b0s[slot] = -1;                                // decode this unit from global memory
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bars[slot]))
                         : "memory");
        }
    };
    static_assert(kHfSlots == 2, "the prefetch queue below holds two units");
    int64_t r = u0 / nseg;
    int s = (int)(u0 - r * nseg);
    int64_t pr = r;                                        // cursor of the next unit to prefetch
    int ps = s;
    int64_t st0 = -1, st1 = -1;                            // this lane's start bit, per slot
    for (int64_t i = 0; i < n && i < kHfSlots; ++i) {
        const int64_t sb = lane_start(pr, ps);
        const int64_t eb = (lane == 0) ? unit_end(pr, ps) : 0;
        if (i == 0) st0 = sb; else st1 = sb;
        if (lane == 0) issue((int)i, sb, eb);
        if (++ps == nseg) { ps = 0; ++pr; }
    }
    __syncwarp();

    float acc[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) acc[t] = 0.f;
    int s_first = s;
    int slot = 0;
    uint32_t phase = 0;
    int64_t i = 0;
    for (; i < n; ++i) {
        const int64_t my_bit = slot ? st1 : st0;
        // prefetch offsets for the unit that will reuse this slot
        int64_t nx_sb = -1, nx_eb = 0;
        const bool more = i + kHfSlots < n;
        if (more) {
            nx_sb = lane_start(pr, ps);
            if (lane == 0) nx_eb = unit_end(pr, ps);
            if (++ps == nseg) { ps = 0; ++pr; }
        }
        const bool ok = mbar_wait_bounded(&bars[slot], phase);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) report(a.status, CBQ_FLAG_TIMEOUT, (uint32_t)r);
            break;
        }
        const int q = 32 * s + lane;                       // this lane's chunk
        uint32_t bad = 0;
        if (q < nch) {
            const int64_t b0 = b0s[slot];
            const int nsym = min(kHfChunk, K - q * kHfChunk);
            const int e0 = XLayoutH<XT>::elem(q * kHfChunk);
            if (b0 >= 0)
                huff_chunk<TB, XT, VALUE>(reinterpret_cast<const uint32_t *>(ring + (size_t)slot * a.cap),
                                          a.cap / 4, (uint64_t)(my_bit - 8 * b0), nsym, lut, sub, hs, gsyms,
                                          a.codebook, cmax, xs, XS, e0, acc, bad);
            else
                huff_chunk<TB, XT, VALUE>(reinterpret_cast<const uint32_t *>(a.stream),
                                          (uint32_t)min((int64_t)0xffffffff, a.stream_bytes / 4),
                                          (uint64_t)my_bit, nsym, lut, sub, hs, gsyms, a.codebook, cmax, xs,
                                          XS, e0, acc, bad);
        }
        if (bad) report(a.status, CBQ_FLAG_CORRUPT, (uint32_t)r);
        __syncwarp();
        if (more) {
            if (slot) st1 = nx_sb; else st0 = nx_sb;
            if (lane == 0) issue(slot, nx_sb, nx_eb);
        }
        if (s == nseg - 1 || i == n - 1) {
            float tot[TB];
#pragma unroll
            for (int t = 0; t < TB; ++t) tot[t] = warp_sum(acc[t]);
            if (lane == 0) huff_finish_piece<TB>(a, tot, r, s_first, s);
#pragma unroll
            for (int t = 0; t < TB; ++t) acc[t] = 0.f;
            s_first = 0;
        }
        if (++s == nseg) { s = 0; ++r; }
        if (++slot == kHfSlots) { slot = 0; phase ^= 1u; }
    }
    if (i < n && lane == 0) {
        for (int64_t j = i; j < n && j < i + kHfSlots; ++j) {
            mbar_wait_bounded(&bars[slot], phase);
            if (++slot == kHfSlots) { slot = 0; phase ^= 1u; }
        }
    }
}

__host__ __device__ inline size_t huff_prefix_bytes(int K, int TB, int xbytes) {
    const int nch = (K + kHfChunk - 1) / kHfChunk;
    const int stride = (xbytes == 4) ? 68 : 72;
    return 1024 + a128(sizeof(HuffSlow)) + a128((size_t)kHfLutSize * 4) + a128((size_t)kHfSubMax * 4) +
           a128((size_t)TB * nch * stride * xbytes);
}

template <int TB, typename XT>
__global__ void __launch_bounds__(kHfWarps * 32, 1) k_linear_huff(const HuffArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int nthreads = kHfWarps * 32;
    const int K = a.K;
    const int XS = a.nch * XLayoutH<XT>::kStride;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);                 // 16 x 2 barriers + 1
    int64_t *b0s = reinterpret_cast<int64_t *>(smem + 512);             // 16 x 2 slot bases
    HuffSlow *hs = reinterpret_cast<HuffSlow *>(smem + 1024);
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem + 1024 + a128(sizeof(HuffSlow)));
    uint32_t *sub = lut + kHfLutSize;                                    // a128(64 KB) == 64 KB
    XT *xs = reinterpret_cast<XT *>(reinterpret_cast<uint8_t *>(sub) + a128((size_t)kHfSubMax * 4));
    uint8_t *rings = smem + huff_prefix_bytes(K, TB, sizeof(XT));

    const int warp = tid >> 5;
    uint64_t *setup_bar = bars + kHfWarps * kHfSlots;       // one more barrier for the table copy
    if ((tid & 31) == 0) {
        for (int s = 0; s < kHfSlots; ++s) mbar_init(&bars[warp * kHfSlots + s], 1);
        if (tid == 0) mbar_init(setup_bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    const uint32_t nsub = min(a.lut[kHfLutSize + 1], (uint32_t)kHfSubMax);
    if (tid == 0) {                                           // decode tables, asynchronously
        const uint32_t sub_bytes = ((nsub * 4u) + 15u) & ~15u;
        mbar_arrive_expect_tx(setup_bar, kHfLutSize * 4 + sub_bytes);
        bulk_g2s(lut, a.lut, kHfLutSize * 4, setup_bar);
        if (sub_bytes) bulk_g2s(sub, a.lut + kHfLutSize + 4, sub_bytes, setup_bar);
    }
    for (int i = tid; i <= kHfMaxLen; i += nthreads) {
        hs->limit[i] = a.tables->limit[i];
        hs->first[i] = a.tables->first[i];
        hs->offset[i] = a.tables->offset[i];
    }
    if (tid == 0) hs->max_len = a.tables->max_len;
    const XT *x = static_cast<const XT *>(a.x);
#pragma unroll 4
    for (int i = tid; i < TB * K; i += nthreads) {
        const int t = i / K, k = i - t * K;
        xs[t * XS + XLayoutH<XT>::elem(k)] = (t < a.ntok) ? x[(a.t0 + t) * a.ldx + k] : XT(0.f);
    }
    const bool value_mode = a.lut[kHfLutSize] == 1u;
    const bool ok = mbar_wait_bounded(setup_bar, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) report(a.status, CBQ_FLAG_TIMEOUT, 0u);
        return;
    }

    const int64_t W = (int64_t)gridDim.x * kHfWarps;
    const int64_t gw = (int64_t)blockIdx.x * kHfWarps + warp;
    int64_t u0, u1;
    if (a.part) {
        const int64_t U = (int64_t)a.M * a.nseg;
        u0 = gw * U / W;
        u1 = (gw + 1) * U / W;
    } else {
        u0 = (gw * a.M / W) * a.nseg;
        u1 = ((gw + 1) * a.M / W) * a.nseg;
    }
    uint8_t *ring = rings + (size_t)warp * kHfSlots * a.cap;
    if (value_mode)
        huff_warp_loop<TB, XT, true>(a, xs, XS, lut, sub, hs, ring, bars + warp * kHfSlots,
                                     b0s + warp * kHfSlots, u0, u1);
    else
        huff_warp_loop<TB, XT, false>(a, xs, XS, lut, sub, hs, ring, bars + warp * kHfSlots,
                                      b0s + warp * kHfSlots, u0, u1);
}

}  // namespace cbq
