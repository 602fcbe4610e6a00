// cbq_hgemv_kernel.cuh -- fused canonical-Huffman decode GEMV for one token
// (sm_100a).
//
// Same function as k_linear_huff (cbq_huff_kernel.cuh), built on the
// structure of the fixed-width one-token kernel (cbq_gemv_kernel.cuh):
//
//   * every CTA owns a block of whole rows; a unit is 32 consecutive 64-symbol
//     chunks of one row (2048 symbols), units are numbered segment-major and
//     dealt to the 16 warps in contiguous ranges, so lane j keeps the 64
//     activations of its chunk in registers across many rows;
//   * a unit's bit range (from the load-time chunk table) is bulk-copied into
//     the warp's ring slot, lane j decodes chunk j with the two-level table
//     (value mode: one shared load per symbol gives length and weight) in a
//     fully unrolled 64-symbol loop and multiplies against its registers;
//   * per-unit row sums go to shared memory and are added in segment order
//     after a CTA barrier (bitwise reproducible, no workspace);
//   * the decode tables and the first units are loaded before the
//     programmatic-dependent-launch wait, i.e. while the previous kernel on
//     the stream finishes.
// With a value-mode table (lossless codebooks), a lane runs four branch-free
// decoders over its chunk, from its codes 0, 16, 32 and 48 (the load-time
// quarter lengths): a symbol costs one shared load from the 14-bit first level
// and a predicated one from the second level; where some prefixes' second
// level did not fit (very deep codes, e.g. a 151936-row lm_head), the lanes
// that meet one take the canonical search under a per-step vote.  Bit
// patterns that match no code decode through guard entries as the reference
// does (symbol 0, one bit).  Symbol-payload tables take a one-decoder loop
// whose second-level load is voted per symbol; a partial last chunk of a row
// (K % 64 != 0) is decoded symbol by symbol.
#pragma once
#include "cbq_huff_kernel.cuh"

namespace cbq {

constexpr int kHgWarps = 16;
constexpr int kHgSlots = 2;
constexpr int kHgNF = kHfChunk;                  // symbols per lane per unit (one chunk)
constexpr int kHgSeg = 32 * kHgNF;               // symbols per unit
static_assert((kHgWarps * kHgSlots + 1) * 8 <= 512 && kHgWarps * kHgSlots * 8 <= 512,
              "barriers and slot bases each occupy a 512-byte region of shared memory");

struct HgArgs {
    const void *x;
    int64_t ldx;
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
    int rows_per_cta;
    const float *bias;
    void *out;
    int64_t ldo;
    int out_bf16;
    uint32_t cap;                     // bytes per ring slot
    uint32_t *status;
    // 4 and 1 << 16 as kernel arguments: the scalings written as products in
    // the decoders stay multiply(-high)-adds on the FMA pipe instead of shifts
    // and masks on the integer pipe, which the decode saturates
    uint32_t m4, m16;
};

__host__ __device__ inline size_t hg_part_bytes(int rows_per_cta, int nseg) {
    return a128((size_t)rows_per_cta * nseg * 4);
}
__host__ __device__ inline size_t hg_prefix_bytes(int rows_per_cta, int nseg) {
    return 1024 + hg_part_bytes(rows_per_cta, nseg) + a128(sizeof(HuffSlow)) + a128((size_t)kHfLutSize * 4) +
           a128((size_t)kHfSubMax * 4);
}

// A lane's 64 activations in registers: fp32, or for bf16 inputs the bf16
// pairs as loaded (32 registers; element i is widened where it is used, one
// shift or mask), which leaves the decoders room to overlap.
template <typename XT> struct HgX;
template <> struct HgX<float> {
    float v[kHgNF];
    __device__ __forceinline__ float operator[](int i) const { return v[i]; }
    __device__ __forceinline__ void load(const float *xr, int k0, int n) {
        if (n == kHgNF) {
            const float4 *p = reinterpret_cast<const float4 *>(xr + k0);
#pragma unroll
            for (int q = 0; q < kHgNF / 4; ++q) {
                const float4 f = __ldg(p + q);
                v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < kHgNF; ++i) v[i] = i < n ? __ldg(xr + k0 + i) : 0.f;
        }
    }
};
template <> struct HgX<__nv_bfloat16> {
    uint32_t v[kHgNF / 2];
    __device__ __forceinline__ float operator[](int i) const {
        return __uint_as_float((i & 1) ? (v[i >> 1] & 0xffff0000u) : (v[i >> 1] << 16));
    }
    __device__ __forceinline__ void load(const __nv_bfloat16 *xr, int k0, int n) {
        if (n == kHgNF) {
            const uint4 *p = reinterpret_cast<const uint4 *>(xr + k0);
#pragma unroll
            for (int q = 0; q < kHgNF / 8; ++q) {
                const uint4 f = __ldg(p + q);
                v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
            }
        } else {
            const uint16_t *h = reinterpret_cast<const uint16_t *>(xr + k0);
#pragma unroll
            for (int i = 0; i < kHgNF / 2; ++i) {
                const uint32_t lo = 2 * i < n ? (uint32_t)__ldg(h + 2 * i) : 0u;
                const uint32_t hi = 2 * i + 1 < n ? (uint32_t)__ldg(h + 2 * i + 1) : 0u;
                v[i] = lo | (hi << 16);
            }
        }
    }
};

__device__ __forceinline__ uint32_t hg_lds(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// MSB-first bit window for the one-token kernel: `hi` holds the next 32 bits
// (valid: nb of hi:lo, nb >= 32 before every symbol).  32-bit operations
// only.  RING: the words are in this warp's shared ring slot, which holds the
// unit plus at least 32 bytes, so a lane never reads past it; otherwise the
// words are in global memory and reads past `nw` return zero.
template <bool RING>
struct HgBits {
    const uint32_t *w;                  // global words (RING = false)
    uint32_t ws;                        // shared address of word 0 (RING = true)
    uint32_t wp, nw;
    uint32_t hi, lo;
    int nb;
    __device__ __forceinline__ uint32_t word(uint32_t i) const {
        if (RING) return bswap32(hg_lds(ws + 4u * i));
        return (i < nw) ? bswap32(w[i]) : 0u;
    }
    __device__ __forceinline__ void init(const uint32_t *base, uint32_t nwords, uint64_t pos) {
        w = base;
        ws = RING ? smem_u32(base) : 0u;
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
    __device__ __forceinline__ void top_up() {                 // keep >= 32 valid bits
        if (nb < 32) {
            const uint32_t W = word(wp++);
            hi |= W >> nb;
            lo = (W << 1) << (31 - nb);
            nb += 32;
        }
    }
    __device__ __forceinline__ void consume(uint32_t n) {       // n in [1, 32]
        hi = __funnelshift_lc(lo, hi, n);
        lo = (n < 32) ? (lo << n) : 0u;
        nb -= (int)n;
    }
};

// Decode the 64 symbols of one full chunk against xr.  Every window takes
// one shared load from the first level; the lanes in `mask` (those decoding
// a full chunk) take the second-level load together, predicated, only when
// one of them needs it.  CANON (a table whose second level did not fit for
// some prefixes): such a prefix's entry is 0 and takes the canonical search.
template <bool VALUE, bool RING, bool CANON, typename XV>
__device__ __forceinline__ float hg_chunk_fast(HgBits<RING> &bb, const XV &xr, uint32_t mask,
                                               uint32_t lut_s, uint32_t sub_s, const HuffSlow *hs,
                                               const uint16_t *gsyms, const float *gcb, uint32_t cmax) {
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int q = 0; q < kHgNF; ++q) {
        bb.top_up();
        uint32_t e = hg_lds(lut_s + ((bb.hi >> (32 - kHfLutBits)) << 2));
        if (__any_sync(mask, e & 0x80u)) {
            const bool ptr = (e & 0x80u) != 0;
            const uint32_t i2 = ptr ? (e >> 16) + ((bb.hi << kHfLutBits) >> (e & 0x3fu)) : 0u;
            const uint32_t e2 = hg_lds(sub_s + (i2 << 2));
            e = ptr ? e2 : e;
        }
        if (CANON && __any_sync(mask, e == 0u)) {   // only tables with prefixes left to the search
            if (e == 0u) {
                int L;
                uint32_t sym = huff_canonical(bb.hi, hs, gsyms, kHfLutBits + 1, L);
                if (L == 0) { L = 1; sym = 0; }                  // the reference's guard
                const uint32_t pay = VALUE ? (__float_as_uint(__ldg(gcb + min(sym, cmax))) >> 16) : sym;
                e = (pay << 16) | (uint32_t)L;
            }
        }
        const float wt = VALUE ? __uint_as_float(e & 0xffff0000u) : __ldg(gcb + min(e >> 16, cmax));
        bb.consume(e & 0x3fu);
        if (q & 1) acc1 = fmaf(xr[q], wt, acc1);
        else acc0 = fmaf(xr[q], wt, acc0);
    }
    return acc0 + acc1;
}

// ld.shared taken only when p is set; otherwise v keeps its value.
__device__ __forceinline__ uint32_t hg_lds_if(uint32_t p, uint32_t addr, uint32_t v) {
    asm("{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %2, 0;\n\t@q ld.shared.u32 %0, [%1];\n\t}"
        : "+r"(v) : "r"(addr), "r"(p));
    return v;
}

// One decoder of the fast path: a window of two byte-swapped stream words
// hi:lo, the raw word after them (nx), the shared address of the word after
// nx (wa) and a running bit count `pos` whose low five bits are the offset of
// the next code in hi (the funnel shift wraps).
struct HgDec {
    uint32_t hi, lo, nx, wa, pos;
    __device__ __forceinline__ void init(uint32_t addr, uint32_t bit) {   // addr: slot's word 0
        const uint32_t a0 = addr + ((bit >> 5) << 2);
        hi = bswap32(hg_lds(a0));
        lo = bswap32(hg_lds(a0 + 4u));
        nx = hg_lds(a0 + 8u);
        wa = a0 + 12u;
        pos = bit & 31u;
    }
    // One code in three phases, so that a lane's decoders can be interleaved
    // phase by phase (a warp issues in order: the loads of all decoders go
    // out before any of their results is needed).  Value-mode two-level table:
    //   * the first-level entry of a pointer prefix holds the second-level
    //     offset (bits 31:16) and 32 - depth (bits 4:0, which the wrapping
    //     funnel shift uses as its count); the second-level load is
    //     predicated on bit 7, so there is no branch;
    //   * an entry's low 16 bits are its code length: the weight is the entry
    //     with them cleared and the position advances by the length;
    //   * a code crossed into lo exactly when bit 5 of `pos` flipped; the
    //     window then moves one word and only those lanes load the word after
    //     it (needed at their next crossing at the earliest), one predicate
    //     for the four moves.
    uint32_t win, e;
    __device__ __forceinline__ void look(uint32_t lut_s, uint32_t m4) {
        win = __funnelshift_l(lo, hi, pos);
        e = hg_lds((win >> (32 - kHfLutBits)) * m4 + lut_s);
    }
    __device__ __forceinline__ void resolve(uint32_t sub_s, uint32_t m4, uint32_t m16) {
        const uint32_t a2 = (__umulhi(e, m16) + __funnelshift_r(win << kHfLutBits, 0u, e)) * m4 + sub_s;
        asm("{\n\t.reg .pred q;\n\t.reg .b32 t;\n\t"
            "and.b32 t, %0, 128;\n\tsetp.ne.u32 q, t, 0;\n\t"
            "@q ld.shared.u32 %0, [%1];\n\t}" : "+r"(e) : "r"(a2));
    }
    // A prefix whose second level did not fit in shared memory has entry 0:
    // those lanes (rare: the longest codes of tables with very deep ones)
    // take the canonical search, the others skip it together.
    __device__ __forceinline__ void canon(uint32_t mask, const HuffSlow *hs, const uint16_t *gsyms,
                                          const float *gcb, uint32_t cmax) {
        if (__any_sync(mask, e == 0u)) {
            if (e == 0u) {
                int L;
                uint32_t sym = huff_canonical(win, hs, gsyms, kHfLutBits + 1, L);
                if (L == 0) { L = 1; sym = 0; }                  // the reference's guard
                e = (__float_as_uint(__ldg(gcb + min(sym, cmax))) & 0xffff0000u) | (uint32_t)L;
            }
        }
    }
    __device__ __forceinline__ float consume(float x, float acc) {
        const uint32_t wt = e & 0xffff0000u;
        const uint32_t len = e - wt;
        const uint32_t np = pos + len;
        asm("{\n\t.reg .pred q;\n\t.reg .b32 t;\n\t"
            "xor.b32 t, %4, %5;\n\tand.b32 t, t, 32;\n\tsetp.ne.u32 q, t, 0;\n\t"
            "@q mov.b32 %0, %1;\n\t"
            "@q prmt.b32 %1, %2, 0, 0x0123;\n\t"
            "@q ld.shared.u32 %2, [%3];\n\t"
            "@q add.u32 %3, %3, 4;\n\t}"
            : "+r"(hi), "+r"(lo), "+r"(nx), "+r"(wa) : "r"(np), "r"(pos));
        pos = np;
        return fmaf(x, __uint_as_float(wt), acc);
    }
};

// The common case: a value-mode table and the chunk in the ring (CANON: some
// prefixes were left to the canonical search, see HgDec::canon).  Four
// independent decoders per lane,
// from the chunk's codes 0, 16, 32 and 48 (the packed quarter lengths of the
// load-time table), interleaved phase by phase against the same registers of
// x: straight-line code whose four dependency chains (window, first- and
// second-level loads) overlap.  The ring slot holds the unit plus 32 bytes,
// so every word a decoder reads is inside the slot.
template <bool CANON, typename XV>
__device__ __forceinline__ float hg_chunk_v2(uint32_t ws, uint32_t bit0, uint32_t quarters, const XV &xr,
                                             uint32_t lut_s, uint32_t sub_s, uint32_t m4, uint32_t m16,
                                             uint32_t mask, const HuffSlow *hs, const uint16_t *gsyms,
                                             const float *gcb, uint32_t cmax) {
    constexpr int kQ = kHgNF / 4;
    HgDec d[4];
    uint32_t b = bit0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        d[j].init(ws, b);
        b += (quarters >> (10 * j)) & 1023u;
    }
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < kQ; ++q) {
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j].look(lut_s, m4);
#pragma unroll
        for (int j = 0; j < 4; ++j) d[j].resolve(sub_s, m4, m16);
        if (CANON) {
#pragma unroll
            for (int j = 0; j < 4; ++j) d[j].canon(mask, hs, gsyms, gcb, cmax);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = d[j].consume(xr[j * kQ + q], acc[j]);
    }
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// Any chunk with any table (a partial last chunk, or a two-level table that
// left prefixes to the canonical search): symbol by symbol.
template <bool VALUE, typename XV>
__device__ __forceinline__ float hg_chunk_any(Bits32 &bb, const XV &xr, int nsym, const uint32_t *lut,
                                              const uint32_t *sub, const HuffSlow *hs, const uint16_t *gsyms,
                                              const float *gcb, uint32_t cmax, uint32_t &bad) {
    float acc = 0.f;
    for (int q = 0; q < nsym; ++q) {
        if (bb.nb < 32) bb.refill();
        const uint32_t e = lut[bb.hi >> (32 - kHfLutBits)];
        const int len = (e & 0x80u) ? 0 : (int)(e & 0x3fu);
        float wt;
        if (len) {
            wt = VALUE ? __uint_as_float(e & 0xffff0000u) : __ldg(gcb + min(e >> 16, cmax));
            bb.consume_short(len);
        } else {
            wt = huff_long<VALUE>(bb, e, sub, hs, gsyms, gcb, cmax, bad, true);
        }
        float xq = 0.f;
#pragma unroll
        for (int i = 0; i < kHgNF; ++i) xq = (i == q) ? xr[i] : xq;
        acc = fmaf(xq, wt, acc);
    }
    return acc;
}

template <typename XT, bool VALUE, bool CANON>
__device__ __forceinline__ void hg_loop(const HgArgs &a, const uint32_t *lut, const uint32_t *sub,
                                        const HuffSlow *hs, uint8_t *ring, uint64_t *bars, int64_t *b0s,
                                        float *part, int64_t m0, int nrows, int u0, int u1) {
    const int lane = threadIdx.x & 31;
    const int n = u1 - u0;
    const int nseg = a.nseg, nch = a.nch, K = a.K;
    const uint32_t cmax = (uint32_t)(a.C - 1);
    const uint16_t *gsyms = blob_syms(a.tables);
    const XT *x = static_cast<const XT *>(a.x);

    // Lane j of unit (row r, segment s) decodes chunk q = 32 s + j from bit
    // rbs[r] + chunk[r][q]; the unit spans up to the start of chunk 32 s + 32
    // (or the row's end).
    auto lane_start = [&](int64_t r, int s) -> int64_t {
        const int q = 32 * s + lane;
        return (q < nch) ? a.rbs[r] + (int64_t)a.chunk[r * nch + q] : -1;
    };
    // packed bit lengths of the quarters of this lane's chunk (fast path decoders)
    const uint32_t *quarter = a.chunk + (int64_t)a.M * nch;
    auto lane_quarters = [&](int64_t r, int s) -> uint32_t {
        const int q = 32 * s + lane;
        return (VALUE && q < nch) ? quarter[r * nch + q] : 0u;
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
            mbar_arrive(&bars[slot]);
        }
    };
    // units u = s * nrows + rl; cursors (pr, ps) of the next unit to prefetch
    int ps = u0 / nrows, prl = u0 - (u0 / nrows) * nrows;
    static_assert(kHgSlots == 2, "the start bits below are kept for two slots");
    int64_t st0 = -1, st1 = -1;                            // this lane's start bit, per slot
    uint32_t hf0 = 0, hf1 = 0;                             // and its chunk's quarter lengths
    for (int i = 0; i < n && i < kHgSlots; ++i) {
        const int64_t r = m0 + prl;
        const int64_t sb = lane_start(r, ps);
        const uint32_t hf = lane_quarters(r, ps);
        if (i == 0) { st0 = sb; hf0 = hf; } else { st1 = sb; hf1 = hf; }
        const int64_t eb = (lane == 0) ? unit_end(r, ps) : 0;
        if (lane == 0) issue(i, sb, eb);
        if (++prl == nrows) { prl = 0; ++ps; }
    }
    __syncwarp();
    pdl_wait();                                            // activations come from the previous kernel

    HgX<XT> xr;
    int xs = -1;
    int s = u0 / nrows, rl = u0 - (u0 / nrows) * nrows;
    int slot = 0;
    uint32_t phase = 0;
    int i = 0;
    for (; i < n; ++i) {
        const int q = 32 * s + lane;                       // this lane's chunk
        const int nsym = q < nch ? min(kHgNF, K - q * kHgNF) : 0;
        if (s != xs) {
            if (nsym > 0) xr.load(x, q * kHgNF, nsym);
            xs = s;
        }
        const int64_t my_bit = slot ? st1 : st0;
        const uint32_t my_quarters = slot ? hf1 : hf0;
        int64_t nx_sb = -1, nx_eb = 0;
        uint32_t nx_hf = 0;
        const bool more = i + kHgSlots < n;
        if (more) {                                        // offsets of the unit that reuses this slot
            const int64_t r2 = m0 + prl;
            nx_sb = lane_start(r2, ps);
            nx_hf = lane_quarters(r2, ps);
            if (lane == 0) nx_eb = unit_end(r2, ps);
            if (++prl == nrows) { prl = 0; ++ps; }
        }
        const bool ok = mbar_wait_bounded(&bars[slot], phase);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) report(a.status, CBQ_FLAG_TIMEOUT, (uint32_t)(m0 + rl));
            break;
        }
        uint32_t bad = 0;
        float acc = 0.f;
        // lanes that decode a full chunk from the ring / from global memory:
        // each group runs the fast loop, whose votes include only its lanes
        const int64_t b0u = b0s[slot];
        const uint32_t fast_ring = __ballot_sync(0xffffffffu, nsym == kHgNF && b0u >= 0);
        const uint32_t fast_glob = __ballot_sync(0xffffffffu, nsym == kHgNF && b0u < 0);
        if (nsym > 0) {
            const int64_t b0 = b0u;
            const uint32_t *wbase = b0 >= 0 ? reinterpret_cast<const uint32_t *>(ring + (size_t)slot * a.cap)
                                            : reinterpret_cast<const uint32_t *>(a.stream);
            const uint32_t nw = b0 >= 0 ? a.cap / 4 : (uint32_t)min((int64_t)0xffffffff, a.stream_bytes / 4);
            const uint64_t pos = b0 >= 0 ? (uint64_t)(my_bit - 8 * b0) : (uint64_t)my_bit;
            if (VALUE && nsym == kHgNF && b0 >= 0) {
                acc = hg_chunk_v2<CANON>(smem_u32(wbase), (uint32_t)pos, my_quarters, xr, smem_u32(lut),
                                         smem_u32(sub), a.m4, a.m16, fast_ring, hs, gsyms, a.codebook, cmax);
            } else if (nsym == kHgNF && b0 >= 0) {
                HgBits<true> bb;
                bb.init(wbase, nw, pos);
                acc = hg_chunk_fast<VALUE, true, CANON>(bb, xr, fast_ring, smem_u32(lut), smem_u32(sub), hs,
                                                        gsyms, a.codebook, cmax);
            } else if (nsym == kHgNF) {
                HgBits<false> bb;
                bb.init(wbase, nw, pos);
                acc = hg_chunk_fast<VALUE, false, CANON>(bb, xr, fast_glob, smem_u32(lut), smem_u32(sub), hs,
                                                         gsyms, a.codebook, cmax);
            } else {
                Bits32 bb;
                bb.init(wbase, nw, pos);
                acc = hg_chunk_any<VALUE>(bb, xr, nsym, lut, sub, hs, gsyms, a.codebook, cmax, bad);
            }
        }
        if (bad) report(a.status, CBQ_FLAG_CORRUPT, (uint32_t)(m0 + rl));
        __syncwarp();
        if (more) {
            if (slot) { st1 = nx_sb; hf1 = nx_hf; } else { st0 = nx_sb; hf0 = nx_hf; }
            if (lane == 0) issue(slot, nx_sb, nx_eb);
        }
        const float tot = warp_sum(acc);
        if (lane == 0) part[(size_t)rl * nseg + s] = tot;
        if (++rl == nrows) { rl = 0; ++s; }
        if (++slot == kHgSlots) { slot = 0; phase ^= 1u; }
    }
    if (i < n && lane == 0) {   // timed out: wait (bounded) for this warp's copies still in flight
        for (int j = i; j < n && j < i + kHgSlots; ++j) {
            mbar_wait_bounded(&bars[slot], phase);
            if (++slot == kHgSlots) { slot = 0; phase ^= 1u; }
        }
    }
}

template <typename XT>
__global__ void __launch_bounds__(kHgWarps * 32, 1) k_gemv_huff(const HgArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5;
    const int64_t m0 = (int64_t)blockIdx.x * a.rows_per_cta;
    if (m0 >= a.M) return;
    const int nrows = (int)min((int64_t)a.rows_per_cta, (int64_t)a.M - m0);
    const int nseg = a.nseg;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    int64_t *b0s = reinterpret_cast<int64_t *>(smem + 512);
    float *part = reinterpret_cast<float *>(smem + 1024);
    HuffSlow *hs = reinterpret_cast<HuffSlow *>(smem + 1024 + hg_part_bytes(a.rows_per_cta, nseg));
    uint32_t *lut = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(hs) + a128(sizeof(HuffSlow)));
    uint32_t *sub = lut + kHfLutSize;                                    // a128(64 KB) == 64 KB
    uint8_t *rings = smem + hg_prefix_bytes(a.rows_per_cta, nseg);

    uint64_t *setup_bar = bars + kHgWarps * kHgSlots;
    if ((tid & 31) == 0) {
        for (int s = 0; s < kHgSlots; ++s) mbar_init(&bars[warp * kHgSlots + s], 1);
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
    for (int i = tid; i <= kHfMaxLen; i += kHgWarps * 32) {
        hs->limit[i] = a.tables->limit[i];
        hs->first[i] = a.tables->first[i];
        hs->offset[i] = a.tables->offset[i];
    }
    if (tid == 0) hs->max_len = a.tables->max_len;
    const bool value_mode = a.lut[kHfLutSize] == 1u;
    const bool complete = a.lut[kHfLutSize + 2] == 1u;     // no prefix left to the canonical search
    const bool ok = mbar_wait_bounded(setup_bar, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) report(a.status, CBQ_FLAG_TIMEOUT, 0u);
        return;
    }

    const int U = nrows * nseg;
    const int u0 = (int)((int64_t)warp * U / kHgWarps);
    const int u1 = (int)((int64_t)(warp + 1) * U / kHgWarps);
    uint8_t *ring = rings + (size_t)warp * kHgSlots * a.cap;
    uint64_t *wb = bars + warp * kHgSlots;
    int64_t *wb0 = b0s + warp * kHgSlots;
    if (value_mode && complete)
        hg_loop<XT, true, false>(a, lut, sub, hs, ring, wb, wb0, part, m0, nrows, u0, u1);
    else if (value_mode)
        hg_loop<XT, true, true>(a, lut, sub, hs, ring, wb, wb0, part, m0, nrows, u0, u1);
    else
        hg_loop<XT, false, true>(a, lut, sub, hs, ring, wb, wb0, part, m0, nrows, u0, u1);
    __syncthreads();
    for (int r = tid; r < nrows; r += kHgWarps * 32) {
        float sum = 0.f;
        for (int q = 0; q < nseg; ++q) sum += part[(size_t)r * nseg + q];
        const int64_t row = m0 + r;
        const float v = sum + (a.bias ? a.bias[row] : 0.f);
        if (a.out_bf16) static_cast<__nv_bfloat16 *>(a.out)[row] = __float2bfloat16_rn(v);
        else static_cast<float *>(a.out)[row] = v;
    }
}

}  // namespace cbq
