// cbq_gemm.cu -- fixed-width codebook GEMM for many tokens (prefill) on the
// 5th-generation tensor cores (sm_100a: tcgen05.mma, TMEM accumulators, TMA).
//
// y[t, r] = sum_k x[t, k] * cb[min(idx(r*K + k), C-1)] (+ bias[r]) for a bf16
// activation matrix x [T, K]; the weights never exist in memory as a matrix:
// each 128 x 64 weight tile is decoded from the packed LSB-first index stream
// (reference src/bitpack.py:32-94) straight into shared memory as bf16, in
// the layout the tensor core reads, once per output tile.
//
// One persistent CTA per SM walks output tiles of 128 weight rows x 256
// tokens.  Warp roles:
//   * warps 0-15: two decoder sets of 256 threads (two per tile row) take
//     alternate K steps; a thread decodes 32 of its row's 64 indices per step
//     (b 32-bit words from global memory, prefetched two of its steps ahead),
//     gathers bf16 codebook values from shared memory and stores its four
//     16-byte chunks of the row with the 128-byte swizzle; after the tile's
//     last step all 16 warps read the fp32 accumulator out of TMEM (warp w:
//     lanes 32*(w%4).., a quarter of the columns) and write y;
//   * warp 16: TMA loads of the x tile (256 tokens x 64 k, bf16, 128-byte
//     swizzle, no multicast) into the stage;
//   * warp 17: owns the TMEM allocation (256 columns = the 128 x 256 fp32
//     accumulator) and one elected thread issues 4 tcgen05.mma (M=128, N=256,
//     K=16) per stage, then tcgen05.commit to the stage's "empty" barrier.
// Four stages of (A 16 KB + B 32 KB) are in flight.  Every mbarrier wait is
// bounded; on a timeout the CTA records CBQ_FLAG_TIMEOUT, all roles stop at
// the next wait, and the TMEM is released before the kernel returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "cbq_common.cuh"

namespace {

using namespace cbq;

constexpr int kBM = 128, kBN = 256, kBK = 64;
// Two shapes of one kernel:
//   BN = 256 (prefill): output tiles of 128 rows x 256 tokens, 3 operand
//     stages (2 for b = 14), 2 packed tiles in flight;
//   BN = 16 / 32 / 64 (3..63 tokens, decode batches): one token tile, the
//     K range split over several CTAs (split-K) so every SM decodes, 4
//     operand stages and 4 packed tiles in flight (the decode and the index
//     stream, not the tensor core, bound these shapes).
template <int BITS, int BN> struct GemmCfg {
    static constexpr bool kSmall = BN < 256;
    static constexpr int kStages = kSmall ? 4 : (BITS <= 13 ? 3 : 2);
    static constexpr int kPStages = kSmall ? 4 : 2;              // packed-index tiles (two K steps each)
    static constexpr uint32_t kPRowBytes = 16u * BITS;           // 128 indices of one row
    static constexpr uint32_t kPBytes = kBM * kPRowBytes;         // one packed tile
    static constexpr uint32_t kBBytes = BN * kBK * 2;             // one x tile
    static constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;      // allocation granularity is 32 columns
};
constexpr int kSetThreads = 256;                      // a decoder set: two threads per tile row
constexpr int kSets = 2;                              // sets decode alternate K steps
constexpr int kDecoders = kSets * kSetThreads;
constexpr int kDecWarps = kDecoders / 32;
constexpr int kThreads = kDecoders + 64;              // + TMA warp + MMA warp
constexpr uint32_t kABytes = kBM * kBK * 2;           // 16 KB
constexpr int kMaxSplits = 4;                          // split-K: K ranges per output tile at most

struct GemmArgs {
    const uint8_t *packed;
    const float *codebook;
    int C, bits;
    int M, K, T;
    const float *bias;
    void *out;
    int64_t ldo;
    int out_bf16;
    int tiles_m, tiles_n;
    uint32_t cb_entries;              // bf16 codebook entries in shared memory (padded to 2^b)
    uint32_t *status;
    // split-K (BN < 256): the K steps of an output tile are split over
    // `splits` work items; each writes its partial tile (fp32) to part
    // [splits][tiles_n * BN][M] and counts its arrival per (tile, epilogue
    // warp) on cnt; the item that completes a warp's count adds the partials
    // in split order and writes y, then resets the count (left 0).
    int splits;
    float *part;
    uint32_t *cnt;
};

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    // K-major, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart.
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]);

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                 "[%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Width-W (4 <= W <= 32, power of two) read of this warp's 32 TMEM lanes.
template <int W>
__device__ __forceinline__ void tmem_ldw(uint32_t taddr, uint32_t (&v)[W]) {
    if constexpr (W == 32) tmem_ld32(taddr, v);
    else if constexpr (W == 16) tmem_ld16(taddr, v);
    else if constexpr (W == 8) tmem_ld8(taddr, v);
    else {
        uint32_t t[8];
        tmem_ld8(taddr, t);
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = t[j];
    }
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    uint16_t v;
    asm("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

// NW consecutive 32-bit words from shared address `addr`, whose offset from
// a 16-byte boundary is OFF bytes (known at compile time): the widest
// aligned loads, so lanes reading rows 16*b bytes apart hit few banks.
template <int NW, int OFF>
__device__ __forceinline__ void lds_words(uint32_t addr, uint32_t (&w)[NW + 1]) {
    int j = 0;
    int off = OFF;
#pragma unroll
    for (int it = 0; it < NW; ++it) {
        if (j >= NW) break;
        if (off % 16 == 0 && j + 4 <= NW) {
            uint32_t a0, a1, a2, a3;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3) : "r"(addr));
            w[j] = a0; w[j + 1] = a1; w[j + 2] = a2; w[j + 3] = a3;
            j += 4; addr += 16; off += 16;
        } else if (off % 8 == 0 && j + 2 <= NW) {
            uint32_t a0, a1;
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(a0), "=r"(a1) : "r"(addr));
            w[j] = a0; w[j + 1] = a1;
            j += 2; addr += 8; off += 8;
        } else {
            uint32_t a0;
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a0) : "r"(addr));
            w[j] = a0;
            j += 1; addr += 4; off += 4;
        }
    }
}

template <int BITS>
__device__ __forceinline__ uint32_t field32(const uint32_t (&w)[BITS + 1], int i) {
    const int bit = i * BITS, wi = bit >> 5, sh = bit & 31;
    constexpr uint32_t mask = (1u << BITS) - 1u;
    const uint32_t v = (sh + BITS <= 32) ? (w[wi] >> sh) : __funnelshift_r(w[wi], w[wi + 1], sh);
    return v & mask;
}

// Bounded wait shared by all roles: false once this CTA has given up.
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              const GemmArgs &a) {
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity)) return true;
    *abort_flag = 1;
    report(a.status, CBQ_FLAG_TIMEOUT, 0u);
    return false;
}

// Work item `tile` -> output tile (tm, tn), split sp and its K steps
// [kb, ke) (whole packed tiles: kb, ke even).
struct GemmItem {
    int tm, tn, sp, kb, ke;
};
__device__ __forceinline__ GemmItem gemm_item(const GemmArgs &a, int tile, int nk) {
    GemmItem it;
    const int per_m = a.tiles_n * a.splits;
    it.tm = tile / per_m;
    const int rem = tile - it.tm * per_m;
    it.tn = rem / a.splits;
    it.sp = rem - it.tn * a.splits;
    const int npair = nk / 2, ppw = (npair + a.splits - 1) / a.splits;
    it.kb = 2 * min(it.sp * ppw, npair);
    it.ke = 2 * min(it.sp * ppw + ppw, npair);
    return it;
}

template <int BITS, int BN>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_fixed(const __grid_constant__ CUtensorMap tmap_x,
                                                            const __grid_constant__ CUtensorMap tmap_p,
                                                            const GemmArgs a) {
    using Cfg = GemmCfg<BITS, BN>;
    constexpr int kStages = Cfg::kStages, kPStages = Cfg::kPStages;
    constexpr uint32_t kPRowBytes = Cfg::kPRowBytes, kPBytes = Cfg::kPBytes, kBBytes = Cfg::kBBytes;
    constexpr uint32_t kTmemCols = Cfg::kTmemCols;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base for the swizzled operand tiles
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = smem;                                       // kStages x 16 KB
    uint8_t *sB = sA + kStages * kABytes;                     // kStages x 32 KB
    uint8_t *sP = sB + kStages * kBBytes;                     // kPStages packed tiles
    uint16_t *scb = reinterpret_cast<uint16_t *>(sP + kPStages * a128(kPBytes));
    uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<uint8_t *>(scb) + a128(a.cb_entries * 2));
    uint64_t *full_a = bars, *full_b = bars + kStages, *empty = bars + 2 * kStages;
    uint64_t *full_p = bars + 3 * kStages, *empty_p = full_p + kPStages;
    uint64_t *acc_full = empty_p + kPStages, *acc_empty = acc_full + 1, *drain = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_launch_dependents();
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_a[s], kSetThreads);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kPStages; ++s) {
            mbar_init(&full_p[s], 1);
            mbar_init(&empty_p[s], kDecoders);               // both decoder sets read a packed tile
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kDecoders);
        mbar_init(drain, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == kDecWarps + 1) {                              // TMEM: the 128 x 256 fp32 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // bf16 codebook, padded to cb_entries with cb[C-1] (the reference's clamp)
    for (uint32_t c = tid; c < a.cb_entries; c += kThreads)
        scb[c] = __bfloat16_as_ushort(__float2bfloat16_rn(__ldg(a.codebook + min((int)c, a.C - 1))));
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int nk = a.K / kBK;
    const int ntiles = a.tiles_m * a.tiles_n * a.splits;

    if (warp < kDecWarps) {
        // ------------------------------------------------ decoders + epilogue
        // set g = t / 256 decodes the K steps k = g, g + 2, ...; within a set,
        // thread t: tile row r, half h of the row's 64 indices (BITS words,
        // 4 chunks of 16 bytes of the swizzled row)
        const int g = tid / kSetThreads, t = tid % kSetThreads;
        const int r = t & (kBM - 1), h = t >> 7;
        const uint32_t cb_s = smem_u32(scb);
        constexpr int NW = BITS;                              // words per half step (32 indices)
        int base_it = 0;                                      // stage uses before this tile
        uint32_t acc_phase = 0;
        bool go = true;
        pdl_wait();                                           // x and y belong to the stream's previous work
        for (int tile = blockIdx.x; tile < ntiles && go; tile += gridDim.x) {
            const GemmItem wi = gemm_item(a, tile, nk);
            const int tm = wi.tm, tn = wi.tn;
            uint32_t w[NW + 1];
            for (int k = wi.kb + g; k < wi.ke; k += kSets) {
                // this row's words of step k from the packed tile (two steps per tile)
                const int pi = (base_it + k - wi.kb) >> 1;    // packed tiles used before
                const int ps = pi % kPStages;
                if (!wait_or_abort(&full_p[ps], (pi / kPStages) & 1, abort_flag, a)) {
                    go = false;
                    break;
                }
                // set g reads the step k with k & 1 == g, warp-uniform h: the
                // offset's alignment class is fixed per warp
                const uint32_t pw = smem_u32(sP + (size_t)ps * a128(kPBytes)) + (uint32_t)r * kPRowBytes +
                                    (uint32_t)(k & 1) * (8u * BITS) + (uint32_t)h * (4u * BITS);
                constexpr int O1 = (4 * BITS) % 16, O2 = (8 * BITS) % 16, O3 = (12 * BITS) % 16;
                switch ((k & 1) * 2 + h) {
                    case 0: lds_words<NW, 0>(pw, w); break;
                    case 1: lds_words<NW, O1>(pw, w); break;
                    case 2: lds_words<NW, O2>(pw, w); break;
                    default: lds_words<NW, O3>(pw, w); break;
                }
                w[NW] = 0u;
                mbar_arrive(&empty_p[ps]);                    // words are in registers
                const int it = base_it + k - wi.kb;
                const int s = it % kStages;
                if (it >= kStages && !wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, abort_flag, a)) {
                    go = false;
                    break;
                }
                uint8_t *dst = sA + (size_t)s * kABytes + (size_t)r * 128;
#pragma unroll
                for (int c = 0; c < 4; ++c) {                 // 4 chunks of 8 bf16 (16 bytes)
                    uint32_t p[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t lo = lds_u16(cb_s + 2u * field32<BITS>(w, c * 8 + 2 * q));
                        const uint32_t hi = lds_u16(cb_s + 2u * field32<BITS>(w, c * 8 + 2 * q + 1));
                        p[q] = __byte_perm(lo, hi, 0x5410);
                    }
                    const int ch = 4 * h + c;
                    *reinterpret_cast<uint4 *>(dst + ((ch ^ (r & 7)) << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
                }
                fence_proxy_async_smem();                     // generic stores -> tensor-core reads
                mbar_arrive(&full_a[s]);
            }
            base_it += wi.ke - wi.kb;
            if (!go) break;
            // epilogue: TMEM lanes 32*(warp%4).. = tile rows; the four warps of
            // a lane quarter take BN/4 accumulator columns each
            if (!wait_or_abort(acc_full, acc_phase, abort_flag, a)) { go = false; break; }
            acc_phase ^= 1u;
            tc_fence_after();
            const int er = (warp & 3) * 32 + lane;
            const int64_t m = (int64_t)tm * kBM + er;
            const float b = a.bias ? a.bias[m] : 0.f;
            constexpr int kWc = BN / 4;                        // columns per warp
            constexpr int kCW = kWc < 32 ? kWc : 32;           // columns per TMEM load
            const int cbeg = (warp >> 2) * kWc;
            auto store_y = [&](int64_t tt, float y) {
                if (a.out_bf16) static_cast<__nv_bfloat16 *>(a.out)[tt * a.ldo + m] = __float2bfloat16_rn(y);
                else static_cast<float *>(a.out)[tt * a.ldo + m] = y;
            };
            if (a.splits == 1) {
#pragma unroll 1
                for (int c0 = cbeg; c0 < cbeg + kWc; c0 += kCW) {
                    uint32_t v[kCW];
                    tmem_ldw<kCW>(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
                    for (int j = 0; j < kCW; ++j) {
                        const int64_t tt = (int64_t)tn * BN + c0 + j;
                        if (tt < a.T) store_y(tt, __uint_as_float(v[j]) + b);
                    }
                }
                tc_fence_before();
                mbar_arrive(acc_empty);
            } else {
                // split-K: this warp's 32 rows x kWc columns as a partial tile
                const int64_t tpad = (int64_t)a.tiles_n * BN;
                uint32_t v[kWc];
#pragma unroll
                for (int c0 = 0; c0 < kWc; c0 += kCW) {
                    uint32_t t[kCW];
                    tmem_ldw<kCW>(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(cbeg + c0), t);
#pragma unroll
                    for (int j = 0; j < kCW; ++j) v[c0 + j] = t[j];
                }
                tc_fence_before();
                mbar_arrive(acc_empty);                       // the accumulator is in registers
#pragma unroll
                for (int j = 0; j < kWc; ++j)
                    a.part[((int64_t)wi.sp * tpad + (int64_t)tn * BN + cbeg + j) * a.M + m] = __uint_as_float(v[j]);
                __threadfence();
                __syncwarp();
                uint32_t old = 0;
                uint32_t *cw = a.cnt + ((int64_t)tm * a.tiles_n + tn) * kDecWarps + warp;
                if (lane == 0) old = atomicAdd(cw, 1u);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == (uint32_t)(a.splits - 1)) {          // this warp's partition is complete
                    __threadfence();
                    // every split's values of the partition, all loads issued
                    // first, then added in split order
                    float pv[kMaxSplits][kWc];
#pragma unroll
                    for (int sp = 0; sp < kMaxSplits; ++sp)
#pragma unroll
                        for (int j = 0; j < kWc; ++j)
                            pv[sp][j] = sp < a.splits
                                            ? __ldcg(a.part + ((int64_t)sp * tpad + (int64_t)tn * BN + cbeg + j) * a.M + m)
                                            : 0.f;
#pragma unroll
                    for (int j = 0; j < kWc; ++j) {
                        const int64_t tt = (int64_t)tn * BN + cbeg + j;
                        float y = 0.f;
#pragma unroll
                        for (int sp = 0; sp < kMaxSplits; ++sp)
                            if (sp < a.splits) y += pv[sp][j];
                        if (tt < a.T) store_y(tt, y + b);
                    }
                    if (lane == 0) *cw = 0u;
                }
            }
        }
    } else if (warp == kDecWarps) {
        // ------------------------------------------------------------ TMA (x)
        if (lane == 0) {
            int it = 0;
            bool go = true;
            pdl_wait();
            for (int tile = blockIdx.x; tile < ntiles && go; tile += gridDim.x) {
                const GemmItem wi = gemm_item(a, tile, nk);
                const int tm = wi.tm, tn = wi.tn;
                for (int k = wi.kb; k < wi.ke; ++k, ++it) {
                    if (((k - wi.kb) & 1) == 0) {             // packed tile of steps k, k+1
                        const int pi = it >> 1, ps = pi % kPStages;
                        if (pi >= kPStages &&
                            !wait_or_abort(&empty_p[ps], ((pi / kPStages) - 1) & 1, abort_flag, a)) {
                            go = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&full_p[ps], kPBytes);
                        tma_load_2d(sP + (size_t)ps * a128(kPBytes), &tmap_p, (k >> 1) * (int)kPRowBytes,
                                    tm * kBM, &full_p[ps]);
                    }
                    const int s = it % kStages;
                    if (it >= kStages && !wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, abort_flag, a)) {
                        go = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full_b[s], kBBytes);
                    tma_load_2d(sB + (size_t)s * kBBytes, &tmap_x, k * kBK, tn * BN, &full_b[s]);
                }
            }
            // No load may still be landing when the CTA exits: wait (bounded)
            // for the last load issued into every stage.
            for (int s = 0; s < kStages && s < it; ++s) {
                const int last = it - 1 - ((it - 1 - s) % kStages);   // last step that used stage s
                mbar_wait_bounded(&full_b[s], (last / kStages) & 1);
            }
            const int np = (it + 1) >> 1;                     // packed tiles issued
            for (int s = 0; s < kPStages && s < np; ++s) {
                const int last = np - 1 - ((np - 1 - s) % kPStages);
                mbar_wait_bounded(&full_p[s], (last / kPStages) & 1);
            }
        }
    } else {
        // ------------------------------------------------------------- MMA issue
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(kBM, BN);
            int it = 0, nt = 0;
            bool go = true;
            for (int tile = blockIdx.x; tile < ntiles && go; tile += gridDim.x, ++nt) {
                const GemmItem wi = gemm_item(a, tile, nk);
                if (nt > 0 && !wait_or_abort(acc_empty, (nt - 1) & 1, abort_flag, a)) { go = false; break; }
                tc_fence_after();
                for (int k = wi.kb; k < wi.ke; ++k, ++it) {
                    const int s = it % kStages;
                    const uint32_t ph = (it / kStages) & 1;
                    if (!wait_or_abort(&full_a[s], ph, abort_flag, a) ||
                        !wait_or_abort(&full_b[s], ph, abort_flag, a)) {
                        go = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + (size_t)s * kABytes), b0 = smem_u32(sB + (size_t)s * kBBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        mma_bf16(tmem, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32), idesc,
                                 (k > wi.kb || kk > 0) ? 1u : 0u);
                    mma_commit(&empty[s]);                    // frees the stage when these MMAs finish
                }
                if (!go) break;
                mma_commit(acc_full);                         // accumulator complete
            }
            if (!go || *abort_flag) {                         // gave up: let issued MMAs finish first
                mma_commit(drain);
                mbar_wait_bounded(drain, 0);
            }
        }
    }
    // every role is done (or gave up): release the TMEM
    tc_fence_before();
    __syncthreads();
    if (warp == kDecWarps + 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (EncodeTiledFn) nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

template <int BITS, int BN>
size_t gemm_smem_bytes(uint32_t cb_entries) {
    using Cfg = GemmCfg<BITS, BN>;
    return 1024 + (size_t)Cfg::kStages * (kABytes + Cfg::kBBytes) + Cfg::kPStages * a128(Cfg::kPBytes) +
           a128((size_t)cb_entries * 2) + 256;
}

template <int BITS, int BN>
int launch_gemm(const CUtensorMap &map, const CUtensorMap &pmap, GemmArgs a, cudaStream_t s) {
    const size_t smem = gemm_smem_bytes<BITS, BN>(a.cb_entries);
    if (smem > (size_t)cbq_host::max_smem_optin()) return CBQ_ERR_UNSUPPORTED;
    const int grid = (int)std::min<int64_t>((int64_t)a.tiles_m * a.tiles_n * a.splits, cbq_host::sm_count());
    auto kern = k_gemm_fixed<BITS, BN>;
    static std::mutex mu;
    static size_t configured[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CBQ_ERR_CUDA;
    {
        std::lock_guard<std::mutex> g(mu);
        if (configured[dev & 63] < smem) {
            CBQ_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            configured[dev & 63] = smem;
        }
    }
    CBQ_CUDA_TRY(cbq_host::launch_pdl(kern, dim3(grid), dim3(kThreads), smem, s, map, pmap, a));
    return CBQ_OK;
}

// Split count for the small-batch shape: the number of work items
// (row tiles x splits) that fills the SMs in the fewest waves per unit of
// work, at most one split per pair of K steps and at most kMaxSplits.
int choose_splits(int64_t tiles, int64_t npair) {
    // time ~ waves x (pairs of K steps per item + a fixed per-item cost of
    // about two pairs: pipeline refill and the partial-tile epilogue)
    const int64_t sms = cbq_host::sm_count();
    int best = 1;
    double best_cost = 1e30;
    for (int sp = 1; sp <= kMaxSplits && sp <= npair; ++sp) {
        const int64_t ppw = (npair + sp - 1) / sp;
        if ((int64_t)(sp - 1) * ppw >= npair) continue;           // an empty split
        const double waves = (double)((tiles * sp + sms - 1) / sms);
        const double cost = waves * ((double)ppw + 2.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = sp;
        }
    }
    return best;
}

// Tensor maps of the activations (bf16 [T, K], box BN x 64) and of the packed
// stream as a [M rows, K*bits/8 bytes] byte matrix (box 128 rows x 16*bits
// bytes = two K steps, a 16-byte multiple for every width).
bool gemm_maps(const void *x, int64_t T, int64_t ldx, const uint8_t *packed, int bits, int64_t M, int64_t K, int BN,
               CUtensorMap &map, CUtensorMap &pmap) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {kBK, (cuuint32_t)BN};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    const cuuint64_t row_bytes = (cuuint64_t)K * bits / 8;
    const cuuint64_t pdims[2] = {row_bytes, (cuuint64_t)M};
    const cuuint64_t pstrides[1] = {row_bytes};
    const cuuint32_t pbox[2] = {(cuuint32_t)(16 * bits), (cuuint32_t)kBM};
    return enc(&pmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(packed), pdims, pstrides, pbox, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
int launch_gemm_bits(int bits, const CUtensorMap &map, const CUtensorMap &pmap, const GemmArgs &a, cudaStream_t s) {
    switch (bits) {
#define CBQ_G(n) case n: return launch_gemm<n, BN>(map, pmap, a, s);
        CBQ_G(1) CBQ_G(2) CBQ_G(3) CBQ_G(4) CBQ_G(5) CBQ_G(6) CBQ_G(7)
        CBQ_G(8) CBQ_G(9) CBQ_G(10) CBQ_G(11) CBQ_G(12) CBQ_G(13) CBQ_G(14)
#undef CBQ_G
    }
    return CBQ_ERR_UNSUPPORTED;
}

}  // namespace

namespace cbq {

int64_t gemm_small_workspace_bytes(int64_t M, int64_t K, int64_t T) {
    if (T < 1 || T > 64 || M % kBM || K % (2 * kBK)) return 0;
    const int BN = T <= 32 ? 32 : 64;
    const int sp = choose_splits(M / kBM, K / (2 * kBK));
    if (sp == 1) return 0;
    return cbq_host::align_up((int64_t)sp * BN * M * 4, 256) + cbq_host::align_up((M / kBM) * kDecWarps * 4, 256);
}

// Small-batch decode-GEMM (3..64 bf16 tokens) on the tensor cores with
// split-K: one 32- or 64-token tile, each 128-row tile's K range split over
// several CTAs (their partial tiles in the workspace, combined in split
// order by the last one), so all SMs decode.  CBQ_ERR_UNSUPPORTED (nothing
// launched) outside its shapes or when the workspace is too small.
int gemm_small(const void *x, int64_t T, int64_t ldx, const uint8_t *packed, const float *cb, int64_t C, int bits,
               int64_t M, int64_t K, const float *bias, void *out, int out_dtype, int64_t ldo, void *ws,
               int64_t ws_bytes, cudaStream_t s) {
    if (bits < 1 || bits > 14 || M % kBM || K % (2 * kBK) || K <= 0 || T < 1 || T > 64 || M <= 0)
        return CBQ_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(packed) & 15))
        return CBQ_ERR_UNSUPPORTED;
    if (M >= (1ll << 31) || K >= (1ll << 31)) return CBQ_ERR_UNSUPPORTED;
    const int BN = T <= 32 ? 32 : 64;
    const int sp = choose_splits(M / kBM, K / (2 * kBK));
    const int64_t need = gemm_small_workspace_bytes(M, K, T);
    if (sp > 1 && (!ws || ws_bytes < need)) return CBQ_ERR_UNSUPPORTED;
    CUtensorMap map, pmap;
    if (!gemm_maps(x, T, ldx, packed, bits, M, K, BN, map, pmap)) return CBQ_ERR_UNSUPPORTED;
    GemmArgs a{};
    a.packed = packed; a.codebook = cb; a.C = (int)C; a.bits = bits;
    a.M = (int)M; a.K = (int)K; a.T = (int)T; a.bias = bias; a.out = out; a.ldo = ldo;
    a.out_bf16 = out_dtype == CBQ_BF16; a.tiles_m = (int)(M / kBM); a.tiles_n = 1;
    a.cb_entries = std::max<uint32_t>((uint32_t)C, 1u << bits); a.status = nullptr;
    a.splits = sp;
    if (sp > 1) {
        a.part = static_cast<float *>(ws);
        a.cnt = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) +
                                             cbq_host::align_up((int64_t)sp * BN * M * 4, 256));
    }
    return BN == 32 ? launch_gemm_bits<32>(bits, map, pmap, a, s) : launch_gemm_bits<64>(bits, map, pmap, a, s);
}

// Prefill GEMM entry used by cbq_linear_fixed for many tokens.  Returns
// CBQ_ERR_UNSUPPORTED (nothing launched) outside its shapes: bf16 x with
// 16-byte aligned rows, M % 128 == 0, K % 64 == 0, b <= 14.
int gemm_fixed(const void *x, int64_t T, int64_t ldx, const uint8_t *packed, const float *cb, int64_t C,
               int bits, int64_t M, int64_t K, const float *bias, void *out, int out_dtype, int64_t ldo,
               cudaStream_t s) {
    if (bits < 1 || bits > 14 || M % kBM || K % (2 * kBK) || K <= 0 || T <= 0 || M <= 0) return CBQ_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16 || (reinterpret_cast<uintptr_t>(packed) & 15))
        return CBQ_ERR_UNSUPPORTED;
    if (M >= (1ll << 31) || T >= (1ll << 31) || K >= (1ll << 31)) return CBQ_ERR_UNSUPPORTED;
    const uint32_t entries = std::max<uint32_t>((uint32_t)C, 1u << bits);
    EncodeTiledFn enc = encode_fn();
    if (!enc) return CBQ_ERR_UNSUPPORTED;
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {kBK, kBN};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return CBQ_ERR_UNSUPPORTED;
    // the packed stream as a [M rows, K*bits/8 bytes] byte matrix; a box is
    // 128 rows x 16*bits bytes = two K steps (16-byte multiple for every width)
    CUtensorMap pmap;
    const cuuint64_t row_bytes = (cuuint64_t)K * bits / 8;
    const cuuint64_t pdims[2] = {row_bytes, (cuuint64_t)M};
    const cuuint64_t pstrides[1] = {row_bytes};
    const cuuint32_t pbox[2] = {(cuuint32_t)(16 * bits), (cuuint32_t)kBM};
    if (enc(&pmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(packed), pdims, pstrides, pbox, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return CBQ_ERR_UNSUPPORTED;
    GemmArgs a{};
    a.packed = packed; a.codebook = cb; a.C = (int)C; a.bits = bits;
    a.M = (int)M; a.K = (int)K; a.T = (int)T; a.bias = bias; a.out = out; a.ldo = ldo;
    a.out_bf16 = out_dtype == CBQ_BF16; a.tiles_m = (int)(M / kBM); a.tiles_n = (int)((T + kBN - 1) / kBN);
    a.cb_entries = entries; a.status = nullptr; a.splits = 1;
    return launch_gemm_bits<kBN>(bits, map, pmap, a, s);
}

}  // namespace cbq
