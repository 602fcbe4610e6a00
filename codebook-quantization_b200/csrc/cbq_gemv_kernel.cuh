// cbq_gemv_kernel.cuh -- fixed-width decode GEMV for one or two tokens
// (sm_100a).
//
// out[t, r] = sum_k x[t, k] * cb[min(idx(r*K + k), C-1)], idx LSB-first b-bit
// fields (reference src/bitpack.py:32-94, src/compressed_matmul.c:334-347).
//
// The hot loop is bound by the integer pipe and by shared-memory wavefronts,
// so this kernel spends as few of both as it can per index:
//
//   * Activations live in registers.  Every CTA owns a block of whole rows;
//     inside it the (row, 1024-index segment) units are numbered
//     segment-major and dealt to the warps in contiguous ranges, so a warp
//     keeps the 32 activations of its lane's share of one segment in
//     registers for many rows in a row.  Each unit's per-row sum goes to
//     shared memory; after a CTA barrier the segment sums of every row are
//     added in segment order (bitwise reproducible, no workspace, no atomics).
//   * The codebook address costs two multiply-adds (FMA pipe) and one min
//     (integer pipe).  The first H entries are replicated once per lane
//     (entry c of lane j at c*128 + 4j: always bank j) and the other entries
//     follow as a single copy (entry c >= H at H*128 + (c-H)*4), so
//         addr(c) = min(c*128 + 4j, c*4 + H*124)
//     picks the replicated copy exactly when c < H.  For b <= 14 the single
//     copy is padded to 2^b entries with cb[C-1], which is the reference's
//     clamp idx >= C -> C-1 without an instruction.  The multipliers arrive as
//     kernel arguments so the compiler keeps them as multiply-adds.
//   * Each warp streams its units through a private ring of shared-memory
//     slots (one cp.async.bulk per unit, completing on the slot's mbarrier)
//     and decodes two rows of a segment at once where it can; the first
//     copies are issued before the codebook is built so that the DRAM latency
//     overlaps the table fill, and with programmatic dependent launch both
//     happen while the previous kernel on the stream is still finishing.
#pragma once
#include <type_traits>

#include "cbq_common.cuh"

namespace cbq {

#ifndef CBQ_GV_WARPS
#define CBQ_GV_WARPS 16
#endif
#ifndef CBQ_GV_PAIR
#define CBQ_GV_PAIR 1
#endif
constexpr int kGvWarps = CBQ_GV_WARPS;   // warps per CTA
// A unit is NF indices per lane (32 * NF per warp) of one row: NF = 32 with
// three ring slots per warp, or NF = 64 with two (fewer per-unit costs for
// long rows of work, same bytes in flight).
template <int NF> struct GvCfg {
    static_assert(NF == 32 || NF == 64, "units of 32 or 64 indices per lane");
    static constexpr int kSeg = 32 * NF;
    static constexpr int kSlots = NF == 32 ? 3 : 2;
};
constexpr int kGvMaxSlots = 3;
constexpr size_t kGvBarBytes = a128((size_t)kGvWarps * kGvMaxSlots * 8);   // one mbarrier per slot
static_assert(kGvWarps * 32 <= 1024, "gemv launch shape");

constexpr int kGvMaxMats = 3;

// One matrix of a launch.  Several matrices that share K, the bit width, the
// codebook and the activations (q/k/v, gate/up) are decoded by one launch.
struct GemvMat {
    const uint8_t *packed;
    void *out;           // [T, ldo] in the output dtype
    const float *bias;   // [M] or null
    const void *resid;   // EPI_RESIDUAL: [T, ldo] in the output dtype (may alias out)
    int64_t ldo;
    int M;
};

enum GemvEpi : int {
    kEpiStore = 0,       // out = acc (+ bias)
    kEpiResidual = 1,    // out = resid + round(acc + bias)      (the residual stream update)
    kEpiSiluMul = 2,     // two matrices of equal M: out0 = round(silu(round(g)) * round(u))
    kEpiPeer = 3,        // tensor parallelism: the partial product goes to every rank's slot
};

constexpr int kGvMaxPeers = 8;

// kEpiPeer: rank s's partial rows go to slot s of every rank's all-reduce
// buffer (peer memory over NVLink), then every CTA adds its row count to
// each rank's arrival counter for slot s (system-scope release); the
// consumer (cbq_rmsnorm_allreduce) waits for the counters and sums the slots.
struct GemvPeers {
    void *slot[kGvMaxPeers];          // rank p's slot for this rank, [T, ldo] in the output dtype
    uint32_t *count[kGvMaxPeers];     // rank p's arrival counter for this rank
    int world;
    // Flagged form (counts unused): every 64-bit slot word carries 32 bits of
    // data and the step's epoch in its high half, stored with one relaxed
    // system-scope 64-bit store, so a reader that sees the epoch sees the
    // data of the same store (no fence, no counter).  bf16: word t * ldo/2 +
    // row/2 holds rows (row, row + 1); fp32: word t * ldo + row.
    const uint32_t *ll_epoch;
};

__device__ __forceinline__ void st_relaxed_sys_u64(void *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const void *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Optional RMSNorm of the launch's updated rows (kEpiResidual with one
// matrix, or kEpiPeer), done by the CTA that finishes last: every CTA fences
// its stores and counts itself on `arrive`; the one that brings the count to
// the number of CTAs normalizes the T rows of n = M values (for kEpiPeer after
// waiting, bounded, for every rank's partial rows in this rank's slots and
// adding them to the residual stream in rank order) and resets the count.
// Values equal cbq_rmsnorm / cbq_rmsnorm_allreduce (same reduction order).
struct GemvNorm {
    uint32_t *arrive;          // null: no norm
    const float *w;            // norm weight [M] (may be null)
    float eps;
    void *out;                 // [T, ldn] normalized rows, output dtype
    int64_t ldn;
    void *resid;               // the residual stream [T, ldr] (kEpiResidual: mat[0].out)
    int64_t ldr;
    const void *slots;         // kEpiPeer: this rank's slots, slot p row t at (p * T + t) * ldo
    const uint32_t *counts;    // kEpiPeer: this rank's arrival counters [world]
    const uint32_t *epoch;     // kEpiPeer: counters are complete at epoch * expect
    uint32_t expect;
};

struct GemvArgs {
    const void *x;
    int64_t ldx;
    int64_t t0;          // first token of this launch
    int ntok;            // tokens in this launch (<= TB)
    const float *codebook;
    int C;
    int M, K, nseg;      // M: rows of all matrices (the launch's row space)
    int rows_per_cta;
    int nmat;
    int epi;             // GemvEpi; kEpiSiluMul interleaves the two matrices' rows
    GemvMat mat[kGvMaxMats];
    int out_bf16;
    uint32_t H;          // replicated codebook entries
    uint32_t NP;         // entries held in shared memory (head + single copy)
    uint32_t m128, m4;   // 128 and 4
    uint32_t *status;
    GemvPeers peers;     // kEpiPeer only
    GemvNorm norm;
    // RMSNorm of the activations on load (the norm that precedes the linear
    // layer): every CTA reduces the sum of squares of each token row of x over
    // K in the same order, then x[k] -> round(w[k] * round(x[k] * rsqrt(
    // mean(x^2) + eps))) (HF Qwen3RMSNorm; round = the activation dtype).
    int pn_on;
    const float *pn_w;   // [K] or null (unit weights)
    float pn_eps;
    // Tensor-parallel all-reduce consumed on load (with pn_on): before the
    // norm, every CTA waits (bounded) until ar_counts[s] >= *ar_epoch *
    // ar_expect for every rank s, then forms x[t] = round(ar_resid[t] +
    // round(sum_s slot_s[t])) in rank order (slot s row t at ar_slots + (s *
    // ntok + t) * K) and writes it to a.x (every CTA the same values; a.x is
    // not ar_resid), from where the launch loads it.
    int ar_on;
    int ar_world;
    int ar_ll;           // the slots are in the flagged form (GemvPeers::ll_epoch; ar_counts unused)
    const void *ar_slots;
    const uint32_t *ar_counts;
    const uint32_t *ar_epoch;
    uint32_t ar_expect;
    const void *ar_resid;
};

// The norm of GemvNorm, run by the last CTA (all its threads).  red: 16
// floats of free shared memory.
__device__ __forceinline__ void gv_norm_last(const GemvArgs &a, float *red) {
    const GemvNorm &nm = a.norm;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const bool bf = a.out_bf16 != 0;
    const bool peer = a.epi == kEpiPeer;
    const int64_t n = a.M;
    auto ldv = [&](const void *p, int64_t i) -> float {             // L2: written by other CTAs / ranks
        return bf ? __bfloat162float(__ldcg(static_cast<const __nv_bfloat16 *>(p) + i))
                  : __ldcg(static_cast<const float *>(p) + i);
    };
    auto stv = [&](void *p, int64_t i, float v) {
        if (bf) static_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
        else static_cast<float *>(p)[i] = v;
    };
    auto rnd = [&](float v) { return bf ? __bfloat162float(__float2bfloat16_rn(v)) : v; };
    __shared__ int late;
    if (peer) {
        // a wait that already gave up in this run: do not wait again
        if (tid == 0)
            late = (a.status && (*(volatile uint32_t *)(a.status + CBQ_STATUS_FLAGS) & CBQ_FLAG_TIMEOUT)) ? 1 : 0;
        __syncthreads();
        if (!late && tid < a.peers.world) {
            const uint32_t want = *nm.epoch * nm.expect;
            const uint64_t t0 = global_timer_ns();
            while (true) {
                uint32_t c;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(c) : "l"(nm.counts + tid) : "memory");
                if ((int32_t)(c - want) >= 0) break;
                if (global_timer_ns() - t0 > kWaitNs) {
                    late = 1;
                    break;
                }
                __nanosleep(64);
            }
        }
        __syncthreads();
        if (late) {
            if (tid == 0) {
                report(a.status, CBQ_FLAG_TIMEOUT, 0u);
                *nm.arrive = 0u;
            }
            return;
        }
        __threadfence_system();
    } else {
        __threadfence();
    }
    const int64_t ldo = a.mat[0].ldo;
    // Thread i < 256 takes elements i, i + 256, ... in that order (the order
    // of cbq_rmsnorm's kernel, so the sums are the same), kNV of them per
    // pass with every load issued before any is used; rows of up to
    // 256 * kNV values stay in registers for the normalising pass.
    constexpr int kNV = 16;
    for (int t = 0; t < a.ntok; ++t) {
        void *xr = static_cast<uint8_t *>(nm.resid) + (a.t0 + t) * nm.ldr * (bf ? 2 : 4);
        float ss = 0.f;
        float keep[kNV];
        if (tid < 256) {
            for (int64_t base = 0; base < n; base += 256 * kNV) {
                float v[kNV];
#pragma unroll
                for (int j = 0; j < kNV; ++j) {
                    const int64_t i = base + tid + 256 * j;
                    v[j] = i < n ? ldv(xr, i) : 0.f;
                }
                if (peer) {
                    float sum[kNV];
#pragma unroll
                    for (int j = 0; j < kNV; ++j) sum[j] = 0.f;
                    for (int p = 0; p < a.peers.world; ++p) {
                        const int64_t so = ((int64_t)p * a.ntok + t) * ldo;
#pragma unroll
                        for (int j = 0; j < kNV; ++j) {
                            const int64_t i = base + tid + 256 * j;
                            if (i < n) sum[j] += ldv(nm.slots, so + i);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kNV; ++j) {
                        const int64_t i = base + tid + 256 * j;
                        if (i < n) {
                            v[j] = rnd(v[j] + rnd(sum[j]));
                            stv(xr, i, v[j]);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < kNV; ++j) {
                    if (base + tid + 256 * j < n) ss += v[j] * v[j];
                    keep[j] = v[j];
                }
            }
        }
        ss = warp_sum(ss);
        if (lane == 0 && w < 8) red[w] = ss;
        __syncthreads();
        if (w == 0) {
            float t2 = lane < 8 ? red[lane] : 0.f;
            t2 = warp_sum(t2);
            if (lane == 0) red[8] = t2;
        }
        __syncthreads();
        const float scale = rsqrtf(red[8] / (float)n + nm.eps);
        void *orow = static_cast<uint8_t *>(nm.out) + (a.t0 + t) * nm.ldn * (bf ? 2 : 4);
        if (n <= 256 * kNV) {
            if (tid < 256) {
#pragma unroll
                for (int j = 0; j < kNV; ++j) {
                    const int64_t i = tid + 256 * j;
                    if (i < n) {
                        float v = rnd(keep[j] * scale);
                        if (nm.w) v = nm.w[i] * v;
                        stv(orow, i, v);
                    }
                }
            }
        } else {
            for (int64_t i = tid; i < n; i += blockDim.x) {
                float v = rnd(ldv(xr, i) * scale);
                if (nm.w) v = nm.w[i] * v;
                stv(orow, i, v);
            }
        }
        __syncthreads();                                   // red[] reuse
    }
    if (tid == 0) *nm.arrive = 0u;
}

// Row v of the launch's row space -> (matrix, row of that matrix).  Rows are
// the matrices' rows one after another, or (kEpiSiluMul) interleaved so that
// row r of both matrices lands in the same CTA.
__device__ __forceinline__ int gv_locate(const GemvArgs &a, int64_t v, int64_t &row) {
    if (a.epi == kEpiSiluMul) {
        row = v >> 1;
        return (int)(v & 1);
    }
    int m = 0;
    int64_t base = 0;
    while (m + 1 < a.nmat && v >= base + a.mat[m].M) base += a.mat[m++].M;
    row = v - base;
    return m;
}

// Shared-memory layout: [barriers][row-segment sums][codebook][rings].
__host__ __device__ inline size_t gemv_part_bytes(int rows_per_cta, int nseg, int TB) {
    return a128((size_t)rows_per_cta * nseg * TB * 4);
}
__host__ __device__ inline size_t gemv_cb_bytes(uint32_t H, uint32_t NP) {
    return a128((size_t)H * 128 + (size_t)(NP - H) * 4);
}
__host__ __device__ inline size_t gemv_ring_bytes(int bits, int nf) {
    return (size_t)kGvWarps * (nf == 32 ? GvCfg<32>::kSlots : GvCfg<64>::kSlots) * 32 * nf * bits / 8;
}

// One lane's share of a unit is NF * BITS / 32 words.
template <int BITS, int NF>
__device__ __forceinline__ void gv_load_share(const uint32_t *p, uint32_t (&w)[NF * BITS / 32 + 1]) {
    // lane stride NW words: 32-bit loads for odd NW (conflict-free), wider
    // loads for even NW so the lanes' loads stay on distinct banks
    constexpr int NW = NF * BITS / 32;
    if constexpr (NW % 4 == 0) {
#pragma unroll
        for (int s = 0; s < NW / 4; ++s) {
            const uint4 v = reinterpret_cast<const uint4 *>(p)[s];
            w[4 * s] = v.x; w[4 * s + 1] = v.y; w[4 * s + 2] = v.z; w[4 * s + 3] = v.w;
        }
    } else if constexpr (NW % 2 == 0) {
#pragma unroll
        for (int s = 0; s < NW / 2; ++s) {
            const uint2 v = reinterpret_cast<const uint2 *>(p)[s];
            w[2 * s] = v.x; w[2 * s + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int s = 0; s < NW; ++s) w[s] = p[s];
    }
    w[NW] = 0u;
}

template <int BITS, int NF>
__device__ __forceinline__ uint32_t gv_field(const uint32_t (&w)[NF * BITS / 32 + 1], int i) {
    const int bit = i * BITS, wi = bit >> 5, sh = bit & 31;
    constexpr uint32_t mask = (1u << BITS) - 1u;
    const uint32_t v = (sh + BITS <= 32) ? (w[wi] >> sh) : __funnelshift_r(w[wi], w[wi + 1], sh);
    return v & mask;
}

__device__ __forceinline__ float gv_lds(uint32_t addr) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// The NF activations of one lane's share starting at k0, token row xr
// (zero past K; K is a multiple of 128, so a share is all in or all out).
template <int NF>
__device__ __forceinline__ void gv_load_x(const float *xr, int k0, int K, float (&v)[NF]) {
    if (k0 < K) {
        const float4 *p = reinterpret_cast<const float4 *>(xr + k0);
#pragma unroll
        for (int q = 0; q < NF / 4; ++q) {
            const float4 f = __ldg(p + q);
            v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < NF; ++i) v[i] = 0.f;
    }
}
template <int NF>
__device__ __forceinline__ void gv_load_x(const __nv_bfloat16 *xr, int k0, int K, float (&v)[NF]) {
    if (k0 < K) {
        const uint4 *p = reinterpret_cast<const uint4 *>(xr + k0);
#pragma unroll
        for (int q = 0; q < NF / 8; ++q) {
            const uint4 f = __ldg(p + q);
            const uint32_t u[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                v[8 * q + 2 * h] = __uint_as_float(u[h] << 16);
                v[8 * q + 2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u);
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < NF; ++i) v[i] = 0.f;
    }
}

// The activation pre-norm of GemvArgs: scale[t] = rsqrt(mean(x[t]^2) + eps)
// for the launch's tokens, every CTA the same value (thread i adds elements
// i, i + blockDim, ... in order, then a fixed tree).  All threads call it.
// Eight consecutive activations as fp32 (k0 a multiple of 8; 16-byte
// aligned rows): one or two 16-byte loads, L2-coherent when `coherent`
// (values written earlier in the same launch).
template <typename XT>
__device__ __forceinline__ void gv_ld8(const XT *p, bool coherent, float (&v)[8]) {
    if constexpr (std::is_same<XT, float>::value) {
        const float4 *q = reinterpret_cast<const float4 *>(p);
        const float4 a = coherent ? __ldcg(q) : __ldg(q), b = coherent ? __ldcg(q + 1) : __ldg(q + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        const uint4 *q = reinterpret_cast<const uint4 *>(p);
        const uint4 f = coherent ? __ldcg(q) : __ldg(q);
        const uint32_t u[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            v[2 * h] = __uint_as_float(u[h] << 16);
            v[2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u);
        }
    }
}

template <typename XT>
__device__ __forceinline__ void gv_st8(XT *p, const float (&v)[8]) {
    if constexpr (std::is_same<XT, float>::value) {
        float4 *q = reinterpret_cast<float4 *>(p);
        q[0] = make_float4(v[0], v[1], v[2], v[3]);
        q[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t u[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * h]));
            const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(v[2 * h + 1]));
            u[h] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4 *>(p) = make_uint4(u[0], u[1], u[2], u[3]);
    }
}

// Adds, in rank order, every rank's values of activations k0..k0+7 of token t
// from its flagged slot (GemvPeers::ll_epoch) to sum: the 64-bit words are
// read, eight ranks' (bf16) or four ranks' (fp32) at a time with all their
// loads issued together, until
// each carries this step's epoch (bounded; on giving up sets *late, records
// CBQ_FLAG_TIMEOUT and returns false).  Slot p of the consumer's buffer is
// ar_slots + p * ntok * K words (fp32) or K/2 words (bf16) per token.
template <typename XT>
__device__ __forceinline__ bool gv_ll_sum8(const GemvArgs &a, int t, int k0, float (&sum)[8], int *late) {
    constexpr bool kBf = !std::is_same<XT, float>::value;
    constexpr int NWD = kBf ? 4 : 8;                        // words per 8 activations
    constexpr int PG = kBf ? 8 : 4;                         // ranks per batch of loads (64 registers)
    const int64_t per_tok = kBf ? a.K / 2 : a.K;
    const uint64_t *base = static_cast<const uint64_t *>(a.ar_slots);
    const uint32_t ep = *a.ar_epoch;
    uint64_t t0 = 0;
    for (int p0 = 0; p0 < a.ar_world; p0 += PG) {
        uint64_t v[PG][NWD];
        while (true) {
            bool ok = true;
#pragma unroll
            for (int g = 0; g < PG; ++g) {
                if (p0 + g < a.ar_world) {
                    const uint64_t *w = base + ((int64_t)(p0 + g) * a.ntok + t) * per_tok + (kBf ? k0 / 2 : k0);
#pragma unroll
                    for (int i = 0; i < NWD; ++i) v[g][i] = ld_relaxed_sys_u64(w + i);
                }
            }
#pragma unroll
            for (int g = 0; g < PG; ++g)
                if (p0 + g < a.ar_world) {
#pragma unroll
                    for (int i = 0; i < NWD; ++i) ok &= (uint32_t)(v[g][i] >> 32) == ep;
                }
            if (ok) break;
            if (*(volatile int *)late) return false;         // this CTA, or an earlier call, gave up
            if (t0 == 0) t0 = global_timer_ns();
            else if (global_timer_ns() - t0 > kWaitNs) {
                if (atomicExch(late, 1) == 0) report(a.status, CBQ_FLAG_TIMEOUT, 0u);
                return false;
            }
            __nanosleep(32);
        }
#pragma unroll
        for (int g = 0; g < PG; ++g) {
            if (p0 + g >= a.ar_world) break;
#pragma unroll
            for (int i = 0; i < NWD; ++i) {
                const uint32_t d = (uint32_t)v[g][i];
                if (kBf) {
                    sum[2 * i] += __uint_as_float(d << 16);
                    sum[2 * i + 1] += __uint_as_float(d & 0xffff0000u);
                } else {
                    sum[i] += __uint_as_float(d);
                }
            }
        }
    }
    return true;
}

// The launch's prologue on its activations (GemvArgs ar_* / pn_*), run by
// every thread of every CTA after pdl_wait:
//   * ar_on: wait (bounded) until every rank's partial rows have arrived,
//     then x[t] = round(ar_resid[t] + round(sum_s slot_s[t])) in rank order,
//     kept in shared memory (xs, [TB][K]) for this CTA's loads and written to
//     a.x by CTA 0 only (the residual stream for later launches);
//   * pn_on: scale[t] = rsqrt(mean(x[t]^2) + eps) of the (new) x rows.
// Thread i takes the 8-element chunks i, i + blockDim, ... of a row, all
// loads of a chunk issued together, then the warps' sums are added in warp
// order, so every CTA computes the same scales.  Returns false when the wait
// gave up (CBQ_FLAG_TIMEOUT recorded) or an earlier wait of this run had.
template <typename XT, int TB>
__device__ __forceinline__ bool gv_prologue(const GemvArgs &a, float (&scale)[TB], float *red, int *late,
                                            XT *xs) {
    constexpr int NT = kGvWarps * 32;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    if (a.ar_on) {
        if (tid == 0)
            *late = (a.status && (*(volatile uint32_t *)(a.status + CBQ_STATUS_FLAGS) & CBQ_FLAG_TIMEOUT)) ? 1 : 0;
        __syncthreads();
        if (!*late && tid < a.ar_world && !a.ar_ll) {
            const uint32_t want = *a.ar_epoch * a.ar_expect;
            const uint64_t t0 = global_timer_ns();
            while (true) {
                uint32_t c;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(c) : "l"(a.ar_counts + tid) : "memory");
                if ((int32_t)(c - want) >= 0) break;
                if (global_timer_ns() - t0 > kWaitNs) {
                    *late = 1;
                    break;
                }
                __nanosleep(32);
            }
        }
        __syncthreads();
        if (*late) {
            if (tid == 0 && blockIdx.x == 0) report(a.status, CBQ_FLAG_TIMEOUT, 0u);
            return false;
        }
        // the pollers' system-scope acquire loads, then the CTA barrier, order
        // every thread's reads of the slots after the ranks' releases
    }
    const XT *slots = static_cast<const XT *>(a.ar_slots);
    const XT *res = static_cast<const XT *>(a.ar_resid);
    XT *x = const_cast<XT *>(static_cast<const XT *>(a.x));
    for (int t = 0; t < TB; ++t) {
        float ss = 0.f;
        if (t < a.ntok) {
            const int64_t row = (a.t0 + t) * a.ldx;
            for (int k0 = tid * 8; k0 < a.K; k0 += NT * 8) {
                float v[8];
                if (a.ar_on) {
                    float r[8], sum[8];
                    gv_ld8<XT>(res + row + k0, false, r);
#pragma unroll
                    for (int e = 0; e < 8; ++e) sum[e] = 0.f;
                    if (a.ar_ll) {
                        // on giving up the values are garbage; every thread
                        // still reaches the barriers below, and the call reports it
                        gv_ll_sum8<XT>(a, t, k0, sum, late);
                    } else {
                        for (int p = 0; p < a.ar_world; ++p) {       // rank order
                            float sp[8];
                            gv_ld8<XT>(slots + ((int64_t)p * a.ntok + t) * a.K + k0, true, sp);
#pragma unroll
                            for (int e = 0; e < 8; ++e) sum[e] += sp[e];
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        v[e] = to_f32<XT>(from_f32<XT>(r[e] + to_f32<XT>(from_f32<XT>(sum[e]))));
                    gv_st8<XT>(xs + (int64_t)t * a.K + k0, v);
                    if (blockIdx.x == 0) gv_st8<XT>(x + row + k0, v);
                } else {
                    gv_ld8<XT>(x + row + k0, false, v);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
            }
        }
        if (!a.pn_on) continue;
        ss = warp_sum(ss);
        if (lane == 0) red[w] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < kGvWarps; ++i) tot += red[i];
        scale[t] = rsqrtf(tot / (float)a.K + a.pn_eps);
        __syncthreads();                                   // red[] reuse
    }
    if (a.ar_on) __syncthreads();                           // xs complete before any warp reads it
    return !(a.ar_on && *(volatile int *)late);
}

// Normalise NF loaded activations starting at k0 (see gv_prologue).
template <typename XT, int NF>
__device__ __forceinline__ void gv_prenorm_apply(float (&v)[NF], float scale, const float *w, int k0, int K) {
    if (k0 >= K) return;
    auto rnd = [](float f) {
        if constexpr (std::is_same<XT, float>::value) return f;
        else return __bfloat162float(__float2bfloat16_rn(f));
    };
#pragma unroll
    for (int i = 0; i < NF; ++i) {
        float y = rnd(v[i] * scale);
        if (w) y = rnd(__ldg(w + k0 + i) * y);
        v[i] = y;
    }
}

// gv_load_x from the shared-memory copy of the activations the all-reduce
// prologue formed (xs row, 16-byte aligned).
template <int NF, typename XT>
__device__ __forceinline__ void gv_load_x_smem(const XT *xr, int k0, int K, float (&v)[NF]) {
    if (k0 < K) {
#pragma unroll
        for (int q = 0; q < NF / 8; ++q) {
            if constexpr (std::is_same<XT, float>::value) {
                const float4 a = reinterpret_cast<const float4 *>(xr + k0)[2 * q];
                const float4 b = reinterpret_cast<const float4 *>(xr + k0)[2 * q + 1];
                v[8 * q] = a.x; v[8 * q + 1] = a.y; v[8 * q + 2] = a.z; v[8 * q + 3] = a.w;
                v[8 * q + 4] = b.x; v[8 * q + 5] = b.y; v[8 * q + 6] = b.z; v[8 * q + 7] = b.w;
            } else {
                const uint4 f = reinterpret_cast<const uint4 *>(xr + k0)[q];
                const uint32_t u[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    v[8 * q + 2 * h] = __uint_as_float(u[h] << 16);
                    v[8 * q + 2 * h + 1] = __uint_as_float(u[h] & 0xffff0000u);
                }
            }
        }
    } else {
#pragma unroll
        for (int i = 0; i < NF; ++i) v[i] = 0.f;
    }
}

template <int BITS, int TB, int NF, typename XT>
__global__ void __launch_bounds__(kGvWarps * 32, 1) k_gemv_fixed(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int kGvSeg = GvCfg<NF>::kSeg, kGvSlots = GvCfg<NF>::kSlots, kNW = NF * BITS / 32;
    constexpr uint32_t kSegBytes = (uint32_t)kGvSeg * BITS / 8;
    constexpr bool kPadded = BITS <= 14;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nseg = a.nseg, K = a.K;
    pdl_launch_dependents();
    const int64_t m0 = (int64_t)blockIdx.x * a.rows_per_cta;
    if (m0 >= a.M) return;                                   // the whole CTA: no barrier pending
    const int nrows = (int)min((int64_t)a.rows_per_cta, (int64_t)a.M - m0);

    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kGvSlots;
    float *part = reinterpret_cast<float *>(smem + kGvBarBytes);
    uint8_t *cbs = smem + kGvBarBytes + gemv_part_bytes(a.rows_per_cta, nseg, TB);
    uint8_t *ring = cbs + gemv_cb_bytes(a.H, a.NP) + (size_t)warp * kGvSlots * kSegBytes;
    // ar_on: the all-reduced activations [TB][K] after the rings
    XT *xsm = reinterpret_cast<XT *>(cbs + gemv_cb_bytes(a.H, a.NP) + gemv_ring_bytes(BITS, NF));

    // this warp's units: u = s * nrows + rl (segment-major)
    const int U = nrows * nseg;
    const int u0 = (int)((int64_t)warp * U / kGvWarps);
    const int u1 = (int)((int64_t)(warp + 1) * U / kGvWarps);
    const int n = u1 - u0;

    int is = u0 / nrows, irl = u0 - (u0 / nrows) * nrows, islot = 0;   // next unit to copy
    auto issue_next = [&]() {                                // lane 0 only
        const int cnt = min(kGvSeg, K - is * kGvSeg);
        const uint32_t bytes = (uint32_t)cnt * BITS / 8;
        int64_t row;
        const int m = gv_locate(a, m0 + irl, row);
        mbar_arrive_expect_tx(&bars[islot], bytes);
        bulk_g2s(ring + (size_t)islot * kSegBytes,
                 a.mat[m].packed + (row * (int64_t)K + (int64_t)is * kGvSeg) * BITS / 8, bytes,
                 &bars[islot]);
        if (++irl == nrows) { irl = 0; ++is; }
        if (++islot == kGvSlots) islot = 0;
    };
    // codebook: replicated head, then the single copy (padded for b <= 14).
    // One load per entry; a head row (32 copies, 128 B) is written as eight
    // 16-byte stores whose order is rotated by lane so that the eight lanes
    // of each store phase hit distinct banks.  The loads of the first pass
    // (the whole table for codebooks of up to 4096 + 12288 entries) are
    // issued before the first stream copies, which would otherwise queue
    // ahead of them, and before any store: the table costs one latency.
    {
        const uint32_t H = a.H, NP = a.NP;
        const int cmax = a.C - 1;
        constexpr int kT = kGvWarps * 32;
        constexpr int kBatch = 8, kTB = 24;
        float vh[kBatch], vt[kTB];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const uint32_t e = j * kT + tid;
            vh[j] = e < H ? __ldg(a.codebook + min((int)e, cmax)) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < kTB; ++j) {
            const uint32_t c = H + j * kT + tid;
            vt[j] = c < NP ? __ldg(a.codebook + min((int)c, cmax)) : 0.f;
        }
        if (lane == 0) {
            for (int s = 0; s < kGvSlots; ++s) mbar_init(&bars[s], 1);
            mbar_fence_init();
            for (int i = 0; i < n && i < kGvSlots; ++i) issue_next();
        }
        auto put_head = [&](uint32_t e, float v) {
            const float4 v4 = make_float4(v, v, v, v);
            float4 *row = reinterpret_cast<float4 *>(cbs + (size_t)e * 128);
#pragma unroll
            for (int q = 0; q < 8; ++q) row[(q + lane) & 7] = v4;
        };
        float *tw = reinterpret_cast<float *>(cbs + (size_t)H * 128);
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
            if (j * kT + tid < H) put_head(j * kT + tid, vh[j]);
#pragma unroll
        for (int j = 0; j < kTB; ++j)
            if (H + j * kT + tid < NP) tw[j * kT + tid] = vt[j];
        for (uint32_t e0 = kT * kBatch; e0 < H; e0 += kT * kBatch) {     // larger tables
            float v[kBatch];
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                const uint32_t e = e0 + j * kT + tid;
                v[j] = e < H ? __ldg(a.codebook + min((int)e, cmax)) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < kBatch; ++j)
                if (e0 + j * kT + tid < H) put_head(e0 + j * kT + tid, v[j]);
        }
        for (uint32_t c0 = H + kT * kTB; c0 < NP; c0 += kT * kTB) {
            float v[kTB];
#pragma unroll
            for (int j = 0; j < kTB; ++j) {
                const uint32_t c = c0 + j * kT + tid;
                v[j] = c < NP ? __ldg(a.codebook + min((int)c, cmax)) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < kTB; ++j) {
                const uint32_t c = c0 + j * kT + tid;
                if (c < NP) tw[c - H] = v[j];
            }
        }
    }
    __syncthreads();
    // Weights and codebook are constant; the activations (and the residual
    // the epilogue reads) come from the previous kernel.
    pdl_wait();
    float pn_scale[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) pn_scale[t] = 1.f;
    if (a.ar_on || a.pn_on) {
        __shared__ float pn_red[kGvWarps];
        __shared__ int ar_late;
        gv_prologue<XT, TB>(a, pn_scale, pn_red, &ar_late, xsm);
    }

    const uint32_t cb_base = smem_u32(cbs);
    const uint32_t head_off = cb_base + (uint32_t)lane * 4u;
    const uint32_t tail_off = cb_base + a.H * 124u;
    const uint32_t m128 = a.m128, m4 = a.m4;
    const uint32_t cmax = (uint32_t)(a.C - 1);
    const XT *x = static_cast<const XT *>(a.x);

    float xr[TB][NF];
    int xs = -1;                                             // segment whose x is loaded
    int s = u0 / nrows, rl = u0 - (u0 / nrows) * nrows;      // unit being decoded
    int slot = 0;
    uint32_t phase = 0;
    auto slot_words = [&](int sl) {
        return reinterpret_cast<const uint32_t *>(ring + (size_t)sl * kSegBytes) + lane * kNW;
    };
    auto gather = [&](uint32_t c) {
        if (!kPadded) c = min(c, cmax);
        return gv_lds(min(c * m128 + head_off, c * m4 + tail_off));
    };
    int i = 0;
    while (i < n) {
        if (s != xs) {
            const int k0 = s * kGvSeg + lane * NF;
#pragma unroll
            for (int t = 0; t < TB; ++t) {
                if (t < a.ntok) {
                    if (a.ar_on) gv_load_x_smem<NF, XT>(xsm + (int64_t)t * K, k0, K, xr[t]);
                    else gv_load_x<NF>(x + (a.t0 + t) * a.ldx, k0, K, xr[t]);
                    if (a.pn_on) gv_prenorm_apply<XT, NF>(xr[t], pn_scale[t], a.pn_w, k0, K);
                } else {
#pragma unroll
                    for (int q = 0; q < NF; ++q) xr[t][q] = 0.f;
                }
            }
            xs = s;
        }
        // Two rows of the same segment at once when the range allows: twice
        // the independent gathers in flight per warp.
        const bool two = CBQ_GV_PAIR && NF == 32 && i + 1 < n && rl + 1 < nrows;
        const int slot2 = slot + 1 == kGvSlots ? 0 : slot + 1;
        const uint32_t phase2 = slot + 1 == kGvSlots ? phase ^ 1u : phase;
        bool ok = mbar_wait_bounded(&bars[slot], phase);
        if (two) ok = mbar_wait_bounded(&bars[slot2], phase2) && ok;
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) report(a.status, CBQ_FLAG_TIMEOUT, (uint32_t)(m0 + rl));
            break;
        }
        float acc[2][2][TB];
#pragma unroll
        for (int t = 0; t < TB; ++t) { acc[0][0][t] = acc[0][1][t] = acc[1][0][t] = acc[1][1][t] = 0.f; }
        const bool live = s * kGvSeg + lane * NF < K;
        uint32_t w[kNW + 1], w2[kNW + 1];
        if (live) {
            gv_load_share<BITS, NF>(slot_words(slot), w);
            if (two) gv_load_share<BITS, NF>(slot_words(slot2), w2);
        }
        if (live) {
            if (two) {
#pragma unroll
                for (int q = 0; q < NF; ++q) {
                    const float v = gather(gv_field<BITS, NF>(w, q));
                    const float v2 = gather(gv_field<BITS, NF>(w2, q));
#pragma unroll
                    for (int t = 0; t < TB; ++t) {
                        acc[0][q & 1][t] = fmaf(xr[t][q], v, acc[0][q & 1][t]);
                        acc[1][q & 1][t] = fmaf(xr[t][q], v2, acc[1][q & 1][t]);
                    }
                }
            } else {
#pragma unroll
                for (int q = 0; q < NF; ++q) {
                    const float v = gather(gv_field<BITS, NF>(w, q));
#pragma unroll
                    for (int t = 0; t < TB; ++t) acc[0][q & 1][t] = fmaf(xr[t][q], v, acc[0][q & 1][t]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            if (i + kGvSlots < n) issue_next();
            if (two && i + 1 + kGvSlots < n) issue_next();
        }
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            const float tot = warp_sum(acc[0][0][t] + acc[0][1][t]);
            if (lane == 0) part[((size_t)rl * nseg + s) * TB + t] = tot;
            if (two) {
                const float tot2 = warp_sum(acc[1][0][t] + acc[1][1][t]);
                if (lane == 0) part[((size_t)(rl + 1) * nseg + s) * TB + t] = tot2;
            }
        }
        const int step = two ? 2 : 1;
        i += step;
        rl += step;
        if (rl == nrows) { rl = 0; ++s; }
        slot += step;
        if (slot >= kGvSlots) { slot -= kGvSlots; phase ^= 1u; }
    }
    if (i < n && lane == 0) {   // timed out: wait (bounded) for this warp's copies still in flight
        for (int j = i; j < n && j < i + kGvSlots; ++j) {
            mbar_wait_bounded(&bars[slot], phase);
            if (++slot == kGvSlots) { slot = 0; phase ^= 1u; }
        }
    }
    __syncthreads();

    // rows: segment sums in segment order, + bias, then the epilogue, in the
    // output dtype.  Intermediate roundings follow the unfused sequence of
    // operations (linear output rounded, then the add / SiLU / product
    // rounded), so fused and unfused decoders compute the same values.
    auto seg_sum = [&](int r, int t) {
        float sum = 0.f;
        for (int q = 0; q < nseg; ++q) sum += part[((size_t)r * nseg + q) * TB + t];
        return sum;
    };
    auto rnd = [&](float v) { return a.out_bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : v; };
    auto store = [&](const GemvMat &mt, int64_t o, float v) {
        if (a.out_bf16) static_cast<__nv_bfloat16 *>(mt.out)[o] = __float2bfloat16_rn(v);
        else static_cast<float *>(mt.out)[o] = v;
    };
    auto load = [&](const void *p, int64_t o) {
        return a.out_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[o])
                          : static_cast<const float *>(p)[o];
    };
    if (a.epi == kEpiSiluMul) {
        const GemvMat &g = a.mat[0], &u = a.mat[1];
        for (int r = 2 * tid; r + 1 < nrows; r += 2 * kGvWarps * 32) {
            const int64_t row = (m0 + r) >> 1;
            const float bg = g.bias ? g.bias[row] : 0.f, bu = u.bias ? u.bias[row] : 0.f;
            for (int t = 0; t < a.ntok; ++t) {
                const float gv = rnd(seg_sum(r, t) + bg), uv = rnd(seg_sum(r + 1, t) + bu);
                const float sv = rnd(gv / (1.0f + expf(-gv)));
                store(g, (a.t0 + t) * g.ldo + row, sv * uv);
            }
        }
    } else if (a.epi == kEpiPeer && a.peers.ll_epoch) {
        const GemvMat &mt = a.mat[0];
        const uint64_t ep = (uint64_t)*a.peers.ll_epoch << 32;
        if (a.out_bf16) {                                  // row pairs (rows_per_cta and M are even)
            for (int r = 2 * tid; r + 1 < nrows; r += 2 * kGvWarps * 32) {
                const int64_t row = m0 + r;
                const float b0 = mt.bias ? mt.bias[row] : 0.f, b1 = mt.bias ? mt.bias[row + 1] : 0.f;
                for (int t = 0; t < a.ntok; ++t) {
                    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(seg_sum(r, t) + b0));
                    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(seg_sum(r + 1, t) + b1));
                    const int64_t w = (a.t0 + t) * (mt.ldo / 2) + row / 2;
                    for (int p = 0; p < a.peers.world; ++p)
                        st_relaxed_sys_u64(static_cast<uint64_t *>(a.peers.slot[p]) + w, ep | lo | (hi << 16));
                }
            }
        } else {
            for (int r = tid; r < nrows; r += kGvWarps * 32) {
                const int64_t row = m0 + r;
                const float b = mt.bias ? mt.bias[row] : 0.f;
                for (int t = 0; t < a.ntok; ++t) {
                    const int64_t w = (a.t0 + t) * mt.ldo + row;
                    const uint64_t v = ep | __float_as_uint(seg_sum(r, t) + b);
                    for (int p = 0; p < a.peers.world; ++p)
                        st_relaxed_sys_u64(static_cast<uint64_t *>(a.peers.slot[p]) + w, v);
                }
            }
        }
    } else if (a.epi == kEpiPeer) {
        const GemvMat &mt = a.mat[0];
        for (int r = tid; r < nrows; r += kGvWarps * 32) {
            const int64_t row = m0 + r;
            const float b = mt.bias ? mt.bias[row] : 0.f;
            for (int t = 0; t < a.ntok; ++t) {
                const int64_t o = (a.t0 + t) * mt.ldo + row;
                const float v = seg_sum(r, t) + b;
                for (int p = 0; p < a.peers.world; ++p) {
                    if (a.out_bf16) static_cast<__nv_bfloat16 *>(a.peers.slot[p])[o] = __float2bfloat16_rn(v);
                    else static_cast<float *>(a.peers.slot[p])[o] = v;
                }
            }
        }
        // The barrier orders every thread's peer stores before the counter
        // updates, and a system-scope release is cumulative over them.
        __syncthreads();
        if (tid < a.peers.world)
            asm volatile("red.release.sys.global.add.u32 [%0], %1;"
                         ::"l"(a.peers.count[tid]), "r"((uint32_t)nrows) : "memory");
    } else {
        for (int r = tid; r < nrows; r += kGvWarps * 32) {
            int64_t row;
            const GemvMat &mt = a.mat[gv_locate(a, m0 + r, row)];
            const float b = mt.bias ? mt.bias[row] : 0.f;
            for (int t = 0; t < a.ntok; ++t) {
                const int64_t o = (a.t0 + t) * mt.ldo + row;
                float v = seg_sum(r, t) + b;
                if (a.epi == kEpiResidual) v = load(mt.resid, o) + rnd(v);
                store(mt, o, v);
            }
        }
    }
    if (a.norm.arrive) {
        __shared__ int last;
        __threadfence();                                   // this CTA's rows, before its count
        __syncthreads();
        if (tid == 0) {
            const uint32_t nct = (uint32_t)((a.M + a.rows_per_cta - 1) / a.rows_per_cta);
            last = atomicAdd(a.norm.arrive, 1u) == nct - 1u;
        }
        __syncthreads();
        if (last) gv_norm_last(a, part);                   // the segment sums are consumed
    }
}

}  // namespace cbq
