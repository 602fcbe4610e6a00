// cbq_fixed_kernel.cuh -- the fixed-width decode-GEMV kernel (sm_100a).
//
// out[t, r] = sum_k x[t, k] * cb[min(idx(r*K + k), C-1)], idx LSB-first b-bit
// fields (reference src/bitpack.py:32-94, src/compressed_matmul.c:334-347).
//
// Work decomposition.  A "unit" is one 1024-index segment of one row
// (32 lanes x 32 consecutive indices = 32 x b words: every lane's share is
// b whole 32-bit words when K % 128 == 0).  Units are numbered row-major and
// every warp of the persistent grid (148 CTAs x 16 warps) owns one contiguous,
// balanced range of them.  Warps never synchronise with each other:
//   * each warp streams its units through a private ring of kFxSlots
//     shared-memory slots, lane 0 issuing one cp.async.bulk per unit that
//     completes on the slot's mbarrier;
//   * lane j decodes its 32 fields from b words with the widest conflict-free
//     shared load, compile-time shifts (b is a template parameter), gathers
//     the codebook values and accumulates against x;
//   * a row whose units all lie in one warp's range is reduced with warp
//     shuffles and written directly; a row split between warps (only at range
//     boundaries) leaves per-piece sums in the caller's workspace and the last
//     piece to arrive (atomic counter) adds them in segment order, so results
//     are bitwise reproducible for a given GPU.  Without a workspace the
//     ranges are rounded to whole rows instead.
// Codebook in shared memory (fp32): the first H entries (the most frequent
// ones when the codebook is frequency-sorted) are replicated once per lane so
// that lane j always reads bank j -- conflict-free -- and a single copy of all
// entries follows; for b <= 14 that copy is padded to 2^b entries with
// cb[C-1], which implements the reference's clamp idx >= C -> C-1 without an
// instruction.  H is as large as shared memory allows.  The decode is integer-
// ALU bound, so the lookup is kept to a compare, a select and two multiply-
// adds (which run on the FMA pipe), and the unit loop uses cursors instead of
// divisions.
// x sits in shared memory skewed so that the lanes' 16-byte loads of their
// 32 consecutive activations hit distinct banks.
#pragma once
#include "cbq_common.cuh"

namespace cbq {

constexpr int kFxWarps = 16;      // warps per CTA
constexpr int kFxSeg = 1024;      // indices per unit
constexpr int kFxSlots = 3;       // ring slots per warp
static_assert(kFxWarps * kFxSlots * 8 <= 512, "the mbarriers occupy the first 512 bytes of shared memory");

struct FixedArgs {
    const void *x;
    int64_t ldx;
    int64_t t0;          // first token of this launch
    int ntok;            // tokens in this launch (<= TB)
    const uint8_t *packed;
    const float *codebook;
    int C;
    int M, K, nseg;
    const float *bias;
    void *out;
    int64_t ldo;
    int out_bf16;
    float *part;         // workspace: per-(row, segment, token) piece sums, or null
    uint32_t *cnt;       // workspace: per-row arrival counters (left zeroed)
    uint32_t cb_bytes;   // shared bytes for the codebook (replicated head + single copy)
    uint32_t *status;
};

template <typename XT> struct XLayout;
// fp32: 32 floats per lane + 4 floats pad -> lane stride 36 words (banks 4j).
template <> struct XLayout<float> {
    static constexpr int kStride = 36;
    __device__ static int elem(int k) { return (k >> 5) * 36 + (k & 31); }
};
// bf16: 32 halves per lane + 8 halves pad -> lane stride 20 words (banks 20j).
template <> struct XLayout<__nv_bfloat16> {
    static constexpr int kStride = 40;
    __device__ static int elem(int k) { return (k >> 5) * 40 + (k & 31); }
};

// Load the BITS words of one lane's share with the widest conflict-free load:
// lane stride BITS words -> 32-bit loads for odd BITS, 64-bit for BITS = 2
// mod 4, 128-bit for BITS = 0 mod 4.
template <int BITS>
__device__ __forceinline__ void load_share(const uint32_t *p, uint32_t (&w)[BITS + 1]) {
    if constexpr (BITS % 4 == 0) {
#pragma unroll
        for (int s = 0; s < BITS / 4; ++s) {
            const uint4 v = reinterpret_cast<const uint4 *>(p)[s];
            w[4 * s] = v.x; w[4 * s + 1] = v.y; w[4 * s + 2] = v.z; w[4 * s + 3] = v.w;
        }
    } else if constexpr (BITS % 2 == 0) {
#pragma unroll
        for (int s = 0; s < BITS / 2; ++s) {
            const uint2 v = reinterpret_cast<const uint2 *>(p)[s];
            w[2 * s] = v.x; w[2 * s + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int s = 0; s < BITS; ++s) w[s] = p[s];
    }
    w[BITS] = 0u;
}

template <int BITS>
__device__ __forceinline__ uint32_t share_field(const uint32_t (&w)[BITS + 1], int i) {
    const int bit = i * BITS, wi = bit >> 5, sh = bit & 31;
    constexpr uint32_t mask = (1u << BITS) - 1u;
    const uint32_t v = (sh + BITS <= 32) ? (w[wi] >> sh) : __funnelshift_r(w[wi], w[wi + 1], sh);
    return v & mask;
}

// 8 activations of token row `xr` starting at element e, as fp32.
__device__ __forceinline__ void load_x8(const float *xr, int e, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4 *>(xr + e);
    const float4 b = *reinterpret_cast<const float4 *>(xr + e + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load_x8(const __nv_bfloat16 *xr, int e, float (&v)[8]) {
    const uint4 a = *reinterpret_cast<const uint4 *>(xr + e);
    const uint32_t u[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        v[2 * q] = __uint_as_float(u[q] << 16);
        v[2 * q + 1] = __uint_as_float(u[q] & 0xffff0000u);
    }
}

struct CbView {
    uint32_t base;         // shared address: head (H entries x 32 lanes), then the single copy
    uint32_t tail;         // shared address of the single copy
    uint32_t H;            // replicated entries
};

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// Codebook value for index c (clamped or padded), read at lane address lane_addr.
__device__ __forceinline__ float cb_value(const CbView &v, uint32_t c, uint32_t lane_addr) {
    const uint32_t addr = (c < v.H) ? (c * 128u + lane_addr) : (c * 4u + v.tail);
    return lds_f32(addr);
}

template <typename OT>
__device__ __forceinline__ void store_out(void *out, int64_t i, float v) {
    static_cast<OT *>(out)[i] = from_f32<OT>(v);
}

// Build the shared codebook from the fp32 copy staged in shared memory
// (stage[0..C)): NP = max(C, padded size) single-copy entries after the head.
__device__ __forceinline__ CbView fill_codebook(uint8_t *dst, const float *stage, int C, int NP,
                                                uint32_t bytes, int nthreads, int tid) {
    CbView v;
    const uint32_t tail = (uint32_t)NP * 4u;
    int H = (bytes > tail) ? (int)((bytes - tail) / 128u) : 0;
    H = min(H, C);
    v.H = (uint32_t)H;
    v.base = smem_u32(dst);
    v.tail = v.base + (uint32_t)H * 128u;
    uint32_t *w = reinterpret_cast<uint32_t *>(dst);
#pragma unroll 4
    for (int i = tid; i < H * 32; i += nthreads) w[i] = __float_as_uint(stage[i >> 5]);
    uint32_t *t = reinterpret_cast<uint32_t *>(dst + (size_t)H * 128);
    for (int c = tid; c < NP; c += nthreads) t[c] = __float_as_uint(stage[min(c, C - 1)]);
    return v;
}

// Write (or combine) the sum of one warp's piece [s_first, s] of row r.
template <int TB>
__device__ __forceinline__ void finish_piece(const FixedArgs &a, const float (&tot)[TB], int64_t r,
                                             int s_first, int s) {
    const int nseg = a.nseg;
    const float b = a.bias ? a.bias[r] : 0.f;
    if (s_first == 0 && s == nseg - 1) {
        for (int t = 0; t < a.ntok; ++t) {
            const int64_t o = (a.t0 + t) * a.ldo + r;
            if (a.out_bf16) store_out<__nv_bfloat16>(a.out, o, tot[t] + b);
            else store_out<float>(a.out, o, tot[t] + b);
        }
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
            const int64_t o = (a.t0 + t) * a.ldo + r;
            if (a.out_bf16) store_out<__nv_bfloat16>(a.out, o, sum + b);
            else store_out<float>(a.out, o, sum + b);
        }
        // leave the row's pieces and its counter zero, so the workspace stays
        // zero-filled for the next call whatever its shape
        for (int i = 0; i < nseg * TB; ++i) pr[i] = 0.f;
        atomicExch(&a.cnt[r], 0u);
    }
}

// The per-warp unit loop.
template <int BITS, int TB, typename XT>
__device__ void fixed_warp_loop(const FixedArgs &a, const XT *xs, int XS, const CbView cbv,
                                uint8_t *ring, uint64_t *bars, int64_t u0, int64_t u1) {
    const int lane = threadIdx.x & 31;
    const uint32_t lane_addr = cbv.base + (uint32_t)lane * 4u;
    constexpr uint32_t kSegBytes = (uint32_t)kFxSeg * BITS / 8;
    constexpr bool kPadded = BITS <= 14;        // single copy padded to 2^BITS: no clamp needed
    const int64_t n = u1 - u0;
    const int nseg = a.nseg, K = a.K;
    const uint32_t cmax = (uint32_t)(a.C - 1);

    // Cursors instead of divisions: (ir, is) = row/segment of the next unit to
    // copy, (r, s) = of the unit being decoded; slots and mbarrier phases cycle.
    int64_t ir = u0 / nseg;
    int is = (int)(u0 - ir * nseg);
    int islot = 0;
    auto issue_next = [&]() {                                 // lane 0 only
        const int cnt = min(kFxSeg, K - is * kFxSeg);
        const uint32_t bytes = (uint32_t)cnt * BITS / 8;
        mbar_arrive_expect_tx(&bars[islot], bytes);
        bulk_g2s(ring + (size_t)islot * kSegBytes,
                 a.packed + (ir * (int64_t)K + (int64_t)is * kFxSeg) * BITS / 8, bytes, &bars[islot]);
        if (++is == nseg) { is = 0; ++ir; }
        if (++islot == kFxSlots) islot = 0;
    };
    if (lane == 0)
        for (int64_t i = 0; i < n && i < kFxSlots; ++i) issue_next();
    __syncwarp();

    float acc[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) acc[t] = 0.f;
    int64_t r = u0 / nseg;
    int s = (int)(u0 - r * nseg);
    int s_first = s;
    int slot = 0;
    uint32_t phase = 0;
    int64_t i = 0;
    for (; i < n; ++i) {
        const bool ok = mbar_wait_bounded(&bars[slot], phase);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) report(a.status, CBQ_FLAG_TIMEOUT, (uint32_t)r);
            break;
        }
        const int k0 = s * kFxSeg + lane * 32;
        if (k0 < K) {
            uint32_t w[BITS + 1];
            load_share<BITS>(reinterpret_cast<const uint32_t *>(ring + (size_t)slot * kSegBytes) +
                                 lane * BITS, w);
            const int e0 = XLayout<XT>::elem(k0);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                float xv[TB][8];
#pragma unroll
                for (int t = 0; t < TB; ++t) load_x8(xs + t * XS, e0 + 8 * g, xv[t]);
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    uint32_t c = share_field<BITS>(w, 8 * g + q);
                    if (!kPadded) c = min(c, cmax);
                    const float wt = cb_value(cbv, c, lane_addr);
#pragma unroll
                    for (int t = 0; t < TB; ++t) acc[t] = fmaf(xv[t][q], wt, acc[t]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + kFxSlots < n) issue_next();
        if (s == nseg - 1 || i == n - 1) {                    // end of this warp's piece of row r
            float tot[TB];
#pragma unroll
            for (int t = 0; t < TB; ++t) tot[t] = warp_sum(acc[t]);
            if (lane == 0) finish_piece<TB>(a, tot, r, s_first, s);
#pragma unroll
            for (int t = 0; t < TB; ++t) acc[t] = 0.f;
            s_first = 0;
        }
        if (++s == nseg) { s = 0; ++r; }
        if (++slot == kFxSlots) { slot = 0; phase ^= 1u; }
    }
    if (i < n && lane == 0) {   // timed out: drain this warp's copies still in flight (bounded)
        for (int64_t j = i; j < n && j < i + kFxSlots; ++j) {
            mbar_wait_bounded(&bars[slot], phase);
            if (++slot == kFxSlots) { slot = 0; phase ^= 1u; }
        }
    }
}

// Shared bytes before the codebook: barriers + x block.
__host__ __device__ inline size_t fixed_prefix_bytes(int K, int TB, int xbytes) {
    const int kc = (K + 31) / 32;
    const int stride = (xbytes == 4) ? 36 : 40;
    return 512 + a128((size_t)TB * kc * stride * xbytes);
}

template <int BITS, int TB, typename XT>
__global__ void __launch_bounds__(kFxWarps * 32, 1) k_linear_fixed(const FixedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int nthreads = kFxWarps * 32;
    const int K = a.K;
    const int XS = ((K + 31) / 32) * XLayout<XT>::kStride;   // elements per token row
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem);
    XT *xs = reinterpret_cast<XT *>(smem + 512);
    uint8_t *cbs = smem + fixed_prefix_bytes(K, TB, sizeof(XT));
    uint8_t *rings = cbs + a128(a.cb_bytes);
    constexpr uint32_t kSegBytes = (uint32_t)kFxSeg * BITS / 8;

    const int warp = tid >> 5;
    if ((tid & 31) == 0) {
        for (int s = 0; s < kFxSlots; ++s) mbar_init(&bars[warp * kFxSlots + s], 1);
        mbar_fence_init();
    }
    // x -> shared (skewed), zero for tokens beyond ntok
    const XT *x = static_cast<const XT *>(a.x);
#pragma unroll 4
    for (int i = tid; i < TB * K; i += nthreads) {
        const int t = i / K, k = i - t * K;
        xs[t * XS + XLayout<XT>::elem(k)] = (t < a.ntok) ? x[(a.t0 + t) * a.ldx + k] : XT(0.f);
    }
    // Stage the fp32 codebook in the (still idle) ring area with one coalesced
    // pass, then build the replicated head and the (padded) single copy.
    float *stage = reinterpret_cast<float *>(rings);
#pragma unroll 4
    for (int c = tid; c < a.C; c += nthreads) stage[c] = a.codebook[c];
    __syncthreads();
    const int NP = (BITS <= 14) ? max(a.C, 1 << BITS) : a.C;
    const CbView cbv = fill_codebook(cbs, stage, a.C, NP, a.cb_bytes, nthreads, tid);
    __syncthreads();

    // this warp's unit range
    const int64_t W = (int64_t)gridDim.x * kFxWarps;
    const int64_t gw = (int64_t)blockIdx.x * kFxWarps + warp;
    int64_t u0, u1;
    if (a.part) {
        const int64_t U = (int64_t)a.M * a.nseg;
        u0 = gw * U / W;
        u1 = (gw + 1) * U / W;
    } else {
        u0 = (gw * a.M / W) * a.nseg;
        u1 = ((gw + 1) * a.M / W) * a.nseg;
    }
    uint8_t *ring = rings + (size_t)warp * kFxSlots * kSegBytes;
    fixed_warp_loop<BITS, TB, XT>(a, xs, XS, cbv, ring, bars + warp * kFxSlots, u0, u1);
}

}  // namespace cbq
