// cbq_fixed.cu -- fixed-width codebook decode-GEMV, embedding and packer (sm_100a).
//
// Stream format: element e of the row-major [M, K] index matrix occupies bits
// [e*b, (e+1)*b) of an LSB-first byte stream (reference src/bitpack.py:32-94,
// read by src/compressed_matmul.c:334-347).
//
// GEMV fast path (K % 128 == 0, codebook <= 16384 entries, 16-byte aligned
// stream): a persistent grid, one 256-thread CTA per SM.
//   * A tile is RB whole rows.  With K % 128 == 0 every row starts on a
//     16-byte boundary, so a tile is one contiguous, aligned byte range that a
//     single cp.async.bulk copies into a shared-memory ring of NST stages,
//     completing on an mbarrier (thread 0 produces, all threads consume).
//   * A "chunk" is 32 consecutive indices of one row = exactly `b` 32-bit
//     words.  Each thread decodes whole chunks: it loads the b words with the
//     widest conflict-free shared load for b (32-bit for odd b, 64-bit for
//     b = 2 mod 4, 128-bit for b = 0 mod 4) and extracts the 32 fields with
//     compile-time shifts (b is a template parameter).
//   * The codebook (fp32) and x (fp32, rows skewed by 4 words every 32 so the
//     128-bit loads of neighbouring chunks hit distinct banks) stay in shared
//     memory for the whole launch.
//   * Per-chunk dot products go to a shared partial array and each row is
//     then summed by one warp in a fixed order, so results are bitwise
//     deterministic.
// Other shapes use a warp-per-row generic kernel with byte loads.
#include <algorithm>
#include <mutex>
#include <numeric>

#include "cbq_common.cuh"

namespace {

using namespace cbq;

constexpr int kMaxCbSmem = 16384;     // codebook entries kept in shared memory
constexpr int kMaxStages = 8;
constexpr uint32_t kStageTarget = 48 * 1024;

struct FixedArgs {
    const void *x;
    int64_t ldx;
    int64_t t0;        // first token of this launch
    int ntok;          // tokens in this launch (<= TB)
    const uint8_t *packed;
    const float *codebook;
    int C;
    int M, K;
    const float *bias;
    void *out;
    int64_t ldo;
    int RB;            // rows per tile
    int ntiles;
    int nst;           // ring stages
    uint32_t stage_bytes;
    uint32_t *status;
};

// Load the `BITS` words of one chunk with the widest conflict-free load.
template <int BITS>
__device__ __forceinline__ void load_chunk_words(const uint32_t *p, uint32_t (&w)[BITS + 1]) {
    if constexpr (BITS % 4 == 0) {
#pragma unroll
        for (int s = 0; s < BITS / 4; ++s) {
            uint4 v = reinterpret_cast<const uint4 *>(p)[s];
            w[4 * s] = v.x; w[4 * s + 1] = v.y; w[4 * s + 2] = v.z; w[4 * s + 3] = v.w;
        }
    } else if constexpr (BITS % 2 == 0) {
#pragma unroll
        for (int s = 0; s < BITS / 2; ++s) {
            uint2 v = reinterpret_cast<const uint2 *>(p)[s];
            w[2 * s] = v.x; w[2 * s + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int s = 0; s < BITS; ++s) w[s] = p[s];
    }
    w[BITS] = 0u;
}

// Field i (0..31) of a chunk held in registers; i is a compile-time constant
// after unrolling, so this is one shift/funnel-shift and a mask.
template <int BITS>
__device__ __forceinline__ uint32_t chunk_field(const uint32_t (&w)[BITS + 1], int i) {
    const int bit = i * BITS;
    const int wi = bit >> 5;
    const int sh = bit & 31;
    constexpr uint32_t mask = (BITS == 32) ? 0xffffffffu : ((1u << BITS) - 1u);
    uint32_t v;
    if (sh + BITS <= 32) v = w[wi] >> sh;
    else v = __funnelshift_r(w[wi], w[wi + 1], sh);
    return v & mask;
}

template <int BITS, int TB, typename XT, typename OT>
__global__ void __launch_bounds__(kThreads, 1) k_linear_fixed(const FixedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int K = a.K;
    const int kc = K >> 5;              // chunks per row
    const int XS = kc * 36;             // skewed x row stride (floats)
    const int RB = a.RB, nst = a.nst;
    const int tile_chunks = RB * kc;

    // Every region starts on a 128-byte boundary (the bulk-copy destination
    // needs 16, the float4 loads of x need 16); fixed_smem() mirrors this.
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
    size_t off = 128;
    float *cb_s = reinterpret_cast<float *>(smem + off);
    off += a128((size_t)a.C * 4);
    float *xs = reinterpret_cast<float *>(smem + off);
    off += a128((size_t)TB * XS * 4);
    float *P = reinterpret_cast<float *>(smem + off);
    off += a128((size_t)TB * tile_chunks * 4);
    uint8_t *stg = smem + off;

    if (tid == 0) {
        for (int s = 0; s < nst; ++s) mbar_init(&bar[s], 1);
        mbar_fence_init();
    }
    for (int i = tid; i < a.C; i += kThreads) cb_s[i] = a.codebook[i];
    const XT *x = static_cast<const XT *>(a.x);
    for (int i = tid; i < TB * K; i += kThreads) {
        const int t = i / K, k = i - t * K;
        const float v = (t < a.ntok) ? to_f32<XT>(x[(a.t0 + t) * a.ldx + k]) : 0.f;
        xs[t * XS + (k >> 5) * 36 + (k & 31)] = v;
    }
    __syncthreads();

    const int my_tiles =
        (blockIdx.x < (unsigned)a.ntiles) ? (a.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int64_t row_bytes = (int64_t)K * BITS / 8;

    auto issue = [&](int j) {
        const int tile = blockIdx.x + j * gridDim.x;
        const int s = j % nst;
        const int rows = min(RB, a.M - tile * RB);
        const uint32_t bytes = (uint32_t)(rows * row_bytes);
        mbar_arrive_expect_tx(&bar[s], bytes);
        bulk_g2s(stg + (size_t)s * a.stage_bytes, a.packed + (int64_t)tile * RB * row_bytes, bytes,
                 &bar[s]);
    };
    if (tid == 0)
        for (int j = 0; j < min(nst, my_tiles); ++j) issue(j);

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
        const int nch = rows * kc;
        const uint32_t *sw = reinterpret_cast<const uint32_t *>(stg + (size_t)s * a.stage_bytes);
        for (int c = tid; c < nch; c += kThreads) {
            uint32_t w[BITS + 1];
            load_chunk_words<BITS>(sw + (size_t)c * BITS, w);
            const float *xb = xs + (c % kc) * 36;
            float acc[TB];
#pragma unroll
            for (int t = 0; t < TB; ++t) acc[t] = 0.f;
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                float4 xv[TB];
#pragma unroll
                for (int t = 0; t < TB; ++t)
                    xv[t] = *reinterpret_cast<const float4 *>(xb + t * XS + 4 * g);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t v = min(chunk_field<BITS>(w, 4 * g + u), cmax);
                    const float wt = cb_s[v];
#pragma unroll
                    for (int t = 0; t < TB; ++t) {
                        const float xk = (u == 0) ? xv[t].x : (u == 1) ? xv[t].y : (u == 2) ? xv[t].z : xv[t].w;
                        acc[t] = fmaf(xk, wt, acc[t]);
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < TB; ++t) P[t * tile_chunks + c] = acc[t];
        }
        __syncthreads();
        if (tid == 0 && j + nst < my_tiles) issue(j + nst);
        for (int p = warp; p < rows * TB; p += kThreads / 32) {
            const int rho = p / TB, t = p - rho * TB;
            if (t >= a.ntok) continue;
            const float *pp = P + t * tile_chunks + rho * kc;
            float sum = 0.f;
            for (int q = lane; q < kc; q += 32) sum += pp[q];
            sum = warp_sum(sum);
            if (lane == 0) {
                const int r = r0 + rho;
                if (a.bias) sum += a.bias[r];
                out[(a.t0 + t) * a.ldo + r] = from_f32<OT>(sum);
            }
        }
        __syncthreads();
    }
    // After a timeout, wait (bounded) for copies still in flight into this CTA.
    if (j < my_tiles && tid == 0) {
        for (int jj = j; jj < min(j + nst, my_tiles); ++jj)
            mbar_wait_bounded(&bar[jj % nst], (uint32_t)(jj / nst) & 1u);
    }
}

// Generic path: any K, any alignment.  One warp per row, lanes stride over k,
// byte loads of the 4-byte window like src/compressed_matmul.c:334-347.
template <typename XT, typename OT>
__global__ void __launch_bounds__(kThreads) k_linear_fixed_generic(
    const XT *x, int64_t ldx, int64_t T, const uint8_t *packed, const float *cb, int C, int bits,
    int64_t M, int64_t K, const float *bias, OT *out, int64_t ldo) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kThreads / 32);
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t r = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); r < M; r += warps) {
        for (int64_t t = 0; t < T; ++t) {
            float sum = 0.f;
            for (int64_t k = lane; k < K; k += 32) {
                const int64_t bit = (r * K + k) * bits;
                const uint8_t *p = packed + (bit >> 3);
                const uint32_t win = (uint32_t)p[0] | ((uint32_t)p[1] << 8) |
                                     ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
                const uint32_t v = min((win >> (bit & 7)) & mask, (uint32_t)(C - 1));
                sum = fmaf(to_f32<XT>(x[t * ldx + k]), __ldg(cb + v), sum);
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                if (bias) sum += bias[r];
                out[t * ldo + r] = from_f32<OT>(sum);
            }
        }
    }
}

template <typename OT>
__global__ void k_embedding_fixed(const int64_t *ids, const uint8_t *packed, const float *cb, int C,
                                  int bits, int64_t vocab, int64_t H, OT *out, uint32_t *status) {
    const int64_t t = blockIdx.y;
    const int64_t id = ids[t];
    const bool valid = id >= 0 && id < vocab;
    if (!valid && blockIdx.x == 0 && threadIdx.x == 0) report(status, CBQ_FLAG_CORRUPT, (uint32_t)t);
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t h = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; h < H;
         h += (int64_t)gridDim.x * blockDim.x) {
        float v = 0.f;
        if (valid) {
            const int64_t bit = (id * H + h) * bits;
            const uint8_t *p = packed + (bit >> 3);
            const uint32_t win = (uint32_t)p[0] | ((uint32_t)p[1] << 8) |
                                 ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
            v = __ldg(cb + min((win >> (bit & 7)) & mask, (uint32_t)(C - 1)));
        }
        out[t * H + h] = from_f32<OT>(v);
    }
}

// One thread per output 32-bit word: OR in every field that overlaps it.
__global__ void k_pack_fixed(const uint16_t *idx, int64_t n, int bits, uint32_t *out,
                             int64_t nwords) {
    const int64_t wi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (wi >= nwords) return;
    const int64_t b0 = wi * 32;
    int64_t e = b0 / bits;
    const int64_t e_end = min(n, (b0 + 31) / bits + 1);
    const uint32_t mask = (1u << bits) - 1u;
    uint32_t v = 0;
    for (; e < e_end; ++e) {
        const int64_t pos = e * bits - b0;
        const uint32_t f = (uint32_t)idx[e] & mask;
        v |= (pos >= 0) ? (uint32_t)(((uint64_t)f << pos) & 0xffffffffu) : (f >> (-pos));
    }
    out[wi] = v;
}

// ---------------------------------------------------------------- planning

struct FixedPlan {
    int RB = 0, nst = 0, TB = 0, ntiles = 0, grid = 0;
    uint32_t stage_bytes = 0;
    size_t smem = 0;
};

size_t fixed_smem(int C, int K, int RB, int TB, int nst, uint32_t stage_bytes) {
    const int kc = K / 32;
    size_t s = 128;
    s += a128((size_t)C * 4);
    s += a128((size_t)TB * kc * 36 * 4);
    s += a128((size_t)TB * RB * kc * 4);
    s += (size_t)nst * stage_bytes;
    return s;
}

bool plan_fixed(int64_t M, int64_t K, int bits, int64_t C, int64_t T, FixedPlan &p) {
    if (K <= 0 || K % 128 != 0 || K > (1 << 18) || M <= 0 || M >= (1ll << 31)) return false;
    if (C > kMaxCbSmem) return false;
    const int kc = (int)(K / 32);
    const int64_t row_bytes = K * bits / 8;
    int RB = 256 / std::gcd(kc, 256);
    while (RB > 1 && RB * row_bytes > (int64_t)kStageTarget) RB /= 2;
    if (RB * row_bytes > (int64_t)(96 * 1024)) return false;
    const size_t budget = (size_t)cbq_host::max_smem_optin() - 1024;
    const uint32_t stage = (uint32_t)(RB * row_bytes);
    // TB: the largest power of two <= min(T, 8) whose x block fits beside 2 stages.
    int TB = 8;
    while (TB > 1 && TB > T) TB /= 2;
    while (TB > 1 && fixed_smem((int)C, (int)K, RB, TB, 2, stage) > budget) TB /= 2;
    if (fixed_smem((int)C, (int)K, RB, TB, 2, stage) > budget) return false;
    int nst = 2;
    while (nst < kMaxStages && fixed_smem((int)C, (int)K, RB, TB, nst + 1, stage) <= budget) ++nst;
    p.RB = RB;
    p.TB = TB;
    p.nst = nst;
    p.stage_bytes = stage;
    p.smem = fixed_smem((int)C, (int)K, RB, TB, nst, stage);
    p.ntiles = (int)((M + RB - 1) / RB);
    p.grid = std::min(p.ntiles, cbq_host::sm_count());
    return true;
}

template <int BITS, int TB, typename XT, typename OT>
int launch_fixed_t(const FixedArgs &a, const FixedPlan &p, cudaStream_t s) {
    auto kern = k_linear_fixed<BITS, TB, XT, OT>;
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

template <int BITS, typename XT, typename OT>
int launch_fixed_tb(const FixedArgs &a, const FixedPlan &p, cudaStream_t s) {
    switch (p.TB) {
        case 1: return launch_fixed_t<BITS, 1, XT, OT>(a, p, s);
        case 2: return launch_fixed_t<BITS, 2, XT, OT>(a, p, s);
        case 4: return launch_fixed_t<BITS, 4, XT, OT>(a, p, s);
        case 8: return launch_fixed_t<BITS, 8, XT, OT>(a, p, s);
    }
    return CBQ_ERR_UNSUPPORTED;
}

template <typename XT, typename OT>
int launch_fixed_bits(int bits, const FixedArgs &a, const FixedPlan &p, cudaStream_t s) {
    switch (bits) {
#define CBQ_B(n) case n: return launch_fixed_tb<n, XT, OT>(a, p, s);
        CBQ_B(1) CBQ_B(2) CBQ_B(3) CBQ_B(4) CBQ_B(5) CBQ_B(6) CBQ_B(7) CBQ_B(8)
        CBQ_B(9) CBQ_B(10) CBQ_B(11) CBQ_B(12) CBQ_B(13) CBQ_B(14) CBQ_B(15) CBQ_B(16)
#undef CBQ_B
    }
    return CBQ_ERR_ARG;
}

template <typename XT, typename OT>
int linear_fixed_impl(const void *x, int64_t T, int64_t ldx, const uint8_t *packed,
                      const float *cb, int64_t C, int bits, int64_t M, int64_t K,
                      const float *bias, void *out, int64_t ldo, cudaStream_t s) {
    FixedPlan p;
    const bool aligned = (reinterpret_cast<uintptr_t>(packed) & 15) == 0;
    if (aligned && plan_fixed(M, K, bits, C, T, p)) {
        FixedArgs a{};
        a.x = x; a.ldx = ldx; a.packed = packed; a.codebook = cb; a.C = (int)C;
        a.M = (int)M; a.K = (int)K; a.bias = bias; a.out = out; a.ldo = ldo;
        a.RB = p.RB; a.ntiles = p.ntiles; a.nst = p.nst; a.stage_bytes = p.stage_bytes;
        a.status = nullptr;
        for (int64_t t0 = 0; t0 < T; t0 += p.TB) {
            a.t0 = t0;
            a.ntok = (int)std::min<int64_t>(p.TB, T - t0);
            const int rc = launch_fixed_bits<XT, OT>(bits, a, p, s);
            if (rc != CBQ_OK) return rc;
        }
        return CBQ_OK;
    }
    const int64_t warps_needed = M;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((warps_needed + 7) / 8,
                                                                 (int64_t)cbq_host::sm_count() * 8));
    k_linear_fixed_generic<XT, OT><<<grid, kThreads, 0, s>>>(
        static_cast<const XT *>(x), ldx, T, packed, cb, (int)C, bits, M, K, bias,
        static_cast<OT *>(out), ldo);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

}  // namespace

// ------------------------------------------------------------------- C ABI

extern "C" int64_t cbq_fixed_stream_bytes(int64_t M, int64_t K, int bits) {
    if (M < 0 || K < 0 || bits < 1 || bits > 16) return -1;
    const int64_t raw = (M * K * bits + 7) / 8;
    return cbq_host::align_up(raw, 16) + 64;
}

extern "C" int cbq_linear_fixed(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                const uint8_t *packed_dev, int64_t packed_bytes,
                                const float *codebook_dev, int64_t C, int bits, int64_t M,
                                int64_t K, const float *bias_dev, void *out_dev, int out_dtype,
                                int64_t ldo, void *stream) {
    if (T < 0 || M < 0 || K < 0 || bits < 1 || bits > 16 || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (T == 0 || M == 0) return CBQ_OK;
    if (!out_dev || !codebook_dev || (K > 0 && (!x_dev || !packed_dev))) return CBQ_ERR_ARG;
    if (ldx < K || ldo < M) return CBQ_ERR_ARG;
    if (packed_bytes < cbq_fixed_stream_bytes(M, K, bits)) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (x_dtype == CBQ_F32 && out_dtype == CBQ_F32)
        return linear_fixed_impl<float, float>(x_dev, T, ldx, packed_dev, codebook_dev, C, bits, M,
                                               K, bias_dev, out_dev, ldo, s);
    if (x_dtype == CBQ_BF16 && out_dtype == CBQ_BF16)
        return linear_fixed_impl<__nv_bfloat16, __nv_bfloat16>(x_dev, T, ldx, packed_dev,
                                                               codebook_dev, C, bits, M, K,
                                                               bias_dev, out_dev, ldo, s);
    if (x_dtype == CBQ_BF16 && out_dtype == CBQ_F32)
        return linear_fixed_impl<__nv_bfloat16, float>(x_dev, T, ldx, packed_dev, codebook_dev, C,
                                                       bits, M, K, bias_dev, out_dev, ldo, s);
    return linear_fixed_impl<float, __nv_bfloat16>(x_dev, T, ldx, packed_dev, codebook_dev, C,
                                                   bits, M, K, bias_dev, out_dev, ldo, s);
}

extern "C" int cbq_embedding_fixed(const int64_t *ids_dev, int64_t T, const uint8_t *packed_dev,
                                   int64_t packed_bytes, const float *codebook_dev, int64_t C,
                                   int bits, int64_t vocab, int64_t H, void *out_dev,
                                   int out_dtype, uint32_t *status_dev, void *stream) {
    if (T < 0 || vocab < 0 || H < 0 || bits < 1 || bits > 16 || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16) return CBQ_ERR_ARG;
    if (T == 0 || H == 0) return CBQ_OK;
    if (!ids_dev || !packed_dev || !codebook_dev || !out_dev) return CBQ_ERR_ARG;
    if (packed_bytes < cbq_fixed_stream_bytes(vocab, H, bits)) return CBQ_ERR_ARG;
    if (T > 65535) return CBQ_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    dim3 grid((unsigned)std::min<int64_t>((H + 255) / 256, 64), (unsigned)T);
    if (out_dtype == CBQ_F32)
        k_embedding_fixed<float><<<grid, 256, 0, s>>>(ids_dev, packed_dev, codebook_dev, (int)C, bits,
                                                      vocab, H, static_cast<float *>(out_dev),
                                                      status_dev);
    else
        k_embedding_fixed<__nv_bfloat16><<<grid, 256, 0, s>>>(
            ids_dev, packed_dev, codebook_dev, (int)C, bits, vocab, H,
            static_cast<__nv_bfloat16 *>(out_dev), status_dev);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

extern "C" int cbq_pack_fixed(const uint16_t *idx_dev, int64_t n, int bits, uint8_t *out_dev,
                              int64_t out_bytes, void *stream) {
    if (n < 0 || bits < 1 || bits > 16) return CBQ_ERR_ARG;
    const int64_t nbytes = (n * bits + 7) / 8;
    const int64_t nwords = (nbytes + 3) / 4;
    if (out_bytes < nwords * 4) return CBQ_ERR_ARG;
    if (n == 0) return CBQ_OK;
    if (!idx_dev || !out_dev || (reinterpret_cast<uintptr_t>(out_dev) & 3)) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    k_pack_fixed<<<(unsigned)((nwords + 255) / 256), 256, 0, s>>>(
        idx_dev, n, bits, reinterpret_cast<uint32_t *>(out_dev), nwords);
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}
