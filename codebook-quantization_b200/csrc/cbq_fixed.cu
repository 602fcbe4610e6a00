// cbq_fixed.cu -- fixed-width codebook decode-GEMV (host side), generic
// kernel, embedding and device packer (sm_100a).
//
// Stream format: element e of the row-major [M, K] index matrix occupies bits
// [e*b, (e+1)*b) of an LSB-first byte stream (reference src/bitpack.py:32-94,
// read by src/compressed_matmul.c:334-347).
//
// The fast GEMV (k_linear_fixed, cbq_fixed_kernel.cuh) needs K % 128 == 0, a
// 16-byte aligned stream and a codebook whose fp32 copy fits in shared
// memory; every other shape runs k_linear_fixed_generic (one warp per row,
// byte loads of the 4-byte window, like the reference).
#include <algorithm>
#include <mutex>

#include "cbq_fixed_kernel.cuh"
#include "cbq_gemv_kernel.cuh"

namespace cbq {
int gemm_fixed(const void *x, int64_t T, int64_t ldx, const uint8_t *packed, const float *cb, int64_t C,
               int bits, int64_t M, int64_t K, const float *bias, void *out, int out_dtype, int64_t ldo,
               cudaStream_t s);
int gemm_small(const void *x, int64_t T, int64_t ldx, const uint8_t *packed, const float *cb, int64_t C, int bits,
               int64_t M, int64_t K, const float *bias, void *out, int out_dtype, int64_t ldo, void *ws,
               int64_t ws_bytes, cudaStream_t s);
int64_t gemm_small_workspace_bytes(int64_t M, int64_t K, int64_t T);
template <int BITS>
int launch_fixed_bits(int TB, bool x_bf16, const FixedArgs &a, size_t smem, int grid, cudaStream_t s);
template <int BITS>
int launch_gemv_bits(int TB, int NF, bool x_bf16, const GemvArgs &a, size_t smem, int grid, cudaStream_t s);
}

namespace {

using namespace cbq;

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

// idx[i] = field i of an LSB-first b-bit stream (the 4-byte window read of
// src/compressed_matmul.c:334-347); grid-stride.
__global__ void k_unpack_fixed(const uint8_t *packed, int bits, int64_t n, uint16_t *out) {
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bit = i * bits;
        const uint8_t *p = packed + (bit >> 3);
        const uint32_t win = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                             ((uint32_t)p[3] << 24);
        out[i] = (uint16_t)((win >> (bit & 7)) & mask);
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
    int TB = 0, grid = 0, nseg = 0;
    uint32_t cb_bytes = 0;
    size_t smem = 0;
};

// Shared-memory plan for the fast kernel; false -> generic kernel.
bool plan_fixed(int64_t M, int64_t K, int bits, int64_t C, int64_t T, int xbytes, FixedPlan &p) {
    if (K <= 0 || K % 128 != 0 || K > (1 << 18) || M <= 0 || M >= (1ll << 31)) return false;
    const size_t budget = (size_t)cbq_host::max_smem_optin() - 256;
    const size_t ring = (size_t)kFxWarps * kFxSlots * kFxSeg * bits / 8;
    if ((size_t)C * 4 > ring) return false;       // the fp32 codebook is staged in the ring area
    const int64_t np = (bits <= 14) ? std::max<int64_t>(C, 1ll << bits) : C;   // single-copy entries
    int TB = 8;
    while (TB > 1 && TB > T) TB /= 2;
    for (; TB >= 1; TB /= 2) {
        const size_t prefix = fixed_prefix_bytes((int)K, TB, xbytes);
        if (prefix + ring + 128 + a128((size_t)np * 4) <= budget) break;
        if (TB == 1) return false;
    }
    const size_t prefix = fixed_prefix_bytes((int)K, TB, xbytes);
    const size_t cb = (budget - prefix - ring) & ~(size_t)127;
    p.TB = TB;
    p.nseg = (int)((K + kFxSeg - 1) / kFxSeg);
    p.cb_bytes = (uint32_t)cb;
    p.smem = prefix + cb + ring;
    p.grid = cbq_host::sm_count();
    return true;
}

// Token counts served by the small-batch tensor-core GEMM (bf16 activations).
constexpr int64_t kSmallGemmMinTokens = 3;

int64_t workspace_bytes_for(int64_t M, int64_t K, int64_t T) {
    const int64_t nseg = (K + kFxSeg - 1) / kFxSeg;
    const int64_t TB = T >= 8 ? 8 : T >= 4 ? 4 : T >= 2 ? 2 : 1;
    const int64_t split_rows = cbq_host::align_up(M * nseg * TB * 4, 256) + cbq_host::align_up(M * 4, 256);
    // 3..63 tokens: also the split-K partial tiles of the tensor-core path
    const int64_t small = (T >= kSmallGemmMinTokens && T < 64) ? gemm_small_workspace_bytes(M, K, T) : 0;
    return std::max(split_rows, small);
}

// Token count from which cbq_linear_fixed uses the tensor-core GEMM.
constexpr int64_t kGemmMinTokens = 64;

// Plan of the one/two-token kernel (k_gemv_fixed); false -> k_linear_fixed.
struct GemvPlan {
    int grid = 0, rows_per_cta = 0, nseg = 0, nf = 32;
    uint32_t H = 0, NP = 0;
    size_t smem = 0;
};

bool plan_gemv(int64_t M, int64_t K, int bits, int64_t C, int64_t T, GemvPlan &p, bool even_rows = false,
               size_t xs_bytes = 0) {
    if (T < 1 || T > 2 || K <= 0 || K % 128 != 0 || K > (1 << 20) || M <= 0 || M >= (1ll << 31))
        return false;
    const int64_t sms = cbq_host::sm_count();
    int64_t rows = (M + sms - 1) / sms;
    if (even_rows) rows += rows & 1;
    // units of 64 indices per lane when every warp still gets several of them
    const int64_t units64 = rows * ((K + GvCfg<64>::kSeg - 1) / GvCfg<64>::kSeg);
    const int nf = (T == 1 && units64 >= 6 * kGvWarps) ? 64 : 32;
    const int nseg = (int)((K + 32 * nf - 1) / (32 * nf));
    const int64_t NP = (bits <= 14) ? std::max<int64_t>(C, 1ll << bits) : C;
    const size_t budget = (size_t)cbq_host::max_smem_optin();
    const size_t fixed = kGvBarBytes + gemv_part_bytes((int)rows, nseg, (int)T) + gemv_ring_bytes(bits, nf) +
                         a128(xs_bytes);
    if (fixed + a128((size_t)NP * 4) > budget) return false;
    int64_t H = (int64_t)((budget - fixed - 128 - (size_t)NP * 4) / 124);
    H = std::min<int64_t>(H, C);
    // The replicated head costs 128 bytes of shared-memory stores per entry in
    // every CTA; for a small share of the stream per CTA those stores cost more
    // than the bank conflicts they save, so the head shrinks with the share.
    const int64_t cta_bytes = rows * K * bits / 8;
    H = std::min<int64_t>(H, std::max<int64_t>(64, cta_bytes / 256));
    p.grid = (int)((M + rows - 1) / rows);
    p.rows_per_cta = (int)rows;
    p.nseg = nseg;
    p.nf = nf;
    p.H = (uint32_t)H;
    p.NP = (uint32_t)NP;
    p.smem = fixed + gemv_cb_bytes(p.H, p.NP);
    return p.smem <= budget;
}

int launch_gemv(int bits, int TB, int NF, bool xbf16, const GemvArgs &a, size_t smem, int grid,
                cudaStream_t s) {
    switch (bits) {
#define CBQ_B(n) case n: return launch_gemv_bits<n>(TB, NF, xbf16, a, smem, grid, s);
        CBQ_B(1) CBQ_B(2) CBQ_B(3) CBQ_B(4) CBQ_B(5) CBQ_B(6) CBQ_B(7) CBQ_B(8)
        CBQ_B(9) CBQ_B(10) CBQ_B(11) CBQ_B(12) CBQ_B(13) CBQ_B(14) CBQ_B(15) CBQ_B(16)
#undef CBQ_B
    }
    return CBQ_ERR_ARG;
}

int launch_bits(int bits, int TB, bool xbf16, const FixedArgs &a, size_t smem, int grid,
                cudaStream_t s) {
    switch (bits) {
#define CBQ_B(n) case n: return launch_fixed_bits<n>(TB, xbf16, a, smem, grid, s);
        CBQ_B(1) CBQ_B(2) CBQ_B(3) CBQ_B(4) CBQ_B(5) CBQ_B(6) CBQ_B(7) CBQ_B(8)
        CBQ_B(9) CBQ_B(10) CBQ_B(11) CBQ_B(12) CBQ_B(13) CBQ_B(14) CBQ_B(15) CBQ_B(16)
#undef CBQ_B
    }
    return CBQ_ERR_ARG;
}

}  // namespace

namespace cbq {

// The fixed-width dispatch behind cbq_linear_fixed and
// cbq_linear_fixed_noalloc.  Only k_linear_fixed (3..63 tokens, or fp32
// activations) uses the workspace.  ws_mode kWsCallerZeroed: `ws` (may be
// null) is kept zeroed by the kernels, as cbq_linear_fixed promises its
// caller; kWsClearFirst: `ws` is a shared array holding an earlier call's
// bytes -- a call that needs more than ws_bytes returns CBQ_ERR_ARG before
// launching, and the bytes it uses are cleared on `s` first.
int linear_fixed_impl(const void *x, int x_dtype, int64_t T, int64_t ldx, const uint8_t *packed,
                      const float *cb, int64_t C, int bits, int64_t M, int64_t K, const float *bias,
                      void *out, int out_dtype, int64_t ldo, void *ws, int64_t ws_bytes,
                      cudaStream_t s, int ws_mode) {
    FixedPlan p;
    const bool aligned = (reinterpret_cast<uintptr_t>(packed) & 15) == 0;
    const int xbytes = x_dtype == CBQ_BF16 ? 2 : 4;
    const bool x_aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx * xbytes) % 16 == 0;
    // many tokens, bf16 activations: the tensor-core GEMM (cbq_gemm.cu)
    if (T >= kGemmMinTokens && x_dtype == CBQ_BF16) {
        const int rc = gemm_fixed(x, T, ldx, packed, cb, C, bits, M, K, bias, out, out_dtype, ldo, s);
        if (rc != CBQ_ERR_UNSUPPORTED) return rc;
    }
    // 3..63 bf16 tokens (decode batches): the split-K tensor-core GEMM
    if (T >= kSmallGemmMinTokens && T < kGemmMinTokens && x_dtype == CBQ_BF16) {
        const int64_t need = gemm_small_workspace_bytes(M, K, T);
        if (need == 0 || (ws && ws_bytes >= need)) {
            if (need > 0 && ws_mode == kWsClearFirst) CBQ_CUDA_TRY(cudaMemsetAsync(ws, 0, (size_t)need, s));
            const int rc = gemm_small(x, T, ldx, packed, cb, C, bits, M, K, bias, out, out_dtype, ldo, ws, ws_bytes, s);
            if (rc != CBQ_ERR_UNSUPPORTED) return rc;
        }
    }
    GemvPlan g;
    if (aligned && x_aligned && plan_gemv(M, K, bits, C, T, g)) {
        GemvArgs a{};
        a.x = x; a.ldx = ldx; a.t0 = 0; a.ntok = (int)T; a.codebook = cb;
        a.C = (int)C; a.M = (int)M; a.K = (int)K; a.nseg = g.nseg; a.rows_per_cta = g.rows_per_cta;
        a.nmat = 1; a.epi = kEpiStore;
        a.mat[0] = GemvMat{packed, out, bias, nullptr, ldo, (int)M};
        a.out_bf16 = out_dtype == CBQ_BF16;
        a.H = g.H; a.NP = g.NP; a.m128 = 128u; a.m4 = 4u; a.status = nullptr;
        return launch_gemv(bits, (int)T, g.nf, x_dtype == CBQ_BF16, a, g.smem, g.grid, s);
    }
    if (aligned && plan_fixed(M, K, bits, C, T, xbytes, p)) {
        FixedArgs a{};
        a.x = x; a.ldx = ldx; a.packed = packed; a.codebook = cb; a.C = (int)C;
        a.M = (int)M; a.K = (int)K; a.nseg = p.nseg; a.bias = bias; a.out = out; a.ldo = ldo;
        a.out_bf16 = out_dtype == CBQ_BF16; a.cb_bytes = p.cb_bytes; a.status = nullptr;
        const int64_t need = workspace_bytes_for(M, K, T);
        if (ws_mode == kWsClearFirst) {
            if (!ws || ws_bytes < need) return CBQ_ERR_ARG;
            CBQ_CUDA_TRY(cudaMemsetAsync(ws, 0, (size_t)need, s));
        }
        if (ws && ws_bytes >= need) {
            const int64_t pb = cbq_host::align_up(M * p.nseg * p.TB * 4, 256);
            a.part = static_cast<float *>(ws);
            a.cnt = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(ws) + pb);
        }
        for (int64_t t0 = 0; t0 < T; t0 += p.TB) {
            a.t0 = t0;
            a.ntok = (int)std::min<int64_t>(p.TB, T - t0);
            const int rc = launch_bits(bits, p.TB, x_dtype == CBQ_BF16, a, p.smem, p.grid, s);
            if (rc != CBQ_OK) return rc;
        }
        return CBQ_OK;
    }
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>((M + 7) / 8, (int64_t)cbq_host::sm_count() * 8));
#define CBQ_GEN(XT, OT)                                                                        \
    k_linear_fixed_generic<XT, OT><<<grid, kThreads, 0, s>>>(                                  \
        static_cast<const XT *>(x), ldx, T, packed, cb, (int)C, bits, M, K, bias,              \
        static_cast<OT *>(out), ldo)
    if (x_dtype == CBQ_F32 && out_dtype == CBQ_F32) CBQ_GEN(float, float);
    else if (x_dtype == CBQ_BF16 && out_dtype == CBQ_BF16) CBQ_GEN(__nv_bfloat16, __nv_bfloat16);
    else if (x_dtype == CBQ_BF16) CBQ_GEN(__nv_bfloat16, float);
    else CBQ_GEN(float, __nv_bfloat16);
#undef CBQ_GEN
    CBQ_CUDA_TRY(cudaGetLastError());
    return CBQ_OK;
}

}  // namespace cbq

// ------------------------------------------------------------------- C ABI

extern "C" int64_t cbq_fixed_stream_bytes(int64_t M, int64_t K, int bits) {
    if (M < 0 || K < 0 || bits < 1 || bits > 16) return -1;
    const int64_t raw = (M * K * bits + 7) / 8;
    return cbq_host::align_up(raw, 16) + 64;
}

extern "C" int64_t cbq_linear_fixed_workspace_bytes(int64_t M, int64_t K, int64_t T) {
    if (M < 0 || K < 0 || T < 0) return -1;
    return workspace_bytes_for(M, K, T);
}

extern "C" int cbq_linear_fixed(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                const uint8_t *packed_dev, int64_t packed_bytes,
                                const float *codebook_dev, int64_t C, int bits, int64_t M,
                                int64_t K, const float *bias_dev, void *out_dev, int out_dtype,
                                int64_t ldo, void *workspace_dev, int64_t workspace_bytes,
                                void *stream) {
    if (T < 0 || M < 0 || K < 0 || bits < 1 || bits > 16 || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (T == 0 || M == 0) return CBQ_OK;
    if (!out_dev || !codebook_dev || (K > 0 && (!x_dev || !packed_dev))) return CBQ_ERR_ARG;
    if (ldx < K || ldo < M) return CBQ_ERR_ARG;
    if (packed_bytes < cbq_fixed_stream_bytes(M, K, bits)) return CBQ_ERR_ARG;
    if (workspace_dev && workspace_bytes < workspace_bytes_for(M, K, T)) return CBQ_ERR_ARG;
    return cbq::linear_fixed_impl(x_dev, x_dtype, T, ldx, packed_dev, codebook_dev, C, bits, M, K,
                                  bias_dev, out_dev, out_dtype, ldo, workspace_dev, workspace_bytes,
                                  static_cast<cudaStream_t>(stream), cbq::kWsCallerZeroed);
}

namespace {

int linear_fixed_multi_impl(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat,
                            const uint8_t *const *packed_dev, const int64_t *packed_bytes, const int64_t *M,
                            const float *codebook_dev, int64_t C, int bits, int64_t K,
                            const float *const *bias_dev, void *const *out_dev, const int64_t *ldo,
                            const void *const *resid_dev, int out_dtype, int epilogue, int pn_on,
                            const float *pn_w, float pn_eps, void *stream, const GemvArgs *ar = nullptr) {
    if (nmat < 1 || nmat > kGvMaxMats || !packed_dev || !packed_bytes || !M || !out_dev || !ldo)
        return CBQ_ERR_ARG;
    if (T < 0 || K < 0 || bits < 1 || bits > 16 || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (epilogue != CBQ_EPI_STORE && epilogue != CBQ_EPI_RESIDUAL && epilogue != CBQ_EPI_SILU_MUL)
        return CBQ_ERR_ARG;
    if (epilogue == CBQ_EPI_SILU_MUL && (nmat != 2 || M[0] != M[1])) return CBQ_ERR_ARG;
    if (epilogue == CBQ_EPI_RESIDUAL && !resid_dev) return CBQ_ERR_ARG;
    int64_t Mt = 0;
    for (int m = 0; m < nmat; ++m) {
        if (M[m] < 1 || !packed_dev[m] || !out_dev[m] || ldo[m] < M[m]) return CBQ_ERR_ARG;
        if (packed_bytes[m] < cbq_fixed_stream_bytes(M[m], K, bits)) return CBQ_ERR_ARG;
        if ((reinterpret_cast<uintptr_t>(packed_dev[m]) & 15) != 0) return CBQ_ERR_UNSUPPORTED;
        if (epilogue == CBQ_EPI_RESIDUAL && !resid_dev[m]) return CBQ_ERR_ARG;
        Mt += M[m];
    }
    if (T == 0) return CBQ_OK;
    if (!x_dev || !codebook_dev || ldx < K) return CBQ_ERR_ARG;
    const int xbytes = x_dtype == CBQ_BF16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(x_dev) & 15) != 0 || (ldx * xbytes) % 16 != 0) return CBQ_ERR_UNSUPPORTED;
    GemvPlan g;
    const size_t xs_bytes = ar ? (size_t)T * K * xbytes : 0;     // the all-reduced activations in shared memory
    if (!plan_gemv(Mt, K, bits, C, T, g, epilogue == CBQ_EPI_SILU_MUL, xs_bytes)) return CBQ_ERR_UNSUPPORTED;
    GemvArgs a{};
    a.x = x_dev; a.ldx = ldx; a.t0 = 0; a.ntok = (int)T; a.codebook = codebook_dev;
    a.C = (int)C; a.M = (int)Mt; a.K = (int)K; a.nseg = g.nseg; a.rows_per_cta = g.rows_per_cta;
    a.nmat = nmat; a.epi = epilogue;
    for (int m = 0; m < nmat; ++m)
        a.mat[m] = GemvMat{packed_dev[m], out_dev[m], bias_dev ? bias_dev[m] : nullptr,
                           resid_dev ? resid_dev[m] : nullptr, ldo[m], (int)M[m]};
    a.out_bf16 = out_dtype == CBQ_BF16;
    a.H = g.H; a.NP = g.NP; a.m128 = 128u; a.m4 = 4u; a.status = nullptr;
    a.pn_on = pn_on; a.pn_w = pn_w; a.pn_eps = pn_eps;
    if (ar) {
        a.ar_on = 1; a.ar_world = ar->ar_world; a.ar_slots = ar->ar_slots; a.ar_counts = ar->ar_counts;
        a.ar_epoch = ar->ar_epoch; a.ar_expect = ar->ar_expect; a.ar_resid = ar->ar_resid; a.ar_ll = ar->ar_ll;
        a.status = ar->status;
    }
    return launch_gemv(bits, (int)T, g.nf, x_dtype == CBQ_BF16, a, g.smem, g.grid,
                       static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" int cbq_linear_fixed_multi(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat,
                                      const uint8_t *const *packed_dev, const int64_t *packed_bytes,
                                      const int64_t *M, const float *codebook_dev, int64_t C, int bits,
                                      int64_t K, const float *const *bias_dev, void *const *out_dev,
                                      const int64_t *ldo, const void *const *resid_dev, int out_dtype,
                                      int epilogue, void *stream) {
    return linear_fixed_multi_impl(x_dev, x_dtype, T, ldx, nmat, packed_dev, packed_bytes, M, codebook_dev, C,
                                   bits, K, bias_dev, out_dev, ldo, resid_dev, out_dtype, epilogue, 0, nullptr,
                                   0.f, stream);
}

extern "C" int cbq_linear_fixed_multi_norm(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat,
                                           const uint8_t *const *packed_dev, const int64_t *packed_bytes,
                                           const int64_t *M, const float *codebook_dev, int64_t C, int bits,
                                           int64_t K, const float *const *bias_dev, void *const *out_dev,
                                           const int64_t *ldo, const void *const *resid_dev, int out_dtype,
                                           int epilogue, const float *norm_weight_dev, float eps, void *stream) {
    return linear_fixed_multi_impl(x_dev, x_dtype, T, ldx, nmat, packed_dev, packed_bytes, M, codebook_dev, C,
                                   bits, K, bias_dev, out_dev, ldo, resid_dev, out_dtype, epilogue, 1,
                                   norm_weight_dev, eps, stream);
}

extern "C" int cbq_linear_fixed_multi_allreduce_norm(
    const void *x_dev, int x_dtype, int64_t T, int64_t ldx, int nmat, const uint8_t *const *packed_dev,
    const int64_t *packed_bytes, const int64_t *M, const float *codebook_dev, int64_t C, int bits, int64_t K,
    const float *const *bias_dev, void *const *out_dev, const int64_t *ldo, const void *const *resid_dev,
    int out_dtype, int epilogue, const float *norm_weight_dev, float eps, int world, const void *resid_in_dev,
    const void *local_slots_dev, const uint32_t *local_counts_dev, const uint32_t *epoch_dev, int64_t expect,
    uint32_t *status_dev, void *stream) {
    // local_counts_dev NULL: the slots are in the flagged form
    // (cbq_linear_fixed_peer_flagged) and expect is unused
    const bool ll = local_counts_dev == nullptr;
    if (world < 1 || world > kGvMaxPeers || !resid_in_dev || !local_slots_dev || !epoch_dev ||
        (!ll && (expect < 1 || expect > 0xffffffffll)) || resid_in_dev == x_dev)
        return CBQ_ERR_ARG;
    if (ll && ((reinterpret_cast<uintptr_t>(local_slots_dev) & 7) || (x_dtype == CBQ_BF16 && K % 2)))
        return CBQ_ERR_ARG;
    GemvArgs ar{};
    ar.ar_world = world; ar.ar_slots = local_slots_dev; ar.ar_counts = local_counts_dev; ar.ar_epoch = epoch_dev;
    ar.ar_expect = (uint32_t)expect; ar.ar_resid = resid_in_dev; ar.status = status_dev; ar.ar_ll = ll;
    return linear_fixed_multi_impl(x_dev, x_dtype, T, ldx, nmat, packed_dev, packed_bytes, M, codebook_dev, C,
                                   bits, K, bias_dev, out_dev, ldo, resid_dev, out_dtype, epilogue, 1,
                                   norm_weight_dev, eps, stream, &ar);
}

namespace {

// GemvArgs of the one-matrix peer-partial GEMV (cbq_linear_fixed_peer*).
int peer_args(const void *x_dev, int x_dtype, int64_t T, int64_t ldx, const uint8_t *packed_dev,
              int64_t packed_bytes, const float *codebook_dev, int64_t C, int bits, int64_t M, int64_t K,
              const float *bias_dev, int world, void *const *slot_dev, uint32_t *const *count_dev, int64_t ldo,
              int out_dtype, GemvArgs &a, GemvPlan &g, const uint32_t *ll_epoch = nullptr) {
    if (world < 1 || world > kGvMaxPeers || !slot_dev || (!count_dev && !ll_epoch)) return CBQ_ERR_ARG;
    // flagged bf16 slots hold row pairs: even M and an even row split
    const bool pairs = ll_epoch && out_dtype == CBQ_BF16;
    if (pairs && (M % 2 || ldo % 2)) return CBQ_ERR_UNSUPPORTED;
    if (T < 1 || M < 1 || K < 1 || bits < 1 || bits > 16 || C < 1 || C > 65536 || ldo < M) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (!x_dev || !packed_dev || !codebook_dev || ldx < K) return CBQ_ERR_ARG;
    if (packed_bytes < cbq_fixed_stream_bytes(M, K, bits)) return CBQ_ERR_ARG;
    for (int p = 0; p < world; ++p)
        if (!slot_dev[p] || (!ll_epoch && !count_dev[p]) || (ll_epoch && (reinterpret_cast<uintptr_t>(slot_dev[p]) & 7)))
            return CBQ_ERR_ARG;
    const int xbytes = x_dtype == CBQ_BF16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(x_dev) & 15) || (ldx * xbytes) % 16 || (reinterpret_cast<uintptr_t>(packed_dev) & 15))
        return CBQ_ERR_UNSUPPORTED;
    if (!plan_gemv(M, K, bits, C, T, g, pairs)) return CBQ_ERR_UNSUPPORTED;
    a = GemvArgs{};
    a.x = x_dev; a.ldx = ldx; a.t0 = 0; a.ntok = (int)T; a.codebook = codebook_dev;
    a.C = (int)C; a.M = (int)M; a.K = (int)K; a.nseg = g.nseg; a.rows_per_cta = g.rows_per_cta;
    a.nmat = 1; a.epi = kEpiPeer;
    a.mat[0] = GemvMat{packed_dev, nullptr, bias_dev, nullptr, ldo, (int)M};
    a.out_bf16 = out_dtype == CBQ_BF16;
    a.H = g.H; a.NP = g.NP; a.m128 = 128u; a.m4 = 4u; a.status = nullptr;
    a.peers.world = world;
    a.peers.ll_epoch = ll_epoch;
    for (int p = 0; p < world; ++p) {
        a.peers.slot[p] = slot_dev[p];
        a.peers.count[p] = count_dev ? count_dev[p] : nullptr;
    }
    return CBQ_OK;
}

}  // namespace

extern "C" int cbq_linear_fixed_peer_flagged(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                             const uint8_t *packed_dev, int64_t packed_bytes,
                                             const float *codebook_dev, int64_t C, int bits, int64_t M, int64_t K,
                                             const float *bias_dev, int world, void *const *slot_dev,
                                             const uint32_t *epoch_dev, int64_t ldo, int out_dtype, void *stream) {
    if (!epoch_dev) return CBQ_ERR_ARG;
    GemvArgs a;
    GemvPlan g;
    const int rc = peer_args(x_dev, x_dtype, T, ldx, packed_dev, packed_bytes, codebook_dev, C, bits, M, K, bias_dev,
                             world, slot_dev, nullptr, ldo, out_dtype, a, g, epoch_dev);
    if (rc != CBQ_OK) return rc;
    return launch_gemv(bits, (int)T, g.nf, x_dtype == CBQ_BF16, a, g.smem, g.grid,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cbq_linear_fixed_peer(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                     const uint8_t *packed_dev, int64_t packed_bytes, const float *codebook_dev,
                                     int64_t C, int bits, int64_t M, int64_t K, const float *bias_dev, int world,
                                     void *const *slot_dev, uint32_t *const *count_dev, int64_t ldo, int out_dtype,
                                     void *stream) {
    GemvArgs a;
    GemvPlan g;
    const int rc = peer_args(x_dev, x_dtype, T, ldx, packed_dev, packed_bytes, codebook_dev, C, bits, M, K, bias_dev,
                             world, slot_dev, count_dev, ldo, out_dtype, a, g);
    if (rc != CBQ_OK) return rc;
    return launch_gemv(bits, (int)T, g.nf, x_dtype == CBQ_BF16, a, g.smem, g.grid,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cbq_linear_fixed_peer_norm(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                          const uint8_t *packed_dev, int64_t packed_bytes,
                                          const float *codebook_dev, int64_t C, int bits, int64_t M, int64_t K,
                                          const float *bias_dev, int world, void *const *slot_dev,
                                          uint32_t *const *count_dev, int64_t ldo, int out_dtype,
                                          const void *local_slots_dev, const uint32_t *local_counts_dev,
                                          const uint32_t *epoch_dev, int64_t expect, void *resid_dev, int64_t ldr,
                                          const float *norm_weight_dev, float eps, void *norm_out_dev, int64_t ldn,
                                          uint32_t *arrive_dev, uint32_t *status_dev, void *stream) {
    GemvArgs a;
    GemvPlan g;
    const int rc = peer_args(x_dev, x_dtype, T, ldx, packed_dev, packed_bytes, codebook_dev, C, bits, M, K, bias_dev,
                             world, slot_dev, count_dev, ldo, out_dtype, a, g);
    if (rc != CBQ_OK) return rc;
    if (!local_slots_dev || !local_counts_dev || !epoch_dev || !resid_dev || !norm_out_dev || !arrive_dev ||
        expect < 1 || expect > 0xffffffffll || ldr < M || ldn < M)
        return CBQ_ERR_ARG;
    a.status = status_dev;
    a.norm = GemvNorm{arrive_dev, norm_weight_dev, eps, norm_out_dev, ldn, resid_dev, ldr, local_slots_dev,
                      local_counts_dev, epoch_dev, (uint32_t)expect};
    return launch_gemv(bits, (int)T, g.nf, x_dtype == CBQ_BF16, a, g.smem, g.grid,
                       static_cast<cudaStream_t>(stream));
}

extern "C" int cbq_linear_fixed_residual_norm(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                              const uint8_t *packed_dev, int64_t packed_bytes,
                                              const float *codebook_dev, int64_t C, int bits, int64_t M,
                                              int64_t K, const float *bias_dev, void *resid_dev, int64_t ldr,
                                              int out_dtype, const float *norm_weight_dev, float eps,
                                              void *norm_out_dev, int64_t ldn, uint32_t *arrive_dev,
                                              void *stream) {
    if (T < 1 || M < 1 || K < 1 || bits < 1 || bits > 16 || C < 1 || C > 65536 || ldr < M || ldn < M)
        return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (!x_dev || !packed_dev || !codebook_dev || !resid_dev || !norm_out_dev || !arrive_dev || ldx < K)
        return CBQ_ERR_ARG;
    if (packed_bytes < cbq_fixed_stream_bytes(M, K, bits)) return CBQ_ERR_ARG;
    const int xbytes = x_dtype == CBQ_BF16 ? 2 : 4;
    if ((reinterpret_cast<uintptr_t>(x_dev) & 15) || (ldx * xbytes) % 16 || (reinterpret_cast<uintptr_t>(packed_dev) & 15))
        return CBQ_ERR_UNSUPPORTED;
    GemvPlan g;
    if (!plan_gemv(M, K, bits, C, T, g)) return CBQ_ERR_UNSUPPORTED;
    GemvArgs a{};
    a.x = x_dev; a.ldx = ldx; a.t0 = 0; a.ntok = (int)T; a.codebook = codebook_dev;
    a.C = (int)C; a.M = (int)M; a.K = (int)K; a.nseg = g.nseg; a.rows_per_cta = g.rows_per_cta;
    a.nmat = 1; a.epi = kEpiResidual;
    a.mat[0] = GemvMat{packed_dev, resid_dev, bias_dev, resid_dev, ldr, (int)M};
    a.out_bf16 = out_dtype == CBQ_BF16;
    a.H = g.H; a.NP = g.NP; a.m128 = 128u; a.m4 = 4u; a.status = nullptr;
    a.norm = GemvNorm{arrive_dev, norm_weight_dev, eps, norm_out_dev, ldn, resid_dev, ldr, nullptr, nullptr,
                      nullptr, 0u};
    return launch_gemv(bits, (int)T, g.nf, x_dtype == CBQ_BF16, a, g.smem, g.grid,
                       static_cast<cudaStream_t>(stream));
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

extern "C" int cbq_unpack_fixed(const uint8_t *packed_dev, int64_t packed_bytes, int bits, int64_t n,
                                uint16_t *idx_dev, void *stream) {
    if (n < 0 || bits < 1 || bits > 16) return CBQ_ERR_ARG;
    if (n == 0) return CBQ_OK;
    if (!packed_dev || !idx_dev || packed_bytes < cbq_fixed_stream_bytes(1, n, bits)) return CBQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)cbq_host::sm_count() * 16);
    k_unpack_fixed<<<(unsigned)blocks, 256, 0, s>>>(packed_dev, bits, n, idx_dev);
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
