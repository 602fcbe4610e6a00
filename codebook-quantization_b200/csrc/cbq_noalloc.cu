// cbq_noalloc.cu -- cbq_linear_fixed_noalloc: the fixed-width decode-GEMV for
// callers that cannot allocate device memory.
//
// Some hosts own every byte of device memory themselves -- a plugin running
// inside a serving framework or game engine that hands it only input and
// output buffers, a runtime with a fixed memory pool, a real-time path where
// an allocation (and the synchronisation cudaFree implies) is not allowed --
// and cannot give cbq_linear_fixed the workspace it uses to combine rows that
// are split between warps.  This entry point supplies that workspace from a
// fixed-size array compiled into the library (kNoAllocScratchBytes, resident
// on every GPU that loads the library until the process exits) and otherwise
// behaves exactly like cbq_linear_fixed.  It never calls cudaMalloc or
// cudaFree.  Only the kernel for 3..63 tokens (and fp32 activations at 64 or
// more) uses the array; the one/two-token GEMV and the tensor-core GEMM run
// without it, so for them the size limit and the clearing do not apply.
#include <cuda.h>

#include <mutex>

#include "cbq_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = CBQ_NOALLOC_SCRATCH_BYTES;

// The workspace shared by every call on a device.  In host code this name is
// only a stand-in for the symbol: its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device addresses are per context, so the cache is keyed by the current
// driver context (a host framework may make its own contexts besides the
// primary one).  cuCtxGetCurrent is reached through the runtime's driver
// entry-point query, so the library needs no link-time libcuda.
using CtxGetCurrent = CUresult (*)(CUcontext *);

struct ScratchCache {
    std::mutex mu;
    CtxGetCurrent get_ctx = nullptr;
    bool resolved = false;
    static constexpr int kSlots = 64;
    CUcontext ctx[kSlots] = {};
    void *addr[kSlots] = {};
    int used = 0;
};
ScratchCache g_cache;

int lookup_symbol(void **addr) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return CBQ_ERR_CUDA;
    *addr = p;
    return CBQ_OK;
}

// Device address of the scratch array in the current context.  The first
// call in a context looks it up (make that first call before any stream
// capture in the context); later calls reuse it.  Without the driver entry
// point every call looks the address up.
int scratch_address(void **addr) {
    std::lock_guard<std::mutex> g(g_cache.mu);
    if (!g_cache.resolved) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_cache.get_ctx = reinterpret_cast<CtxGetCurrent>(fn);
        g_cache.resolved = true;
    }
    auto current = [](CUcontext &c) {
        return g_cache.get_ctx && g_cache.get_ctx(&c) == CUDA_SUCCESS && c;
    };
    CUcontext ctx = nullptr;
    if (current(ctx)) {
        for (int i = 0; i < g_cache.used; ++i)
            if (g_cache.ctx[i] == ctx) {
                *addr = g_cache.addr[i];
                return CBQ_OK;
            }
    }
    // not seen yet (or no context before this call: the lookup makes the
    // runtime's primary context current)
    const int rc = lookup_symbol(addr);
    if (rc != CBQ_OK) return rc;
    if (!ctx && !current(ctx)) return CBQ_OK;           // no driver entry point: not cached
    if (g_cache.used < ScratchCache::kSlots) {
        g_cache.ctx[g_cache.used] = ctx;
        g_cache.addr[g_cache.used] = *addr;
        ++g_cache.used;
    }
    return CBQ_OK;
}

}  // namespace

extern "C" int cbq_linear_fixed_noalloc(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                        const uint8_t *packed_dev, int64_t packed_bytes,
                                        const float *codebook_dev, int64_t C, int bits, int64_t M,
                                        int64_t K, const float *bias_dev, void *out_dev, int out_dtype,
                                        int64_t ldo, void *stream) {
    // the argument checks of cbq_linear_fixed
    if (T < 0 || M < 0 || K < 0 || bits < 1 || bits > 16 || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (T == 0 || M == 0) return CBQ_OK;
    if (!out_dev || !codebook_dev || (K > 0 && (!x_dev || !packed_dev))) return CBQ_ERR_ARG;
    if (ldx < K || ldo < M) return CBQ_ERR_ARG;
    if (packed_bytes < cbq_fixed_stream_bytes(M, K, bits)) return CBQ_ERR_ARG;
    void *scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != CBQ_OK) return rc;
    // The array keeps the previous call's contents: the dispatch clears the
    // bytes it uses on `stream` before the launch that uses them, and returns
    // CBQ_ERR_ARG, launching nothing, when those bytes exceed the array.
    return cbq::linear_fixed_impl(x_dev, x_dtype, T, ldx, packed_dev, codebook_dev, C, bits, M, K, bias_dev,
                                  out_dev, out_dtype, ldo, scratch, (int64_t)kNoAllocScratchBytes,
                                  static_cast<cudaStream_t>(stream), cbq::kWsClearFirst);
}
