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
// cudaFree.
#include <mutex>

#include "cbq_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = CBQ_NOALLOC_SCRATCH_BYTES;

// The workspace shared by every call on a device.  In host code this name is
// only a stand-in for the symbol: its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void *g_scratch_addr[64] = {nullptr};

// Device address of the scratch array on the current device, looked up once
// per device (the first call on a device does this; make that first call
// before any stream capture).
int scratch_address(void **addr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CBQ_ERR_CUDA;
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return CBQ_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *addr = g_scratch_addr[dev];
    return CBQ_OK;
}

}  // namespace

extern "C" int cbq_linear_fixed_noalloc(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                        const uint8_t *packed_dev, int64_t packed_bytes,
                                        const float *codebook_dev, int64_t C, int bits, int64_t M,
                                        int64_t K, const float *bias_dev, void *out_dev, int out_dtype,
                                        int64_t ldo, void *stream) {
    const int64_t need = cbq_linear_fixed_workspace_bytes(M, K, T);
    if (need < 0) return CBQ_ERR_ARG;
    if ((size_t)need > kNoAllocScratchBytes) return CBQ_ERR_ARG;   // matrix too large for the built-in scratch
    if (T == 0 || M == 0) return CBQ_OK;
    void *scratch = nullptr;
    const int rc = scratch_address(&scratch);
    if (rc != CBQ_OK) return rc;
    // The array keeps the previous call's contents; the row counters in it
    // must start at zero, so the part this call uses is cleared first.
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(scratch, 0, (size_t)need, s) != cudaSuccess) return CBQ_ERR_CUDA;
    return cbq_linear_fixed(x_dev, x_dtype, T, ldx, packed_dev, packed_bytes, codebook_dev, C, bits, M, K,
                            bias_dev, out_dev, out_dtype, ldo, scratch, need, stream);
}
