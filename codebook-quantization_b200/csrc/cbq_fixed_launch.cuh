// cbq_fixed_launch.cuh -- per-width launchers of k_linear_fixed and
// k_gemv_fixed, explicitly instantiated in cbq_fixed_w*.cu (split so the
// variants compile in parallel).
#pragma once
#include <mutex>

#include "cbq_fixed_kernel.cuh"
#include "cbq_gemv_kernel.cuh"

namespace cbq {

template <int BITS, int TB, typename XT>
int launch_fixed_one(const FixedArgs &a, size_t smem, int grid, cudaStream_t s) {
    auto kern = k_linear_fixed<BITS, TB, XT>;
    static std::mutex mu;
    static size_t configured[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CBQ_ERR_CUDA;
    {
        std::lock_guard<std::mutex> g(mu);
        if (configured[dev & 63] < smem) {
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess)
                return CBQ_ERR_CUDA;
            configured[dev & 63] = smem;
        }
    }
    kern<<<grid, kFxWarps * 32, smem, s>>>(a);
    return cudaGetLastError() == cudaSuccess ? CBQ_OK : CBQ_ERR_CUDA;
}

template <int BITS>
int launch_fixed_bits(int TB, bool x_bf16, const FixedArgs &a, size_t smem, int grid, cudaStream_t s) {
    if (x_bf16) {
        switch (TB) {
            case 1: return launch_fixed_one<BITS, 1, __nv_bfloat16>(a, smem, grid, s);
            case 2: return launch_fixed_one<BITS, 2, __nv_bfloat16>(a, smem, grid, s);
            case 4: return launch_fixed_one<BITS, 4, __nv_bfloat16>(a, smem, grid, s);
            case 8: return launch_fixed_one<BITS, 8, __nv_bfloat16>(a, smem, grid, s);
        }
    } else {
        switch (TB) {
            case 1: return launch_fixed_one<BITS, 1, float>(a, smem, grid, s);
            case 2: return launch_fixed_one<BITS, 2, float>(a, smem, grid, s);
            case 4: return launch_fixed_one<BITS, 4, float>(a, smem, grid, s);
            case 8: return launch_fixed_one<BITS, 8, float>(a, smem, grid, s);
        }
    }
    return CBQ_ERR_UNSUPPORTED;
}

// Raise a kernel's dynamic shared-memory limit once per device.
template <typename Kern>
int ensure_smem(Kern kern, size_t smem, std::mutex &mu, size_t (&configured)[64]) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CBQ_ERR_CUDA;
    std::lock_guard<std::mutex> g(mu);
    if (configured[dev & 63] < smem) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return CBQ_ERR_CUDA;
        configured[dev & 63] = smem;
    }
    return CBQ_OK;
}

template <int BITS, int TB, int NF, typename XT>
int launch_gemv_one(const GemvArgs &a, size_t smem, int grid, cudaStream_t s) {
    auto kern = k_gemv_fixed<BITS, TB, NF, XT>;
    static std::mutex mu;
    static size_t configured[64] = {0};
    const int rc = ensure_smem(kern, smem, mu, configured);
    if (rc != CBQ_OK) return rc;
    return cbq_host::launch_pdl(kern, dim3(grid), dim3(kGvWarps * 32), smem, s, a) == cudaSuccess
               ? CBQ_OK
               : CBQ_ERR_CUDA;
}

// Token counts 1 and 2 with units of 32 indices per lane, and one token with
// units of 64.
template <int BITS>
int launch_gemv_bits(int TB, int NF, bool x_bf16, const GemvArgs &a, size_t smem, int grid, cudaStream_t s) {
    if (x_bf16) {
        if (TB == 1 && NF == 64) return launch_gemv_one<BITS, 1, 64, __nv_bfloat16>(a, smem, grid, s);
        if (TB == 1 && NF == 32) return launch_gemv_one<BITS, 1, 32, __nv_bfloat16>(a, smem, grid, s);
        if (TB == 2 && NF == 32) return launch_gemv_one<BITS, 2, 32, __nv_bfloat16>(a, smem, grid, s);
    } else {
        if (TB == 1 && NF == 64) return launch_gemv_one<BITS, 1, 64, float>(a, smem, grid, s);
        if (TB == 1 && NF == 32) return launch_gemv_one<BITS, 1, 32, float>(a, smem, grid, s);
        if (TB == 2 && NF == 32) return launch_gemv_one<BITS, 2, 32, float>(a, smem, grid, s);
    }
    return CBQ_ERR_UNSUPPORTED;
}

#define CBQ_INSTANTIATE_FIXED(B)                                                              \
    template int launch_fixed_bits<B>(int, bool, const FixedArgs &, size_t, int, cudaStream_t); \
    template int launch_gemv_bits<B>(int, int, bool, const GemvArgs &, size_t, int, cudaStream_t);

}  // namespace cbq
