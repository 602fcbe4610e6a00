// cbq_common.cuh -- device helpers shared by the codebook decode-matmul kernels
// (sm_100a): mbarrier + 1-D bulk-copy (TMA) staging, bounded waits, dtype I/O.
#pragma once
#include <cuda_runtime.h>
#include <utility>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/cbq.h"

namespace cbq {

constexpr int kThreads = 256;            // threads per CTA of the GEMV kernels
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s bound on any device-side wait

__host__ __device__ constexpr size_t a128(size_t v) { return (v + 127) & ~(size_t)127; }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Plain arrive (release semantics at CTA scope) by the calling thread.
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` while the phase is
// incomplete (the hardware wakes it when the phase completes), so a waiting
// warp does not spin through the issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, giving up after kWaitNs.
// Returns false on timeout (the caller records CBQ_FLAG_TIMEOUT and stops).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
        if (global_timer_ns() - t0 > kWaitNs) return false;
    }
}

// Order this thread's earlier shared-memory accesses (generic proxy) before
// its later bulk copies into the same bytes (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// Record a decode error in the caller's status word (may be null).
__device__ __forceinline__ void report(uint32_t *status, uint32_t flag, uint32_t row) {
    if (!status) return;
    atomicOr(status + CBQ_STATUS_FLAGS, flag);
    atomicMin(status + CBQ_STATUS_FIRST_ROW, row);
    atomicAdd(status + CBQ_STATUS_COUNT, 1u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Programmatic dependent launch.  A kernel launched with
// cbq_host::launch_pdl may start while the previous kernel on its stream is
// still running: it lets its own successor launch as soon as all of its CTAs
// are running (pdl_launch_dependents, so no launch ever waits for CTAs that
// cannot be scheduled), does the work that reads nothing the predecessor
// writes (weight prefetch, tables), then waits for the predecessor to finish
// and its writes to be visible (pdl_wait) before touching activations.
// Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace cbq

namespace cbq {
// How linear_fixed_impl (cbq_fixed.cu) treats the workspace it is given.
enum WsMode : int {
    kWsCallerZeroed = 0,   // kept zeroed by the kernels between calls (cbq_linear_fixed)
    kWsClearFirst = 1,     // shared scratch: cleared before use, too small -> CBQ_ERR_ARG
};
int linear_fixed_impl(const void *x, int x_dtype, int64_t T, int64_t ldx, const uint8_t *packed,
                      const float *cb, int64_t C, int bits, int64_t M, int64_t K, const float *bias,
                      void *out, int out_dtype, int64_t ldo, void *ws, int64_t ws_bytes,
                      cudaStream_t s, int ws_mode);
}  // namespace cbq

// Host-side helpers shared by the .cu files.
namespace cbq_host {
int sm_count();           // SMs of the current device (cached per device)
int max_smem_optin();     // opt-in dynamic shared memory per block
inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }
bool pdl_enabled();       // programmatic dependent launch (CBQ_PDL=0 in the environment turns it off)
bool attn_cluster_enabled();   // split attention as clusters (CBQ_ATTN_CLUSTER=0 turns it off)

// Launch `kern` on `s` with the programmatic-stream-serialization attribute
// (see pdl_wait above); plain stream order when PDL is off.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// launch_pdl with the grid tiled into thread-block clusters of `cluster`
// consecutive CTAs (x dimension).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, unsigned cluster,
                               cudaStream_t s, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
}  // namespace cbq_host

#define CBQ_CUDA_TRY(expr)                                   \
    do {                                                     \
        cudaError_t e_ = (expr);                             \
        if (e_ != cudaSuccess) return CBQ_ERR_CUDA;          \
    } while (0)
