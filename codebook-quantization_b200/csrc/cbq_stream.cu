// cbq_stream.cu -- fixed-width decode-GEMV over a stream that stays in host
// memory (models whose packed indices do not fit in device memory).
//
// The reference keeps such streams on disk as flat .idx files, memory-maps
// them and runs its CPU kernel on the mapping (MmappedPackedBuffer,
// src/compressed_matmul_cpu.py:23-63; exported by export_flat_idx,
// src/adaptive_compressor.py:1254-1316).  Here the host bytes (pinned memory,
// or a memory-mapped .idx file registered with cbq_host_register) are copied
// to the device in row chunks through two staging buffers: the copy of chunk
// i+1 runs on a copy stream of the library while chunk i's GEMV runs on the
// caller's stream, so the host link and the GEMV overlap and the device holds
// only the staging buffers.  Rows are independent, so a chunk's GEMV is the
// ordinary one over its rows, writing its slice of the output.
#include <algorithm>
#include <mutex>

#include "cbq_common.cuh"

namespace {

struct StreamState {
    bool ready = false;
    cudaStream_t copy = nullptr;
    cudaEvent_t start = nullptr, copied[2] = {nullptr, nullptr}, consumed[2] = {nullptr, nullptr};
};

std::mutex g_stream_mu;
StreamState g_state[64];

int state_for_device(StreamState *&st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return CBQ_ERR_CUDA;
    st = &g_state[dev];
    if (st->ready) return CBQ_OK;
    if (cudaStreamCreateWithFlags(&st->copy, cudaStreamNonBlocking) != cudaSuccess) return CBQ_ERR_CUDA;
    cudaEvent_t *evs[5] = {&st->start, &st->copied[0], &st->copied[1], &st->consumed[0], &st->consumed[1]};
    for (cudaEvent_t *e : evs)
        if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess) return CBQ_ERR_CUDA;
    st->ready = true;
    return CBQ_OK;
}

int64_t row_bytes_of(int64_t K, int bits) { return K * bits / 8; }

}  // namespace

extern "C" int64_t cbq_streamed_chunk_rows(int64_t M, int64_t K, int bits, int64_t staging_bytes) {
    if (M < 1 || K < 1 || K % 128 || bits < 1 || bits > 16 || staging_bytes < 0) return -1;
    const int64_t half = (staging_bytes / 2) & ~(int64_t)255;
    const int64_t rb = row_bytes_of(K, bits);
    int64_t rows = (half - 64 - 16) / rb;
    if (rows < 1) return -1;
    return std::min(rows, M);
}

extern "C" int cbq_host_register(void *host_ptr, int64_t bytes, int read_only) {
    if (!host_ptr || bytes < 1) return CBQ_ERR_ARG;
    unsigned flags = cudaHostRegisterPortable;
    if (read_only) {
        int dev = 0, ok = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) return CBQ_ERR_CUDA;
        if (cudaDeviceGetAttribute(&ok, cudaDevAttrHostRegisterReadOnlySupported, dev) != cudaSuccess || !ok)
            return CBQ_ERR_UNSUPPORTED;
        flags |= cudaHostRegisterReadOnly;
    }
    const cudaError_t e = cudaHostRegister(host_ptr, (size_t)bytes, flags);
    if (e != cudaSuccess) {
        cudaGetLastError();                                    // not sticky; leave no error behind
        return CBQ_ERR_CUDA;
    }
    return CBQ_OK;
}

extern "C" int cbq_host_unregister(void *host_ptr) {
    if (!host_ptr) return CBQ_ERR_ARG;
    if (cudaHostUnregister(host_ptr) != cudaSuccess) {
        cudaGetLastError();
        return CBQ_ERR_CUDA;
    }
    return CBQ_OK;
}

extern "C" int cbq_linear_fixed_streamed(const void *x_dev, int x_dtype, int64_t T, int64_t ldx,
                                         const uint8_t *packed_host, int64_t packed_bytes,
                                         const float *codebook_dev, int64_t C, int bits, int64_t M, int64_t K,
                                         const float *bias_dev, void *out_dev, int out_dtype, int64_t ldo,
                                         void *staging_dev, int64_t staging_bytes, void *workspace_dev,
                                         int64_t workspace_bytes, void *stream) {
    if (T < 0 || M < 0 || K < 0 || bits < 1 || bits > 16 || C < 1 || C > 65536) return CBQ_ERR_ARG;
    if ((x_dtype != CBQ_F32 && x_dtype != CBQ_BF16) || (out_dtype != CBQ_F32 && out_dtype != CBQ_BF16))
        return CBQ_ERR_ARG;
    if (T == 0 || M == 0) return CBQ_OK;
    if (!x_dev || !packed_host || !codebook_dev || !out_dev || !staging_dev || ldx < K || ldo < M)
        return CBQ_ERR_ARG;
    if (K % 128) return CBQ_ERR_UNSUPPORTED;                   // every chunk starts 16-byte aligned
    if (packed_bytes < (M * K * bits + 7) / 8) return CBQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(staging_dev) & 255) return CBQ_ERR_ARG;
    const int64_t rows = cbq_streamed_chunk_rows(M, K, bits, staging_bytes);
    if (rows < 1) return CBQ_ERR_ARG;
    const int64_t half = (staging_bytes / 2) & ~(int64_t)255;
    const int64_t rb = row_bytes_of(K, bits);
    const int ob = out_dtype == CBQ_BF16 ? 2 : 4;
    std::lock_guard<std::mutex> g(g_stream_mu);
    StreamState *st = nullptr;
    int rc = state_for_device(st);
    if (rc != CBQ_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // copies start after everything already queued on the caller's stream
    // (earlier calls' GEMVs read the same staging buffers)
    CBQ_CUDA_TRY(cudaEventRecord(st->start, s));
    CBQ_CUDA_TRY(cudaStreamWaitEvent(st->copy, st->start, 0));
    int64_t chunk = 0;
    for (int64_t r0 = 0; r0 < M; r0 += rows, ++chunk) {
        const int b = (int)(chunk & 1);
        const int64_t r1 = std::min(M, r0 + rows);
        uint8_t *buf = static_cast<uint8_t *>(staging_dev) + b * half;
        if (chunk >= 2) CBQ_CUDA_TRY(cudaStreamWaitEvent(st->copy, st->consumed[b], 0));
        CBQ_CUDA_TRY(cudaMemcpyAsync(buf, packed_host + r0 * rb, (size_t)((r1 - r0) * rb), cudaMemcpyHostToDevice,
                                     st->copy));
        CBQ_CUDA_TRY(cudaEventRecord(st->copied[b], st->copy));
        CBQ_CUDA_TRY(cudaStreamWaitEvent(s, st->copied[b], 0));
        rc = cbq::linear_fixed_impl(x_dev, x_dtype, T, ldx, buf, codebook_dev, C, bits, r1 - r0, K,
                                    bias_dev ? bias_dev + r0 : nullptr, static_cast<uint8_t *>(out_dev) + r0 * ob,
                                    out_dtype, ldo, workspace_dev, workspace_bytes, s, cbq::kWsCallerZeroed);
        if (rc != CBQ_OK) return rc;
        CBQ_CUDA_TRY(cudaEventRecord(st->consumed[b], s));
    }
    return CBQ_OK;
}
