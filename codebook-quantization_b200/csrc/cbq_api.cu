// cbq_api.cu -- library-wide C ABI entry points and host helpers.
#include <cstdlib>
#include <mutex>

#include "cbq_common.cuh"

namespace cbq_host {

namespace {
struct DevInfo {
    int sms = 0;
    int smem_optin = 0;
};
std::mutex g_mu;
DevInfo g_info[64];

const DevInfo &info() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    std::lock_guard<std::mutex> g(g_mu);
    DevInfo &d = g_info[dev & 63];
    if (d.sms == 0) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            d.sms = 148;
        if (cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) !=
            cudaSuccess)
            d.smem_optin = 227 * 1024;
    }
    return d;
}
}  // namespace

int sm_count() { return info().sms; }
int max_smem_optin() { return info().smem_optin; }

bool pdl_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("CBQ_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

bool attn_cluster_enabled() {
    static const bool on = [] {
        const char *v = std::getenv("CBQ_ATTN_CLUSTER");
        return !(v && v[0] == '0');
    }();
    return on;
}

}  // namespace cbq_host

extern "C" const char *cbq_status_string(int status) {
    switch (status) {
        case CBQ_OK: return "ok";
        case CBQ_ERR_CUDA: return "CUDA runtime error";
        case CBQ_ERR_ARG: return "invalid argument";
        case CBQ_ERR_CORRUPT: return "corrupt stream";
        case CBQ_ERR_TIMEOUT: return "device wait timed out";
        case CBQ_ERR_UNSUPPORTED: return "unsupported shape or format";
    }
    return "unknown status";
}

extern "C" int cbq_version(void) { return 1; }
