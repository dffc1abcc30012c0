// lib.cu -- library-wide helpers of libcdlb200: status strings, version,
// per-device SM count cache.
#include <atomic>

#include "common.cuh"

namespace cdlb200 {

// Poll limit of the grid-wide barrier in the fused NVFP4 quantizer (about a
// second at the default); read by the host at each launch.
std::atomic<uint32_t> g_wait_limit{1u << 20};

uint32_t wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

// SMs the persistent kernels (the pair GEMM, the dual encoder) may fill; 0 =
// all (cdlb200_set_persistent_sm_limit).
std::atomic<int> g_persistent_sm_limit{0};

int num_sms() {
    static int cache[128] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

int persistent_sms() {
    const int n = num_sms(), lim = g_persistent_sm_limit.load(std::memory_order_relaxed);
    return lim >= 2 && lim < n ? lim : n;
}

}  // namespace cdlb200

extern "C" const char* cdlb200_status_string(int status) {
    switch (status) {
        case CDLB200_OK: return "ok";
        case CDLB200_ERR_INVALID_ARG: return "invalid argument";
        case CDLB200_ERR_ALIGNMENT: return "misaligned pointer or leading dimension";
        case CDLB200_ERR_UNSUPPORTED: return "unsupported device (needs sm_100)";
        case CDLB200_ERR_LAUNCH: return "CUDA kernel launch failed";
        case CDLB200_ERR_TIMEOUT: return "bounded device-side wait timed out";
        case CDLB200_ERR_WORKSPACE: return "workspace missing or too small";
        case CDLB200_ERR_CUDA: return "CUDA runtime error";
        default: return "unknown status";
    }
}

extern "C" int cdlb200_version(void) { return 101; }

extern "C" uint32_t cdlb200_set_wait_limit(uint32_t polls) {
    return cdlb200::g_wait_limit.exchange(polls, std::memory_order_relaxed);
}

extern "C" int cdlb200_set_persistent_sm_limit(int sms) {
    if (sms < 0) return CDLB200_ERR_INVALID_ARG;
    cdlb200::g_persistent_sm_limit.store(sms, std::memory_order_relaxed);
    return CDLB200_OK;
}
