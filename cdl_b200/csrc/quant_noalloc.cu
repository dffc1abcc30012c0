// quant_noalloc.cu -- NVFP4 quantize for callers that cannot allocate device memory.
//
// cdlb200_nvfp4_quant() needs a few KiB of device scratch for its global amax
// (per-CTA partial maxima and an arrival counter) and expects its caller to
// allocate that scratch and pass it in.  Some callers cannot: a host program
// that binds this C ABI from another language runtime and has no CUDA
// allocator of its own to call, or a serving or training runtime that reserves
// all device memory up front in its own arena and does not let an operator
// allocate on its own.  cdlb200_nvfp4_quant_noalloc() takes the same inputs and
// outputs and keeps its scratch in a fixed array that lives in the library's
// own device memory instead.
//
// That array costs kNoAllocScratchBytes (8 KiB) on every GPU that loads the
// library, for as long as the library stays loaded.  The first call on each
// device looks up the array's device address (cudaGetSymbolAddress) while
// that device is current; make that first call before any stream capture.
// The address is cached per device together with the CUDA context it was
// looked up in: a call in another context (after cudaDeviceReset, or once
// the primary context was released and created again) looks it up afresh.
// Every call on a device shares the one array: the arrival counter is cleared
// at the start of each call, and two calls that run at the same time on the
// GPU (different streams without ordering between them) race on it.
// No cudaMalloc, cudaFree or other allocating routine is called here.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace cdlb200 {
int launch_amax(const void* x, int64_t rows, int64_t k, int64_t ldx, uint32_t* partial,
                uint32_t* counter, float* gmax, float* alpha, cudaStream_t st);
int launch_nvfp4_encode(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                        void* packed, void* scale, int scale_layout, const float* gmax,
                        const float* alpha, cudaStream_t st);
}  // namespace cdlb200

namespace {

// Layout (same as the caller-provided workspace of cdlb200_nvfp4_quant):
// [0, 4) arrival counter, [256, 256 + 4*1024) partial maxima, then one float
// holding gmax when the caller passes no gmax output.
constexpr size_t kNoAllocScratchBytes = 8192;
constexpr size_t kCounterOff = 0;
constexpr size_t kPartialOff = 256;
constexpr size_t kGmaxOff = kPartialOff + 4 * 1024;

static __device__ __align__(256) unsigned char g_nvfp4_scratch[kNoAllocScratchBytes];

// cuCtxGetCurrent through the runtime's driver entry point query, so the
// library does not need libcuda at load time (it loads on hosts without a GPU)
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CUcontext current_context() {
    static CtxGetCurrentFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    }
    CUcontext ctx = nullptr;
    if (!fn || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

struct ScratchAddress {
    CUcontext ctx;  // context the address was looked up in
    void* ptr;
};
std::mutex g_scratch_mu;
ScratchAddress g_scratch[128] = {};

// Device address of g_nvfp4_scratch on the current device, looked up once per
// device and context.
int scratch_for_current_device(unsigned char** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return CDLB200_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    CUcontext ctx = current_context();
    if (ctx == nullptr || g_scratch[dev].ctx != ctx || g_scratch[dev].ptr == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_nvfp4_scratch);
        if (e != cudaSuccess || p == nullptr) {
            (void)cudaGetLastError();
            return CDLB200_ERR_CUDA;
        }
        // the lookup made the device's primary context current if none was
        if (ctx == nullptr) ctx = current_context();
        g_scratch[dev].ctx = ctx;
        g_scratch[dev].ptr = p;
    }
    *out = static_cast<unsigned char*>(g_scratch[dev].ptr);
    return CDLB200_OK;
}

}  // namespace

extern "C" int cdlb200_nvfp4_quant_noalloc(const void* x, int64_t rows, int64_t k, int64_t ldx,
                                           int transpose, void* packed, void* scale,
                                           int scale_layout, float* gmax, float* alpha,
                                           void* stream) {
    if (rows < 0 || k < 0 || (transpose != 0 && transpose != 1)) return CDLB200_ERR_INVALID_ARG;
    if (scale_layout != CDLB200_SCALE_LINEAR && scale_layout != CDLB200_SCALE_SWIZZLED)
        return CDLB200_ERR_INVALID_ARG;
    if (!alpha) return CDLB200_ERR_INVALID_ARG;
    if (rows > 0 && k > 0) {
        if (!x || !packed || !scale || ldx < k) return CDLB200_ERR_INVALID_ARG;
        if ((reinterpret_cast<uintptr_t>(x) & 1u) != 0) return CDLB200_ERR_ALIGNMENT;
    }
    // The scratch this call needs must fit in the fixed array.
    if (cdlb200_nvfp4_quant_workspace_bytes(rows, k) > kNoAllocScratchBytes) return CDLB200_ERR_WORKSPACE;
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return CDLB200_ERR_CUDA;
    if (major != 10) return CDLB200_ERR_UNSUPPORTED;

    unsigned char* ws = nullptr;
    int rc = scratch_for_current_device(&ws);
    if (rc != CDLB200_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t* counter = reinterpret_cast<uint32_t*>(ws + kCounterOff);
    uint32_t* partial = reinterpret_cast<uint32_t*>(ws + kPartialOff);
    float* g = gmax ? gmax : reinterpret_cast<float*>(ws + kGmaxOff);
    // The arrival counter must start at zero; the array keeps the last call's contents.
    if (cudaMemsetAsync(counter, 0, sizeof(uint32_t), st) != cudaSuccess) return CDLB200_ERR_CUDA;
    rc = cdlb200::launch_amax(x, rows, k, ldx, partial, counter, g, alpha, st);
    if (rc != CDLB200_OK || rows == 0 || k == 0) return rc;
    return cdlb200::launch_nvfp4_encode(x, rows, k, ldx, transpose, packed, scale, scale_layout, g,
                                        alpha, st);
}
