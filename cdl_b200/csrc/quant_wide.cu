// quant_wide.cu -- block-scaled quantize of fp32 and fp16 input (sm_100a).
//
// cdl's `_quant` (cdl/core/kernel/quant.py:71-123) takes any floating tensor:
// its Triton kernel loads each block and casts it to fp32 (quant.py:36-38), and
// the NVFP4 global amax is `x.abs().amax().float()` (quant.py:96-101).  The
// bf16 kernels of quant.cu replace the per-element divide by a multiply that
// is only exact for bf16's 8 significant bits, so wider inputs take this path,
// which performs cdl's fp32 operations literally:
//   NVFP4  alpha = RN(gmax * RN(1 / 2688)) (nvfp4_alpha), q = RN(RN(bamax * 448) / gmax),
//          byte = e4m3_rne(clamp(q, 2^-9, 448)), s = RN(e4m3(byte) * alpha)
//   MX     byte = clamp(floor(log2(max(bamax, FLT_MIN))) - emax + 127, 0, 254),
//          s = 2^(byte - 127) (byte 0: the subnormal 2^-127); an infinite
//          block amax gives byte 254, as cdl's torch path (core/ecdl.py:59-73)
//          and the bf16 kernels do
//   v = RN(x / s); e2m1 magnitude = the number of midpoints
//   {.25, .75, 1.25, 1.75, 2.5, 3.5, 5} that min(|v|, 6) exceeds, sign = the
//   sign bit of v (formats/ordinals.py:7-20); e4m3 = RNE with saturation of
//   clamp(v, -448, 448) (quant.py:66-68).
// One thread per (row, block); elements are read through a row and a column
// stride, so the transposed quantize and the 128x4 scale layout come for free.
// This path is not tuned: the QAT step's tensors are bf16.
#include <cuda_fp16.h>
#include <float.h>

#include "common.cuh"

namespace cdlb200 {

namespace {

// Word of the caller's NVFP4 workspace that holds the global amax of this path
// (fp32 magnitude bits).  The workspace layout of quant.cu uses bytes 0..15
// and 256.. ; byte 16 is this path's.
constexpr int kWsWideAmaxOff = 16;

__device__ __forceinline__ float load_f32(const float* p) { return *p; }
__device__ __forceinline__ float load_f32(const __half* p) { return __half2float(*p); }

template <typename T>
__global__ void __launch_bounds__(256) wide_amax_kernel(const T* __restrict__ x, int64_t rows, int64_t k,
                                                        int64_t ldx, uint32_t* __restrict__ word) {
    uint32_t m = 0;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
        for (int64_t c = threadIdx.x; c < k; c += blockDim.x)
            m = max(m, f2u(load_f32(x + r * ldx + c)) & 0x7fffffffu);  // NaN bits order above inf
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0 && m != 0) atomicMax(word, m);
}

__device__ __forceinline__ uint32_t e2m1_code(float v) {
    const float av = fminf(fabsf(v), 6.0f);
    const uint32_t mag = (av > 0.25f) + (av > 0.75f) + (av > 1.25f) + (av > 1.75f) + (av > 2.5f) + (av > 3.5f) +
                         (av > 5.0f);
    return mag | ((f2u(v) >> 31) << 3);
}

template <int EMAX>
__device__ __forceinline__ uint32_t e8m0_byte_from_f32(float bamax) {
    if (bamax != bamax) return 0u;
    if (bamax == INFINITY) return 254u;
    const int e = (int)(f2u(fmaxf(bamax, FLT_MIN)) >> 23) - 127;
    const int b = e - EMAX + 127;
    return (uint32_t)(b < 0 ? 0 : (b > 254 ? 254 : b));
}

// ROWWISE: consecutive threads take consecutive blocks of a row (the column
// stride is 1); otherwise consecutive rows (the row stride is 1: transposed).
template <typename T, int FMT, bool SWZ, bool ROWWISE>
__global__ void __launch_bounds__(256) wide_quant_kernel(const T* __restrict__ x, int64_t R, int64_t C, int64_t sr,
                                                         int64_t sc, uint8_t* __restrict__ packed, int64_t pstride,
                                                         uint8_t* __restrict__ scale, int64_t nb, int64_t c4,
                                                         const uint32_t* __restrict__ amax_word,
                                                         float* __restrict__ alpha_out) {
    constexpr int B = FmtTraits<FMT>::kBlock;
    float gmax = 0.f, alpha = 0.f;
    if constexpr (FMT == kNVFP4) {
        const float g = u2f(*amax_word);
        gmax = g < FLT_MIN ? FLT_MIN : g;  // clamp_min(tiny); a NaN stays NaN
        alpha = nvfp4_alpha(gmax);
        if (blockIdx.x == 0 && threadIdx.x == 0) *alpha_out = alpha;
    }
    const int64_t total = R * nb;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = ROWWISE ? idx / nb : idx % R;
        const int64_t b = ROWWISE ? idx - r * nb : idx / R;
        float v[B];
        float bamax = 0.f;
#pragma unroll
        for (int i = 0; i < B; ++i) {
            const int64_t c = b * B + i;
            v[i] = c < C ? load_f32(x + r * sr + c * sc) : 0.f;
            bamax = fmaxf(bamax, fabsf(v[i]));
        }
        uint32_t byte;
        float s;
        if constexpr (FMT == kNVFP4) {
            byte = ue4m3_scale_byte(__fdiv_rn(__fmul_rn(bamax, 448.0f), gmax));
            s = __fmul_rn(e4m3_to_f32(byte), alpha);
        } else {
            byte = e8m0_byte_from_f32<FmtTraits<FMT>::kEmax>(bamax);
            s = e8m0_to_f32(byte);
        }
        uint8_t* prow = packed + r * pstride;
        if constexpr (FmtTraits<FMT>::kFp4) {
#pragma unroll
            for (int i = 0; i < B; i += 2)
                prow[(b * B + i) / 2] =
                    (uint8_t)(e2m1_code(__fdiv_rn(v[i], s)) | (e2m1_code(__fdiv_rn(v[i + 1], s)) << 4));
        } else {
#pragma unroll
            for (int i = 0; i < B; i += 2) {
                const float lo = fminf(fmaxf(__fdiv_rn(v[i], s), -448.0f), 448.0f);
                const float hi = fminf(fmaxf(__fdiv_rn(v[i + 1], s), -448.0f), 448.0f);
                const uint32_t p = cvt_e4m3x2(hi, lo);
                prow[b * B + i] = (uint8_t)(p & 0xffu);
                prow[b * B + i + 1] = (uint8_t)(p >> 8);
            }
        }
        scale[SWZ ? swizzle_offset(r, b, c4) : r * nb + b] = (uint8_t)byte;
    }
}

template <typename T, int FMT, bool SWZ>
int launch_wide(const T* x, int64_t rows, int64_t k, int64_t ldx, int transpose, void* packed, void* scale,
                const uint32_t* word, float* alpha, cudaStream_t st) {
    constexpr int B = FmtTraits<FMT>::kBlock;
    const int64_t R = transpose ? k : rows, C = transpose ? rows : k;
    const int64_t nb = (C + B - 1) / B;
    const int64_t c4 = (nb + 3) / 4;
    const int64_t pstride = FmtTraits<FMT>::kFp4 ? nb * B / 2 : nb * B;
    const int64_t sr = transpose ? 1 : ldx, sc = transpose ? ldx : 1;
    int64_t grid = (R * nb + 255) / 256;
    const int64_t cap = (int64_t)num_sms() * 16;
    grid = grid < 1 ? 1 : (grid < cap ? grid : cap);
    if (transpose)
        wide_quant_kernel<T, FMT, SWZ, false><<<(unsigned)grid, 256, 0, st>>>(
            x, R, C, sr, sc, static_cast<uint8_t*>(packed), pstride, static_cast<uint8_t*>(scale), nb, c4, word, alpha);
    else
        wide_quant_kernel<T, FMT, SWZ, true><<<(unsigned)grid, 256, 0, st>>>(
            x, R, C, sr, sc, static_cast<uint8_t*>(packed), pstride, static_cast<uint8_t*>(scale), nb, c4, word, alpha);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

template <typename T, int FMT>
int wide_entry(const void* xv, int64_t rows, int64_t k, int64_t ldx, int transpose, void* packed, void* scale,
               int scale_layout, float* alpha, uint8_t* ws, cudaStream_t st) {
    const T* x = static_cast<const T*>(xv);
    uint32_t* word = nullptr;
    if constexpr (FMT == kNVFP4) {
        word = reinterpret_cast<uint32_t*>(ws + kWsWideAmaxOff);
        if (cudaMemsetAsync(word, 0, sizeof(uint32_t), st) != cudaSuccess) return CDLB200_ERR_CUDA;
        if (rows > 0 && k > 0) {
            const int64_t grid = rows < (int64_t)num_sms() * 8 ? rows : (int64_t)num_sms() * 8;
            wide_amax_kernel<T><<<(unsigned)grid, 256, 0, st>>>(x, rows, k, ldx, word);
            CDLB200_CHECK_LAUNCH();
        }
    }
    if (rows == 0 || k == 0) {
        if constexpr (FMT == kNVFP4)  // alpha of an empty tensor: FLT_MIN / 2688, as cdl's
            return launch_wide<T, FMT, false>(x, 0, 0, ldx, 0, packed, scale, word, alpha, st);
        return CDLB200_OK;
    }
    if (scale_layout == CDLB200_SCALE_SWIZZLED) {
        constexpr int B = FmtTraits<FMT>::kBlock;
        const int64_t R = transpose ? k : rows, C = transpose ? rows : k;
        const int64_t nb = (C + B - 1) / B;
        if ((R % 128) != 0 || (nb % 4) != 0) {
            const size_t bytes = (size_t)((R + 127) / 128 * 128) * (size_t)((nb + 3) / 4 * 4);
            if (cudaMemsetAsync(scale, 0, bytes, st) != cudaSuccess) return CDLB200_ERR_CUDA;
        }
        return launch_wide<T, FMT, true>(x, rows, k, ldx, transpose, packed, scale, word, alpha, st);
    }
    return launch_wide<T, FMT, false>(x, rows, k, ldx, transpose, packed, scale, word, alpha, st);
}

template <typename T>
int wide_dispatch(int format, const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose, void* packed,
                  void* scale, int scale_layout, float* alpha, uint8_t* ws, cudaStream_t st) {
    switch (format) {
        case kNVFP4:
            return wide_entry<T, kNVFP4>(x, rows, k, ldx, transpose, packed, scale, scale_layout, alpha, ws, st);
        case kMXFP4:
            return wide_entry<T, kMXFP4>(x, rows, k, ldx, transpose, packed, scale, scale_layout, alpha, ws, st);
        default:
            return wide_entry<T, kMXFP8>(x, rows, k, ldx, transpose, packed, scale, scale_layout, alpha, ws, st);
    }
}

}  // namespace

}  // namespace cdlb200

using namespace cdlb200;

extern "C" int cdlb200_quant_wide(const void* x, int dtype, int format, int64_t rows, int64_t k, int64_t ldx,
                                  int transpose, void* packed, void* scale, int scale_layout, float* alpha,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (dtype != CDLB200_DTYPE_F32 && dtype != CDLB200_DTYPE_F16) return CDLB200_ERR_INVALID_ARG;
    if (format != kNVFP4 && format != kMXFP4 && format != kMXFP8) return CDLB200_ERR_INVALID_ARG;
    if (rows < 0 || k < 0 || (transpose != 0 && transpose != 1)) return CDLB200_ERR_INVALID_ARG;
    if (scale_layout != CDLB200_SCALE_LINEAR && scale_layout != CDLB200_SCALE_SWIZZLED)
        return CDLB200_ERR_INVALID_ARG;
    const int esize = dtype == CDLB200_DTYPE_F32 ? 4 : 2;
    if (rows > 0 && k > 0) {
        if (!x || !packed || !scale || ldx < k) return CDLB200_ERR_INVALID_ARG;
        if ((reinterpret_cast<uintptr_t>(x) & (uintptr_t)(esize - 1)) != 0) return CDLB200_ERR_ALIGNMENT;
    }
    if (format == kNVFP4) {
        if (!alpha) return CDLB200_ERR_INVALID_ARG;
        if (!workspace || workspace_bytes < cdlb200_nvfp4_quant_workspace_bytes(rows, k))
            return CDLB200_ERR_WORKSPACE;
    }
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return CDLB200_ERR_CUDA;
    if (major != 10) return CDLB200_ERR_UNSUPPORTED;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (dtype == CDLB200_DTYPE_F32)
        return wide_dispatch<float>(format, x, rows, k, ldx, transpose, packed, scale, scale_layout, alpha, ws, st);
    return wide_dispatch<__half>(format, x, rows, k, ldx, transpose, packed, scale, scale_layout, alpha, ws, st);
}
