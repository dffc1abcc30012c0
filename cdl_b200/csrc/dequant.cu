// dequant.cu -- FP4 / MXFP8 dequantize and the 128x4 scale swizzle (sm_100a).
//
// Replaces cdl's Triton `_fp4_dequant_kernel` / `_mxfp8_dequant_kernel`
// (cdl/core/kernel/dequant.py:25-143) and the torch `swizzle_scale_factors`
// (cdl/core/mm/swizzle.py:5-14).  Dequantize computes
//     out = bf16((value * scale) * alpha)
// in fp32 with round-to-nearest-even, in the reference's operation order.
//
// Fast path: rows are contiguous and k % block == 0, so codes, scales and
// outputs are flat arrays; one thread turns 16 elements (8 packed bytes or
// 16 e4m3 bytes, one scale byte) into 32 bytes of bf16 with vector stores.
#include <cuda_bf16.h>

#include "common.cuh"

namespace cdlb200 {

namespace {

__device__ __forceinline__ float e2m1_value(uint32_t nib) {
    // magnitudes {0, .5, 1, 1.5, 2, 3, 4, 6}: m < 4 -> m/2, else 2^(m/2-1) * (1 + (m&1)/2)
    const uint32_t m = nib & 7u;
    float mag = m < 4u ? 0.5f * (float)m : (float)(1u << ((m >> 1) - 1)) * ((m & 1u) ? 1.5f : 1.0f);
    return (nib & 8u) ? -mag : mag;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int BLOCK, bool E8M0>
__global__ void __launch_bounds__(256) fp4_dequant_flat_kernel(const uint2* __restrict__ packed,
                                                               const uint8_t* __restrict__ scale,
                                                               const float* __restrict__ alpha_p,
                                                               int64_t n16, uint4* __restrict__ out) {
    const float alpha = *alpha_p;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n16;
         t += (int64_t)gridDim.x * blockDim.x) {
        const uint2 p = packed[t];
        const uint32_t sb = scale[(t * 16) / BLOCK];
        const float sc = E8M0 ? e8m0_to_f32(sb) : e4m3_to_f32(sb);
        const uint32_t words[2] = {p.x, p.y};
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t byte = (words[i >> 2] >> (8 * (i & 3))) & 0xffu;
            const float lo = __fmul_rn(__fmul_rn(e2m1_value(byte & 15u), sc), alpha);
            const float hi = __fmul_rn(__fmul_rn(e2m1_value(byte >> 4), sc), alpha);
            o[i] = pack_bf16x2(lo, hi);
        }
        out[2 * t] = make_uint4(o[0], o[1], o[2], o[3]);
        out[2 * t + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

template <int BLOCK, bool E8M0>
__global__ void fp4_dequant_generic_kernel(const uint8_t* __restrict__ packed,
                                           const uint8_t* __restrict__ scale,
                                           const float* __restrict__ alpha_p, int64_t rows,
                                           int64_t k, uint16_t* __restrict__ out) {
    const float alpha = *alpha_p;
    const int64_t n = rows * k;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / k, c = e % k;
        const uint32_t byte = packed[r * (k / 2) + c / 2];
        const uint32_t sb = scale[r * (k / BLOCK) + c / BLOCK];
        const float sc = E8M0 ? e8m0_to_f32(sb) : e4m3_to_f32(sb);
        const float v = __fmul_rn(__fmul_rn(e2m1_value((c & 1) ? byte >> 4 : byte & 15u), sc), alpha);
        out[e] = (uint16_t)(pack_bf16x2(v, 0.0f) & 0xffffu);
    }
}

// FP4 dequantize, 32 elements (16 code bytes) per thread and step with two
// steps in flight; scales read from the linear [rows, k/BLOCK] layout or, with
// SWZ, from the 128x4 tiled layout the GEMM consumes (block b of the flat
// array sits at row b / nb, column b % nb).
template <int BLOCK, bool E8M0, bool SWZ>
__global__ void __launch_bounds__(256) fp4_dequant32_kernel(const uint4* __restrict__ packed,
                                                            const uint8_t* __restrict__ scale,
                                                            const float* __restrict__ alpha_p, int64_t n32,
                                                            FastDiv nb, uint32_t c4, uint4* __restrict__ out) {
    constexpr int kU = 2, kSb = 32 / BLOCK;
    const float alpha = *alpha_p;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t0 < n32; t0 += kU * stride) {
        uint4 p[kU];
        uint32_t sb[kU][kSb];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int64_t t = t0 + u * stride;
            if (t < n32) {
                p[u] = ldg_stream(packed + t);
#pragma unroll
                for (int j = 0; j < kSb; ++j) {
                    const int64_t b = t * kSb + j;
                    int64_t off = b;
                    if (SWZ) {
                        const uint32_t r = nb.div((uint32_t)b);
                        off = swizzle_offset(r, (int64_t)((uint32_t)b - r * nb.d), c4);
                    }
                    sb[u][j] = __ldg(scale + off);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int64_t t = t0 + u * stride;
            if (t >= n32) continue;
            const uint32_t words[4] = {p[u].x, p[u].y, p[u].z, p[u].w};
            uint32_t o[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t b = sb[u][(i * 8) / BLOCK];
                const float sc = E8M0 ? e8m0_to_f32(b) : e4m3_to_f32(b);
                uint32_t h[4];
                e2m1x8_to_f16x2(words[i], h);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float lo, hi;
                    f16x2_to_f32(h[j], lo, hi);
                    o[4 * i + j] = pack_bf16x2(__fmul_rn(__fmul_rn(lo, sc), alpha), __fmul_rn(__fmul_rn(hi, sc), alpha));
                }
            }
            uint4* dst = out + 4 * t;
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            dst[2] = make_uint4(o[8], o[9], o[10], o[11]);
            dst[3] = make_uint4(o[12], o[13], o[14], o[15]);
        }
    }
}

template <bool HAS_ALPHA>
__global__ void __launch_bounds__(256) mxfp8_dequant_flat_kernel(const uint4* __restrict__ packed,
                                                                 const uint8_t* __restrict__ scale,
                                                                 const float* __restrict__ alpha_p,
                                                                 int64_t n16, uint4* __restrict__ out) {
    const float alpha = HAS_ALPHA ? *alpha_p : 1.0f;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n16;
         t += (int64_t)gridDim.x * blockDim.x) {
        const uint4 p = packed[t];
        const float sc = e8m0_to_f32(scale[(t * 16) / 32]);
        const uint32_t words[4] = {p.x, p.y, p.z, p.w};
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t w = words[i >> 1] >> (16 * (i & 1));
            float lo = __fmul_rn(e4m3_to_f32(w & 0xffu), sc);
            float hi = __fmul_rn(e4m3_to_f32((w >> 8) & 0xffu), sc);
            if (HAS_ALPHA) {
                lo = __fmul_rn(lo, alpha);
                hi = __fmul_rn(hi, alpha);
            }
            o[i] = pack_bf16x2(lo, hi);
        }
        out[2 * t] = make_uint4(o[0], o[1], o[2], o[3]);
        out[2 * t + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

template <bool HAS_ALPHA>
__global__ void mxfp8_dequant_generic_kernel(const uint8_t* __restrict__ packed,
                                             const uint8_t* __restrict__ scale,
                                             const float* __restrict__ alpha_p, int64_t rows,
                                             int64_t k, uint16_t* __restrict__ out) {
    const float alpha = HAS_ALPHA ? *alpha_p : 1.0f;
    const int64_t n = rows * k;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / k, c = e % k;
        float v = __fmul_rn(e4m3_to_f32(packed[e]), e8m0_to_f32(scale[r * (k / 32) + c / 32]));
        if (HAS_ALPHA) v = __fmul_rn(v, alpha);
        out[e] = (uint16_t)(pack_bf16x2(v, 0.0f) & 0xffffu);
    }
}

__global__ void swizzle_kernel(const uint8_t* __restrict__ sf, int64_t m, int64_t b, int64_t c4,
                               int64_t total, uint8_t* __restrict__ out) {
    for (int64_t off = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; off < total;
         off += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tile = off >> 9, within = off & 511;
        const int64_t r = (tile / c4) * 128 + ((within >> 2) & 3) * 32 + (within >> 4);
        const int64_t c = (tile % c4) * 4 + (within & 3);
        out[off] = (r < m && c < b) ? sf[r * b + c] : (uint8_t)0;
    }
}

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(a - 1)) == 0; }

unsigned grid_for(int64_t work, int per_cta) {
    int64_t g = (work + per_cta - 1) / per_cta;
    int64_t cap = (int64_t)num_sms() * 16;
    return (unsigned)(g < 1 ? 1 : (g < cap ? g : cap));
}

}  // namespace
}  // namespace cdlb200

using namespace cdlb200;

namespace {

int fp4_dequant_impl(const void* packed, const void* scale, const float* alpha, int64_t rows, int64_t k, int block,
                     int scale_is_e8m0, bool swizzled, void* out, cudaStream_t st) {
    if (rows < 0 || k < 0 || (block != 16 && block != 32)) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || k == 0) return CDLB200_OK;
    if (!packed || !scale || !alpha || !out || (k % block) != 0) return CDLB200_ERR_INVALID_ARG;
    const int64_t n = rows * k;
    const int64_t nblocks = n / block;
    const bool vec = aligned(packed, 16) && aligned(out, 16) && (n % 32) == 0 && nblocks < (1ll << 31);
    if (swizzled && (!vec || (k % 32) != 0)) return CDLB200_ERR_ALIGNMENT;
    if (vec) {
        const int64_t n32 = n / 32;
        const FastDiv nb((uint32_t)(k / block));
        const uint32_t c4 = (uint32_t)((k / block + 3) / 4);
        const unsigned grid = grid_for(n32, 512);
#define CDLB200_FP4_DQ32(BLK, E8)                                                                            \
    if (swizzled)                                                                                            \
        fp4_dequant32_kernel<BLK, E8, true><<<grid, 256, 0, st>>>(                                           \
            static_cast<const uint4*>(packed), static_cast<const uint8_t*>(scale), alpha, n32, nb, c4,       \
            static_cast<uint4*>(out));                                                                       \
    else                                                                                                     \
        fp4_dequant32_kernel<BLK, E8, false><<<grid, 256, 0, st>>>(                                          \
            static_cast<const uint4*>(packed), static_cast<const uint8_t*>(scale), alpha, n32, nb, c4,       \
            static_cast<uint4*>(out));
        if (block == 16 && !scale_is_e8m0) {
            CDLB200_FP4_DQ32(16, false)
        } else if (block == 16) {
            CDLB200_FP4_DQ32(16, true)
        } else if (!scale_is_e8m0) {
            CDLB200_FP4_DQ32(32, false)
        } else {
            CDLB200_FP4_DQ32(32, true)
        }
#undef CDLB200_FP4_DQ32
        CDLB200_CHECK_LAUNCH();
        return CDLB200_OK;
    }
    const bool flat = aligned(packed, 8) && aligned(out, 16);
#define CDLB200_FP4_DQ(BLK, E8)                                                                   \
    if (flat)                                                                                     \
        fp4_dequant_flat_kernel<BLK, E8><<<grid_for(n / 16, 256), 256, 0, st>>>(                 \
            static_cast<const uint2*>(packed), static_cast<const uint8_t*>(scale), alpha, n / 16, \
            static_cast<uint4*>(out));                                                            \
    else                                                                                          \
        fp4_dequant_generic_kernel<BLK, E8><<<grid_for(n, 256), 256, 0, st>>>(                   \
            static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scale), alpha, rows, \
            k, static_cast<uint16_t*>(out));
    if (block == 16 && !scale_is_e8m0) {
        CDLB200_FP4_DQ(16, false)
    } else if (block == 16) {
        CDLB200_FP4_DQ(16, true)
    } else if (!scale_is_e8m0) {
        CDLB200_FP4_DQ(32, false)
    } else {
        CDLB200_FP4_DQ(32, true)
    }
#undef CDLB200_FP4_DQ
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

}  // namespace

extern "C" int cdlb200_fp4_dequant(const void* packed, const void* scale, const float* alpha,
                                   int64_t rows, int64_t k, int block, int scale_is_e8m0, void* out,
                                   void* stream) {
    return fp4_dequant_impl(packed, scale, alpha, rows, k, block, scale_is_e8m0, false, out,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int cdlb200_fp4_dequant_swizzled(const void* packed, const void* scale, const float* alpha,
                                            int64_t rows, int64_t k, int block, int scale_is_e8m0, void* out,
                                            void* stream) {
    return fp4_dequant_impl(packed, scale, alpha, rows, k, block, scale_is_e8m0, true, out,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int cdlb200_mxfp8_dequant(const void* packed, const void* scale, const float* alpha,
                                     int64_t rows, int64_t k, void* out, void* stream) {
    if (rows < 0 || k < 0) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || k == 0) return CDLB200_OK;
    if (!packed || !scale || !out || (k % 32) != 0) return CDLB200_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t n = rows * k;
    const bool flat = aligned(packed, 16) && aligned(out, 16);
    if (flat) {
        if (alpha)
            mxfp8_dequant_flat_kernel<true><<<grid_for(n / 16, 256), 256, 0, st>>>(
                static_cast<const uint4*>(packed), static_cast<const uint8_t*>(scale), alpha, n / 16,
                static_cast<uint4*>(out));
        else
            mxfp8_dequant_flat_kernel<false><<<grid_for(n / 16, 256), 256, 0, st>>>(
                static_cast<const uint4*>(packed), static_cast<const uint8_t*>(scale), alpha, n / 16,
                static_cast<uint4*>(out));
    } else {
        if (alpha)
            mxfp8_dequant_generic_kernel<true><<<grid_for(n, 256), 256, 0, st>>>(
                static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scale), alpha, rows, k,
                static_cast<uint16_t*>(out));
        else
            mxfp8_dequant_generic_kernel<false><<<grid_for(n, 256), 256, 0, st>>>(
                static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scale), alpha, rows, k,
                static_cast<uint16_t*>(out));
    }
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int cdlb200_swizzle_scales(const void* sf, int64_t m, int64_t b, void* out, void* stream) {
    if (m < 0 || b < 0) return CDLB200_ERR_INVALID_ARG;
    if (m == 0 || b == 0) return CDLB200_OK;
    if (!sf || !out) return CDLB200_ERR_INVALID_ARG;
    const int64_t c4 = (b + 3) / 4;
    const int64_t total = (m + 127) / 128 * 128 * c4 * 4;
    swizzle_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(sf), m, b, c4, total, static_cast<uint8_t*>(out));
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}
