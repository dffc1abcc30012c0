// common.cuh -- shared helpers for the cdl_b200 sm_100a kernels.
//
// Number formats (OCP MX / NVIDIA NVFP4):
//   e2m1  : 4-bit element, magnitudes {0,.5,1,1.5,2,3,4,6}, nibble = sign<<3 | m
//   e4m3  : 8-bit (fn variant, max 448, 0x7f = NaN), used as NVFP4 block scale
//           (always positive, bytes 1..126) and as the MXFP8 element
//   e8m0  : 8-bit power-of-two scale, byte b -> 2^(b-127), byte 0 = 2^-127
//
// Everything here is plain IEEE fp32 arithmetic with explicit rounding
// intrinsics; the library is built without --use_fast_math (no FTZ, IEEE
// divide), because the e8m0 byte 0 scale and tiny NVFP4 scales are subnormal.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cdlb200.h"

namespace cdlb200 {

enum Fmt : int { kNVFP4 = 0, kMXFP4 = 1, kMXFP8 = 2 };

template <int FMT>
struct FmtTraits;
template <>
struct FmtTraits<kNVFP4> {
    static constexpr int kBlock = 16;
    static constexpr bool kFp4 = true;
    static constexpr int kEmax = 2;
};
template <>
struct FmtTraits<kMXFP4> {
    static constexpr int kBlock = 32;
    static constexpr bool kFp4 = true;
    static constexpr int kEmax = 2;  // floor(log2(6))
};
template <>
struct FmtTraits<kMXFP8> {
    static constexpr int kBlock = 32;
    static constexpr bool kFp4 = false;
    static constexpr int kEmax = 8;  // floor(log2(448))
};

__host__ __device__ __forceinline__ float u2f(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    union { uint32_t u; float f; } c{u};
    return c.f;
#endif
}
__host__ __device__ __forceinline__ uint32_t f2u(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    union { float f; uint32_t u; } c{f};
    return c.u;
#endif
}

// E4M3 (fn) byte -> fp32, from the format definition: bias 7, 3 mantissa bits,
// exponent field 0 = subnormal m * 2^-9.  Only called on NVFP4 scale bytes
// (1..126) and MXFP8 element bytes; 0x7f/0xff decode to NaN.
__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
    uint32_t sign = (b & 0x80u) << 24;
    uint32_t e = (b >> 3) & 0xfu, m = b & 7u;
    uint32_t bits;
    if ((b & 0x7fu) == 0x7fu) {
        bits = 0x7fc00000u;
    } else if (e == 0) {
        // m * 2^-9 : exact in fp32 (normal for m >= 1)
        bits = f2u(__int2float_rn((int)m) * 0.001953125f);
    } else {
        bits = ((e + 120u) << 23) | (m << 20);  // (1 + m/8) * 2^(e-7)
    }
    return u2f(bits | sign);
}

// fp32 -> e4m3 with round-to-nearest-even and saturation to +-448, two at a
// time (hardware cvt).  The value converted from `hi` lands in bits 15:8.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float hi, float lo) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// NVFP4 block-scale byte (UE4M3, zero excluded): e4m3_rne(clamp(q, 2^-9, 448)),
// a NaN q gives byte 126 like the reference's ordinal/pack round trip
// (cdl/core/format/fp8.py:21-31).
__device__ __forceinline__ uint32_t ue4m3_scale_byte(float q) {
    if (q != q) return 126u;
    q = fminf(fmaxf(q, 0.001953125f), 448.0f);
    return cvt_e4m3x2(0.0f, q) & 0xffu;
}

// NVFP4 per-tensor scale alpha = gmax / (6 * 448).  cdl forms it with torch on
// the device (cdl/core/kernel/quant.py:96-101, core/ecdl.py:46-56), where
// `tensor / python_float` runs as a multiply by the fp32 reciprocal of the
// scalar; a true division (what the same line computes on the CPU) differs in
// the last bit for about a fifth of all gmax values.
__device__ __forceinline__ float nvfp4_alpha(float gmax) { return __fmul_rn(gmax, __frcp_rn(2688.0f)); }

// e8m0 scale value 2^(b-127); byte 0 is the fp32 subnormal 2^-127.
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) {
    return u2f(b == 0 ? 0x00400000u : (b << 23));
}

// 1 / e8m0 value = 2^(127-b); b = 254 gives the subnormal 2^-127.
__device__ __forceinline__ float e8m0_inv(uint32_t b) {
    return u2f(b == 254u ? 0x00400000u : ((254u - b) << 23));
}

// MX shared-exponent byte from the block amax given as bf16 magnitude bits
// (cdl/core/ecdl.py:59-73): clamp(floor(log2(max(amax, FLT_MIN))) - emax + 127,
// 0, 254).  +inf -> 254 (log2(inf) clamps to 254); NaN -> 0.
template <int EMAX>
__device__ __forceinline__ uint32_t e8m0_byte_from_bf16_mag(uint32_t mag) {
    if (mag > 0x7f80u) return 0u;
    if (mag == 0x7f80u) return 254u;
    int e = (int)(mag >> 7);            // biased exponent; 0 means below FLT_MIN
    int eb = e == 0 ? 1 : e;            // clamp_min(FLT_MIN) -> exponent -126
    int b = eb - EMAX;                  // (eb - 127) - EMAX + 127
    return (uint32_t)(b < 0 ? 0 : (b > 254 ? 254 : b));
}

// Swizzled 128x4 scale-factor offset (cdl/core/mm/swizzle.py:5-14) of (row r,
// block column c) in a matrix with `c4` = ceil(nb/4) column groups.
__host__ __device__ __forceinline__ int64_t swizzle_offset(int64_t r, int64_t c, int64_t c4) {
    return (((r >> 7) * c4 + (c >> 2)) * 32 + (r & 31)) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
}

// Quotient by a divisor fixed for a launch, for numerators below 2^31, by
// one multiply-high (Granlund & Montgomery, "Division by invariant integers
// using multiplication", PLDI 1994): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (mulhi(m, n) + n) >> l.
struct FastDiv {
    uint32_t d, m, l;
    FastDiv() : d(1), m(1), l(0) {}
    explicit FastDiv(uint32_t div) : d(div < 1 ? 1 : div) {
        l = 0;
        while ((1ull << l) < d) ++l;
        m = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(m, n) + n) >> l; }
};

// Eight e2m1 codes (one 32-bit word, element 2j in the low nibble of byte j)
// -> four f16x2 by the hardware converter (every e2m1 value is exact in f16).
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&h)[4]) {
    asm("{\n"
        ".reg .b8 b0, b1, b2, b3;\n"
        "mov.b32 {b0, b1, b2, b3}, %4;\n"
        "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
        "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
        "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
        "cvt.rn.f16x2.e2m1x2 %3, b3;\n"
        "}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(w));
}

__device__ __forceinline__ void f16x2_to_f32(uint32_t h, float& lo, float& hi) {
    asm("{\n"
        ".reg .f16 a, b;\n"
        "mov.b32 {a, b}, %2;\n"
        "cvt.f32.f16 %0, a;\n"
        "cvt.f32.f16 %1, b;\n"
        "}"
        : "=f"(lo), "=f"(hi)
        : "r"(h));
}

// Streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return u2f(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return u2f(w & 0xffff0000u); }

int num_sms();  // SM count of the current device (cached per device)
uint32_t wait_limit();  // poll limit of bounded grid-wide waits (cdlb200_set_wait_limit)
int persistent_sms();   // SMs a persistent kernel may fill (cdlb200_set_persistent_sm_limit)

}  // namespace cdlb200

#define CDLB200_CHECK_LAUNCH()                                   \
    do {                                                         \
        cudaError_t _e = cudaGetLastError();                     \
        if (_e != cudaSuccess) return CDLB200_ERR_LAUNCH;        \
    } while (0)
