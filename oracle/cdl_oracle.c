/*
 * cdl_oracle.c -- CPU restatement of cdl's block-scaled quantize / dequantize
 * (NVFP4, MXFP4, MXFP8) and of its 128x4 scale-factor swizzle.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the CUDA kernels are
 * compared against; nothing in the product path links, loads or calls it.
 * It is pinned against golden vectors produced by running the reference's own
 * torch path (fp32 format tables) -- see tests/golden/make_golden.py.
 *
 * The arithmetic follows the reference's torch "nearest round" path, which is
 * the bit-exact contract for the quantize kernels:
 *   cdl/core/ecdl.py:46-56    compute_nvidia_scale  (NVFP4 block scale)
 *   cdl/core/ecdl.py:59-73    compute_ocp_scale     (MX e8m0 shared exponent)
 *   cdl/core/ecdl.py:115-131  extended_nearest_round
 *   cdl/core/format/fp4.py:15-21  E2M1 ordinal (strict '>' vs midpoints) + pack
 *   cdl/core/format/fp8.py:7-44   E4M3 / UE4M3ExcludeZero / E8M0 ordinal + pack
 *   cdl/core/tables.py:8-56       level tables (fp32)
 * and the kernel-side conventions of the reference's Triton path:
 *   cdl/core/kernel/quant.py:34,84   K tail zero-padded to whole blocks
 *   cdl/core/kernel/quant.py:96-101  gmax = max|x| clamped to FLT_MIN, alpha = gmax/2688,
 *                                    formed on the device, where torch divides a tensor by
 *                                    a Python float as a multiply by the fp32 reciprocal
 *                                    (on the CPU the same line divides; the two differ in
 *                                    the last bit for about a fifth of all gmax values, none
 *                                    of them in the golden cases)
 *   cdl/core/kernel/dequant.py:6-47  e8m0 byte 0 = 2^-127, dequant = (v*s)*alpha -> bf16
 *   cdl/core/mm/swizzle.py:5-14      128x4 scale-factor tile layout
 *
 * Plain C, IEEE fp32 arithmetic (build without -ffast-math so divides are
 * correctly rounded and subnormals are kept).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define FP32_TINY 1.1754943508222875e-38f /* torch.finfo(float32).tiny */

static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* fp32 -> bf16, round to nearest even (torch .to(bfloat16)); NaN -> quiet NaN. */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

/* OCP FP8 E4M3 (fn: no inf, 0x7f/0xff = NaN, max 448) decode. */
float oracle_e4m3_to_f32(uint8_t b) {
    uint32_t sign = (uint32_t)(b & 0x80) << 24;
    uint32_t e = (b >> 3) & 0xf, m = b & 7;
    float v;
    if ((b & 0x7f) == 0x7f) return u2f(sign | 0x7fc00000u);
    if (e == 0) v = (float)m * (1.0f / 512.0f);           /* subnormal m * 2^-9 */
    else v = ldexpf(1.0f + (float)m / 8.0f, (int)e - 7);
    return u2f(f2u(v) | sign);
}

/* fp32 -> E4M3 round-to-nearest-even, as torch .to(float8_e4m3fn) for
 * |f| <= 448 (callers clamp first, as the reference does).  Magnitudes above
 * 448 saturate to 448 here; NaN -> 0x7f with the input's sign. */
uint8_t oracle_f32_to_e4m3(float f) {
    uint32_t u = f2u(f);
    uint8_t sign = (uint8_t)((u >> 24) & 0x80);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7f;
    if (a >= 0x43e00000u) return sign | 0x7e;              /* >= 448 */
    if (a < 0x3c800000u) {                                  /* < 2^-6: subnormal grid 2^-9 */
        float scaled = u2f(a) * 512.0f;                     /* exact */
        float r = nearbyintf(scaled);                       /* default mode: ties to even */
        return sign | (uint8_t)r;                           /* r == 8 encodes 2^-6 */
    }
    int32_t e = (int32_t)(a >> 23) - 127;                   /* -6 .. 8 */
    uint32_t man = a & 0x7fffffu;
    uint32_t keep = man >> 20, rem = man & 0xfffffu;
    uint32_t up = (rem > 0x80000u) || (rem == 0x80000u && (keep & 1u));
    uint32_t code = ((uint32_t)(e + 7) << 3) + keep + up;  /* carry rolls into exponent */
    if (code > 0x7e) code = 0x7e;
    return sign | (uint8_t)code;
}

/* e8m0 scale value: byte b -> 2^(b-127); byte 0 is the fp32 subnormal 2^-127. */
float oracle_e8m0_to_f32(uint8_t b) {
    return b == 0 ? u2f(0x00400000u) : u2f((uint32_t)b << 23);
}

/* E2M1 ordinal + nibble pack (fp4.py:15-21): m = #{j : min(|v|,6) > mid_j},
 * nibble = m for a clear sign bit, 8 + m for a set sign bit (incl. -0). */
static const float E2M1_MID[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
uint8_t oracle_e2m1_nibble(float v) {
    float a = fabsf(v);
    if (a > 6.0f) a = 6.0f;                                 /* clamp(max=6); NaN stays NaN */
    uint8_t m = 0;
    for (int j = 0; j < 7; ++j) m += (a > E2M1_MID[j]);
    return (uint8_t)((signbit(v) ? 8 : 0) + m);
}

static const float E2M1_LEVEL[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
float oracle_e2m1_value(uint8_t nib) {
    float mag = E2M1_LEVEL[nib & 7];
    return (nib & 8) ? -mag : mag;
}

/* max |x| over n bf16 values, propagating NaN like torch.amax. */
static float absmax_bf16(const uint16_t* x, int64_t n, int* has_nan) {
    float m = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float a = fabsf(bf16_to_f32(x[i]));
        if (a != a) { *has_nan = 1; continue; }
        if (a > m) m = a;
    }
    return m;
}

/* alpha = gmax / (6 * 448) as torch forms it on the device: gmax * RN(1 / 2688). */
static inline float nvfp4_alpha(float gmax) {
    volatile float inv = 1.0f / 2688.0f; /* RN(1/2688), an fp32 constant */
    return gmax * inv;
}

/* Global amax and alpha of the NVFP4 path (quant.py:96-101, ecdl.py:52-56). */
void oracle_nvfp4_global(const uint16_t* x, int64_t n, float* gmax_out, float* alpha_out) {
    int has_nan = 0;
    float g = n > 0 ? absmax_bf16(x, n, &has_nan) : 0.0f;
    if (has_nan) g = u2f(0x7fc00000u);
    else if (g < FP32_TINY) g = FP32_TINY;
    *gmax_out = g;
    *alpha_out = nvfp4_alpha(g);
}

/* Shared exponent byte of an MX block (ecdl.py:59-73): clamp(floor(log2(max(bamax,
 * tiny))) - emax + 127, 0, 254).  +inf -> 254 (log2(inf) = inf, clamped). */
static uint8_t e8m0_byte(float bamax, int emax) {
    if (bamax != bamax) return 0;                           /* undefined in torch (NaN->uint8) */
    if (isinf(bamax)) return 254;
    if (bamax < FP32_TINY) bamax = FP32_TINY;
    int e = (int)(f2u(bamax) >> 23) - 127;                  /* floor(log2) of a normal float */
    int b = e - emax + 127;
    if (b < 0) b = 0;
    if (b > 254) b = 254;
    return (uint8_t)b;
}

/*
 * Row-wise block quantize of a bf16 [rows, k] matrix (row stride ld elements).
 * fmt: 0 = NVFP4 (block 16, ue4m3 scale, per-tensor alpha)
 *      1 = MXFP4 (block 32, e8m0 scale)
 *      2 = MXFP8 (block 32, e8m0 scale, e4m3 elements)
 * Outputs: packed [rows, nb*16/2] (FP4) or [rows, nb*32] (FP8) bytes; scale
 * [rows, nb] linear row-major bytes.  gmax is only read for NVFP4 (pass the
 * value from oracle_nvfp4_global).  K tail zero-padded (quant.py:34).
 */
void oracle_quant(const uint16_t* x, int64_t rows, int64_t k, int64_t ld, int fmt,
                  float gmax, uint8_t* packed, uint8_t* scale) {
    const int B = fmt == 0 ? 16 : 32;
    const int64_t nb = (k + B - 1) / B;
    const int64_t pstride = fmt == 2 ? nb * B : nb * B / 2;
    const float alpha = nvfp4_alpha(gmax);
    float v[32];
    for (int64_t r = 0; r < rows; ++r) {
        const uint16_t* xr = x + r * ld;
        for (int64_t b = 0; b < nb; ++b) {
            float bamax = 0.0f;
            int nan_in_block = 0;
            for (int i = 0; i < B; ++i) {
                int64_t c = b * B + i;
                float f = c < k ? bf16_to_f32(xr[c]) : 0.0f;
                v[i] = f;
                float a = fabsf(f);
                if (a != a) nan_in_block = 1;
                else if (a > bamax) bamax = a;
            }
            if (nan_in_block) bamax = u2f(0x7fc00000u);
            uint8_t sb;
            float s;
            if (fmt == 0) {
                /* ecdl.py:55 q = bamax * 448 / a_b ; fp8.py:27-31 ordinal/pack */
                float q = (bamax * 448.0f) / gmax;
                if (q != q) sb = 126;
                else {
                    float qc = q < 0x1p-9f ? 0x1p-9f : (q > 448.0f ? 448.0f : q);
                    sb = oracle_f32_to_e4m3(qc);
                    if (sb > 126) sb = 126;
                    if (sb < 1) sb = 1;
                }
                s = oracle_e4m3_to_f32(sb) * alpha;          /* ecdl.py:129 */
            } else {
                sb = e8m0_byte(bamax, fmt == 1 ? 2 : 8);
                s = oracle_e8m0_to_f32(sb) * 1.0f;
            }
            scale[r * nb + b] = sb;
            if (fmt == 2) {
                for (int i = 0; i < B; ++i) {
                    float q = v[i] / s;
                    float qc = q != q ? q : (q < -448.0f ? -448.0f : (q > 448.0f ? 448.0f : q));
                    uint8_t u = oracle_f32_to_e4m3(qc);
                    /* fp8.py:13-18 ordinal/pack round trip: NaN bytes become +-448 */
                    if (u == 0x7f) u = 0x7e;
                    else if (u == 0xff) u = 0x7e;
                    packed[r * pstride + b * B + i] = u;
                }
            } else {
                for (int i = 0; i < B; i += 2) {
                    uint8_t lo = oracle_e2m1_nibble(v[i] / s);
                    uint8_t hi = oracle_e2m1_nibble(v[i + 1] / s);
                    packed[r * pstride + (b * B + i) / 2] = (uint8_t)(lo | (hi << 4));
                }
            }
        }
    }
}

/* Dequantize (dequant.py:25-72): bf16((value * scale) * alpha).  fmt as above.
 * k must be a multiple of the block.  alpha is ignored (treated as absent)
 * when has_alpha == 0 (MXFP8 default). */
void oracle_dequant(const uint8_t* packed, const uint8_t* scale, int64_t rows, int64_t k,
                    int fmt, float alpha, int has_alpha, uint16_t* out) {
    const int B = fmt == 0 ? 16 : 32;
    const int64_t nb = k / B;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t c = 0; c < k; ++c) {
            uint8_t sb = scale[r * nb + c / B];
            float sc = fmt == 0 ? oracle_e4m3_to_f32(sb) : oracle_e8m0_to_f32(sb);
            float val;
            if (fmt == 2) val = oracle_e4m3_to_f32(packed[r * k + c]);
            else {
                uint8_t byte = packed[r * (k / 2) + c / 2];
                val = oracle_e2m1_value((uint8_t)((c & 1) ? byte >> 4 : byte & 15));
            }
            float o = val * sc;
            if (fmt != 2 || has_alpha) o = o * alpha;
            out[r * k + c] = oracle_f32_to_bf16(o);
        }
    }
}

/* swizzle_scale_factors (swizzle.py:5-14): [m, b] -> zero-padded
 * [ceil(m/128)*128, ceil(b/4)*4] in 128x4 tiles of 512 bytes; inside a tile the
 * byte for (row r, col c) sits at (r%32)*16 + ((r/32)%4)*4 + c%4. */
void oracle_swizzle(const uint8_t* sf, int64_t m, int64_t b, uint8_t* out) {
    const int64_t rows = (m + 127) / 128 * 128, cols = (b + 3) / 4 * 4;
    const int64_t c4 = cols / 4;
    memset(out, 0, (size_t)(rows * cols));
    for (int64_t r = 0; r < m; ++r)
        for (int64_t c = 0; c < b; ++c) {
            int64_t off = (((r / 128) * c4 + c / 4) * 32 + r % 32) * 16 + ((r / 32) % 4) * 4 + c % 4;
            out[off] = sf[r * b + c];
        }
}
