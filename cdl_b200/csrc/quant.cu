// quant.cu -- block-scaled NVFP4 / MXFP4 / MXFP8 quantize kernels (sm_100a).
//
// Replaces cdl's Triton `_quant_kernel` + host `_quant`
// (cdl/core/kernel/quant.py:13-146) and the torch global amax it launches
// (quant.py:96-101).  Results are bit-identical to cdl's torch nearest-round
// path (cdl/core/ecdl.py:46-131 with fp32 format tables).
//
// Layout in HBM.  A row-major bf16 [rows, k] matrix with k % block == 0 is one
// flat array of blocks; so are its packed codes (k/2 or k bytes per row) and
// its linear scales (one byte per block).  The fast path therefore streams
// 16-byte vectors: one vector = 8 elements, a block = 2 (NVFP4) or 4 (MX)
// adjacent lanes of a warp, reduced with one or two shuffles.  Every global
// load and store of a warp covers one contiguous span (512 B in, 128 B or
// 256 B out).
//
// E2M1 encoding without a per-element divide.  cdl computes v = RN(x / s) and
// counts the e2m1 midpoints mid_j in {.25,.75,1.25,1.75,2.5,3.5,5} that
// |v| exceeds (strict '>', so ties round toward zero; cdl/core/format/
// fp4.py:15-17).  The hardware cvt.rn.satfinite.e2m1x2 rounds ties to even
// instead, so it is only used on a value nudged just below the true one:
//
//   MX (s = 2^e): x * 2^-e is exact (bf16 has 8 significant bits), it differs
//   from every midpoint it is not equal to by >= 2^-9 relative, so
//   v' = RN(x * 2^-e * (1 - 2^-20)) lies on the same side of every midpoint
//   and strictly below a midpoint it equals.  cvt(v') is then exactly cdl's
//   code, sign and -0 included.
//
//   NVFP4 (general fp32 s): all mid_j have an even last mantissa bit, so
//       RN(|x|/s) > mid_j  <=>  |x| > T_j := RD((mid_j + ulp(mid_j)/2) * s)
//   with T_j = fma_rd(mid_j, s, s*ulp(mid_j)/2) exact for s >= 2^-100.  A bf16
//   |x| exceeds T_j iff it is >= n_j, the next bf16 value above T_j.  With
//   c = RN(RN(1/s) * (1 - 2^-20)), RN(T_j*c) < mid_j always, and
//   RN(n_j*c) > mid_j whenever n_j - T_j >= 64 ulp(T_j) (2^-18 relative).  A
//   block whose seven T_j all keep that margin (about 99.3% of blocks) is
//   encoded as cvt(RN(x*c)); the others compare |x| against T_j directly.
//   Blocks with a tiny or non-finite s use the literal IEEE divide.
//
// The NVFP4 scale byte needs q = RN(RN(bamax*448) / gmax) only up to its e4m3
// rounding.  RN(bamax*448) has <= 11 significant bits and gmax <= 8, so their
// quotient either equals an e4m3 rounding boundary (<= 5 bits) exactly or is
// >= 2^-14 away from it; one Markstein correction of RN(p * RN(1/gmax))
// (exact when the quotient is representable, within 2 ulp otherwise) gives
// the same byte as the IEEE divide.
#include <vector>

#include "cdlb200_step.h"
#include "common.cuh"

namespace cdlb200 {

namespace {

// e2m1 midpoints mid_j and ulp(mid_j) / 2 = 2^(floor(log2(mid_j)) - 24)
__device__ __forceinline__ constexpr float mid_j(int j) {
    return j == 0 ? 0.25f : j == 1 ? 0.75f : j == 2 ? 1.25f : j == 3 ? 1.75f : j == 4 ? 2.5f : j == 5 ? 3.5f : 5.0f;
}
__device__ __forceinline__ constexpr float half_ulp_j(int j) {
    return j == 0 ? 0x1p-26f : j == 1 ? 0x1p-25f : j <= 3 ? 0x1p-24f : j <= 5 ? 0x1p-23f : 0x1p-22f;
}
// NVFP4 workspace: [0] arrival counter, [4] departure counter (fused kernel),
// [8] status word (non-zero after a timed-out grid barrier), [12] running max
// of the fused kernel, [16] global amax of the fp32 / fp16 path (quant_wide.cu),
// [256..) partial maxima.
constexpr int kWsCounterOff = 0;
constexpr int kWsDepartOff = 4;
constexpr int kWsStatusOff = 8;
constexpr int kWsGmaxOff = 12;  // fused kernel: running max of the CTA maxima (bf16 magnitude bits)
constexpr int kWsPartialOff = 256;
constexpr int kMaxAmaxGrid = 1024;

struct BlockCode {
    float t[7];      // e2m1 thresholds on |x| (FP4) ; t[0] = 1/scale (FP8)
    float s;         // block scale (NVFP4 fallback divide)
    bool exact_div;  // NVFP4 fallback: divide literally
    uint32_t byte;   // stored scale byte
};

// Per 16-bit lane, max(|a|, |b|) of two bf16 pairs: one instruction that
// propagates NaN (the canonical NaN, magnitude 0x7fff, above every finite
// value and Inf); the result's sign bits are the XOR of the inputs' and are
// masked off by the callers.
__device__ __forceinline__ uint32_t absmax2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t lane_max(uint32_t m) {
    m &= 0x7fff7fffu;
    return max(m & 0xffffu, m >> 16);
}

// max |x| of 8 bf16 values as bf16 magnitude bits (any NaN -> 0x7fff, above Inf).
__device__ __forceinline__ uint32_t amax8(const uint4& w) {
    return lane_max(absmax2(absmax2(w.x, w.y), absmax2(w.z, w.w)));
}

// max |x| of the 16 bf16 values of one NVFP4 block (two 8-value vectors).
__device__ __forceinline__ uint32_t amax16(const uint4& a, const uint4& b) {
    return lane_max(absmax2(absmax2(absmax2(a.x, a.y), absmax2(a.z, a.w)), absmax2(absmax2(b.x, b.y), absmax2(b.z, b.w))));
}

__device__ __forceinline__ float mag_to_f32(uint32_t mag) { return u2f(mag << 16); }

template <int FMT>
__device__ __forceinline__ void block_setup(uint32_t mag, float gmax, float alpha, BlockCode& bc) {
    if constexpr (FMT == kNVFP4) {
        // cdl/core/ecdl.py:55  q = bamax * 448 / gmax (two roundings, as cdl)
        float bamax = mag > 0x7f80u ? u2f(0x7fc00000u) : mag_to_f32(mag);
        float q = __fdiv_rn(__fmul_rn(bamax, 448.0f), gmax);
        bc.byte = ue4m3_scale_byte(q);  // same byte as nvfp4_scale_byte (see header)
        float s = __fmul_rn(e4m3_to_f32(bc.byte), alpha);  // ecdl.py:129
        bc.s = s;
        bc.exact_div = !(s >= 0x1p-100f && s <= 3.4028234e38f);
#pragma unroll
        for (int j = 0; j < 7; ++j) bc.t[j] = __fmaf_rd(mid_j(j), s, __fmul_rn(s, half_ulp_j(j)));
    } else {
        bc.byte = e8m0_byte_from_bf16_mag<FmtTraits<FMT>::kEmax>(mag);
        bc.exact_div = false;
        if constexpr (FMT == kMXFP4) {
            float s = e8m0_to_f32(bc.byte);
            bc.s = s;
            // mid_j * 2^127 overflows for mid_j >= 2.5; finite |x| / 2^127 < 2 never
            // exceeds those midpoints while +-inf exceeds all of them, so FLT_MAX
            // is the exact threshold there.
#pragma unroll
            for (int j = 0; j < 7; ++j) bc.t[j] = fminf(__fmul_rn(mid_j(j), s), 3.4028234664e38f);
        } else {
            bc.s = e8m0_inv(bc.byte);  // RN(x / 2^e) == x * 2^-e exactly
        }
    }
}

__device__ __forceinline__ uint32_t e2m1_mag_thresh(float a, const float* t) {
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 7; ++j) m += (a > t[j]) ? 1u : 0u;
    return m;
}

// nibble of one bf16 element (given as its 16 bits in the low half of h)
__device__ __forceinline__ uint32_t e2m1_nibble(uint32_t h, const BlockCode& bc) {
    if (!bc.exact_div) {
        uint32_t m = e2m1_mag_thresh(u2f((h & 0x7fffu) << 16), bc.t);
        return m | ((h >> 12) & 8u);
    }
    float v = __fdiv_rn(u2f(h << 16), bc.s);
    float a = fabsf(v);
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 7; ++j) m += (a > mid_j(j)) ? 1u : 0u;
    return m | (signbit(v) ? 8u : 0u);
}

// 8 elements -> 8 nibbles (element e at bits 4e..4e+3)
__device__ __forceinline__ uint32_t encode8_fp4(const uint4& w, const BlockCode& bc) {
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t lo = e2m1_nibble(ws[i] & 0xffffu, bc);
        uint32_t hi = e2m1_nibble(ws[i] >> 16, bc);
        out |= (lo | (hi << 4)) << (8 * i);
    }
    return out;
}

// 8 elements -> 8 e4m3 bytes
__device__ __forceinline__ uint2 encode8_fp8(const uint4& w, const BlockCode& bc) {
    const float inv = bc.s;
    uint32_t b01 = cvt_e4m3x2(__fmul_rn(bf16hi(w.x), inv), __fmul_rn(bf16lo(w.x), inv));
    uint32_t b23 = cvt_e4m3x2(__fmul_rn(bf16hi(w.y), inv), __fmul_rn(bf16lo(w.y), inv));
    uint32_t b45 = cvt_e4m3x2(__fmul_rn(bf16hi(w.z), inv), __fmul_rn(bf16lo(w.z), inv));
    uint32_t b67 = cvt_e4m3x2(__fmul_rn(bf16hi(w.w), inv), __fmul_rn(bf16lo(w.w), inv));
    return make_uint2(b01 | (b23 << 16), b45 | (b67 << 16));
}

// Per-tensor NVFP4 constants shared by every block of one call.
struct Nvfp4Tensor {
    float gmax, alpha, yg;  // yg = RN(1 / gmax)
    bool markstein;         // gmax in [2^-100, 1e35]: p / gmax via one Markstein step
};

__device__ __forceinline__ Nvfp4Tensor nvfp4_tensor(const float* gmax_p, const float* alpha_p) {
    Nvfp4Tensor g;
    g.gmax = *gmax_p;
    g.alpha = *alpha_p;
    g.markstein = g.gmax >= 0x1p-100f && g.gmax <= 1.0e35f;
    g.yg = g.markstein ? __frcp_rn(g.gmax) : 0.0f;
    return g;
}

// e4m3 scale byte of a block with bf16 amax bits `mag` (cdl/core/ecdl.py:52-55).
__device__ __forceinline__ uint32_t nvfp4_scale_byte(uint32_t mag, const Nvfp4Tensor& g) {
    const float bamax = u2f(mag << 16);  // a NaN magnitude (> 0x7f80) is a NaN float
    const float p = __fmul_rn(bamax, 448.0f);
    float q;
    if (g.markstein) {
        const float q0 = __fmul_rn(p, g.yg);
        const float r = __fmaf_rn(-q0, g.gmax, p);
        q = __fmaf_rn(r, g.yg, q0);
    } else {
        q = __fdiv_rn(p, g.gmax);
    }
    return ue4m3_scale_byte(q);
}

// 8 values (fp32 bit patterns f0..f7, here bf16 values widened) times c -> 8
// e2m1 nibbles, value i at bits 4i..4i+3.  Each pair is one packed fp32 multiply
// (mul.rn.f32x2: each lane an IEEE round-to-nearest product, the same as two
// __fmul_rn) and one hardware conversion (RNE, saturating); the four code
// bytes are packed by one move.
__device__ __forceinline__ uint32_t cvt8_bits_scaled(uint32_t f0, uint32_t f1, uint32_t f2, uint32_t f3, uint32_t f4,
                                                     uint32_t f5, uint32_t f6, uint32_t f7, float c) {
    uint32_t out;
    asm("{\n"
        ".reg .b64 cc, p0, p1, p2, p3;\n"
        ".reg .f32 l0, h0, l1, h1, l2, h2, l3, h3;\n"
        ".reg .b8 b0, b1, b2, b3;\n"
        "mov.b64 cc, {%9, %9};\n"
        "mov.b64 p0, {%1, %2};\n"
        "mov.b64 p1, {%3, %4};\n"
        "mov.b64 p2, {%5, %6};\n"
        "mov.b64 p3, {%7, %8};\n"
        "mul.rn.f32x2 p0, p0, cc;\n"
        "mul.rn.f32x2 p1, p1, cc;\n"
        "mul.rn.f32x2 p2, p2, cc;\n"
        "mul.rn.f32x2 p3, p3, cc;\n"
        "mov.b64 {l0, h0}, p0;\n"
        "mov.b64 {l1, h1}, p1;\n"
        "mov.b64 {l2, h2}, p2;\n"
        "mov.b64 {l3, h3}, p3;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b0, h0, l0;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b1, h1, l1;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b2, h2, l2;\n"
        "cvt.rn.satfinite.e2m1x2.f32 b3, h3, l3;\n"
        "mov.b32 %0, {b0, b1, b2, b3};\n"
        "}"
        : "=r"(out)
        : "r"(f0), "r"(f1), "r"(f2), "r"(f3), "r"(f4), "r"(f5), "r"(f6), "r"(f7), "f"(c));
    return out;
}

// 8 bf16 (one uint4: pairs (x0, x1) .. (x6, x7)) times c, element i at bits 4i..
__device__ __forceinline__ uint32_t cvt8_scaled(const uint4& w, float c) {
    return cvt8_bits_scaled(w.x << 16, w.x & 0xffff0000u, w.y << 16, w.y & 0xffff0000u, w.z << 16, w.z & 0xffff0000u,
                            w.w << 16, w.w & 0xffff0000u, c);
}

// The same for the low (HI = false) or high 16-bit halves of eight words:
// value i is half HI of v[i] (a column of a row-major bf16 tile, two columns
// per word), without regrouping the halves first.
template <bool HI>
__device__ __forceinline__ uint32_t cvt8_halves_scaled(const uint32_t* v, float c) {
    auto f = [](uint32_t w) { return HI ? (w & 0xffff0000u) : (w << 16); };
    return cvt8_bits_scaled(f(v[0]), f(v[1]), f(v[2]), f(v[3]), f(v[4]), f(v[5]), f(v[6]), f(v[7]), c);
}

// RN(1/s) to within 2^-22 relative: hardware approximation refined by one
// Newton-Raphson step (y1 = y0 + y0 * (1 - s*y0)).  The fast encoder's bounds
// hold for any reciprocal within 2^-21.
__device__ __forceinline__ float recip_nr(float s) {
    float y0;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y0) : "f"(s));
    const float e = __fmaf_rn(-s, y0, 1.0f);
    return __fmaf_rn(y0, e, y0);
}

__device__ __forceinline__ uint32_t bf16x2_gt(uint32_t a, uint32_t b) {
    uint32_t m;
    asm("set.gt.u32.bf16x2 %0, %1, %2;" : "=r"(m) : "r"(a), "r"(b));
    return m;  // 0xffff in each half where a > b
}

// 8 elements (one uint4: pairs (x0,x1) .. (x6,x7)) -> 8 nibbles, exact, by a
// three-level binary search of each bf16 magnitude against the thresholds.
// Words are regrouped as (x_k, x_k+4) so that each lane's result bits land in
// its own 16-bit half: nibble k in bits 4k.., nibble k+4 in bits 16+4k...
__device__ __forceinline__ uint32_t search8(const uint4& w, const uint32_t* tt) {
    const uint32_t r[4] = {__byte_perm(w.x, w.z, 0x5410), __byte_perm(w.x, w.z, 0x7632),
                           __byte_perm(w.y, w.w, 0x5410), __byte_perm(w.y, w.w, 0x7632)};
    uint32_t out = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t a = r[k] & 0x7fff7fffu;
        const uint32_t c3 = bf16x2_gt(a, tt[3]);
        const uint32_t c2 = bf16x2_gt(a, (c3 & tt[5]) | (~c3 & tt[1]));
        const uint32_t hi = (c2 & tt[6]) | (~c2 & tt[4]);
        const uint32_t lo = (c2 & tt[2]) | (~c2 & tt[0]);
        const uint32_t c1 = bf16x2_gt(a, (c3 & hi) | (~c3 & lo));
        const uint32_t sh = 4 * k;
        out |= (c1 & (0x00010001u << sh)) | (c2 & (0x00020002u << sh)) | (c3 & (0x00040004u << sh)) |
               ((r[k] >> (12 - sh)) & (0x00080008u << sh));
    }
    return out;
}

// One NVFP4 block of 16 elements (w0, w1) with amax bits `mag`: returns the
// scale byte and writes the 8 code bytes to out.x / out.y.
//
// The fast-path check needs only four thresholds: T_0 = RD(0.25 s (1+2^-24))
// = 0.25 s, and T_4 = 2 T_2, T_5 = 2 T_3, T_6 = 4 T_2 (directed rounding
// commutes with scaling by 2), so the low 16 bits of s, T_1, T_2, T_3 cover
// all seven.
__device__ __forceinline__ uint32_t nvfp4_block16(const uint4& w0, const uint4& w1, uint32_t mag,
                                                  const Nvfp4Tensor& g, uint2& out) {
    const uint32_t byte = nvfp4_scale_byte(mag, g);
    const float s = __fmul_rn(e4m3_to_f32(byte), g.alpha);  // cdl/core/ecdl.py:129
    if (s >= 0x1p-100f && s <= 3.4028234e38f) {
        const float t1 = __fmaf_rd(0.75f, s, __fmul_rn(s, 0x1p-25f));
        const float t2 = __fmaf_rd(1.25f, s, __fmul_rn(s, 0x1p-24f));
        const float t3 = __fmaf_rd(1.75f, s, __fmul_rn(s, 0x1p-24f));
        uint32_t a, b, hi;
        asm("max.u16x2 %0, %1, %2;" : "=r"(a) : "r"(f2u(s)), "r"(f2u(t1)));
        asm("max.u16x2 %0, %1, %2;" : "=r"(b) : "r"(f2u(t2)), "r"(f2u(t3)));
        asm("max.u16x2 %0, %1, %2;" : "=r"(hi) : "r"(a), "r"(b));
        if ((hi & 0xffffu) <= 0xffc0u) {  // every threshold keeps >= 64 ulp below the next bf16
            const float c = __fmul_rn(recip_nr(s), 0.99999904632568359375f);  // (1 - 2^-20) / s
            out.x = cvt8_scaled(w0, c);
            out.y = cvt8_scaled(w1, c);
        } else {
            // a threshold lies within 64 ulp below a bf16 value: compare the
            // bf16 magnitudes against t_j = RD_bf16(T_j) (x > T_j <=> x > t_j
            // for bf16 x), packed two per word
            uint32_t tt[7];
#pragma unroll
            for (int j = 0; j < 7; ++j) tt[j] = (f2u(__fmaf_rd(mid_j(j), s, __fmul_rn(s, half_ulp_j(j)))) >> 16) * 0x00010001u;
            out.x = search8(w0, tt);
            out.y = search8(w1, tt);
        }
    } else {
        BlockCode bc;
        bc.s = s;
        bc.exact_div = true;
        out.x = encode8_fp4(w0, bc);
        out.y = encode8_fp4(w1, bc);
    }
    return byte;
}

// ---------------------------------------------------------------------------
// global amax (NVFP4): per-CTA partial maxima, the last CTA to finish reduces
// them and writes gmax / alpha, then re-arms the counter for the next call.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512, 2) amax_kernel(const uint16_t* __restrict__ x, int64_t rows,
                                                   int64_t k, int64_t ldx, int vec_ok,
                                                   uint32_t* __restrict__ partial,
                                                   uint32_t* __restrict__ counter,
                                                   float* __restrict__ gmax_out,
                                                   float* __restrict__ alpha_out) {
    uint32_t m = 0;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
    if (vec_ok) {  // contiguous, 16-byte aligned: flat vector loop + scalar tail
        const int64_t n = rows * k;
        const int64_t nvec = n >> 3;
        const uint4* xv = reinterpret_cast<const uint4*>(x);
        int64_t v = tid;
        for (; v + 3 * nthr < nvec; v += 4 * nthr) {
            uint4 a = ldg_stream(xv + v), b = ldg_stream(xv + v + nthr);
            uint4 c = ldg_stream(xv + v + 2 * nthr), d = ldg_stream(xv + v + 3 * nthr);
            m = max(m, max(amax16(a, b), amax16(c, d)));
        }
        for (; v < nvec; v += nthr) m = max(m, amax8(ldg_stream(xv + v)));
        for (int64_t i = (nvec << 3) + tid; i < n; i += nthr) m = max(m, (uint32_t)(x[i] & 0x7fffu));
    } else {
        for (int64_t r = blockIdx.x; r < rows; r += gridDim.x)
            for (int64_t c = threadIdx.x; c < k; c += blockDim.x)
                m = max(m, (uint32_t)(x[r * ldx + c] & 0x7fffu));
    }
    m = __reduce_max_sync(0xffffffffu, m);
    __shared__ uint32_t warp_max[16];
    __shared__ bool is_last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) warp_max[warp] = m;
    __syncthreads();
    if (warp == 0) {
        uint32_t wm = lane < (int)(blockDim.x >> 5) ? warp_max[lane] : 0u;
        wm = __reduce_max_sync(0xffffffffu, wm);
        if (lane == 0) {
            partial[blockIdx.x] = wm;
            __threadfence();
            uint32_t prev = atomicAdd(counter, 1u);
            is_last = prev == gridDim.x - 1;
        }
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    uint32_t g = 0;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x) g = max(g, __ldcg(partial + i));
    g = __reduce_max_sync(0xffffffffu, g);
    if (lane == 0) warp_max[warp] = g;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t gm = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) gm = max(gm, warp_max[w]);
        float gmax;
        if (gm > 0x7f80u) gmax = u2f(0x7fc00000u);
        else gmax = fmaxf(mag_to_f32(gm), 1.1754943508222875e-38f);  // clamp_min(tiny)
        if (gmax_out) *gmax_out = gmax;
        *alpha_out = nvfp4_alpha(gmax);
        *counter = 0u;
    }
}

// gmax for an empty tensor (quant.py:99-101): tiny, alpha = nvfp4_alpha(tiny)
__global__ void empty_alpha_kernel(float* gmax_out, float* alpha_out) {
    const float tiny = 1.1754943508222875e-38f;
    if (gmax_out) *gmax_out = tiny;
    *alpha_out = nvfp4_alpha(tiny);
}

// ---------------------------------------------------------------------------
// fast path: contiguous rows, k % block == 0, 16-byte aligned input
// ---------------------------------------------------------------------------
template <int FMT, bool SWZ, int U>
__global__ void __launch_bounds__(256) quant_flat_kernel(const uint4* __restrict__ x, int64_t nvec,
                                                         uint8_t* __restrict__ packed,
                                                         uint8_t* __restrict__ scale, FastDiv nb,
                                                         int64_t c4, const float* __restrict__ gmax_p,
                                                         const float* __restrict__ alpha_p) {
    constexpr int B = FmtTraits<FMT>::kBlock;
    constexpr int VPB = B / 8;
    float gmax = 0.f, alpha = 0.f;
    if constexpr (FMT == kNVFP4) {
        gmax = *gmax_p;
        alpha = *alpha_p;
    }
    const int lane = threadIdx.x & 31;
    const int64_t warp_base = (int64_t)blockIdx.x * blockDim.x * U + (threadIdx.x & ~31) * U;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x * U;
    for (int64_t base = warp_base; base < nvec; base += stride) {
        uint4 w[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int64_t v = base + 32 * u + lane;
            w[u] = v < nvec ? ldg_stream(x + v) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t v = base + 32 * u + lane;
            uint32_t mag = amax8(w[u]);
            mag = max(mag, __shfl_xor_sync(0xffffffffu, mag, 1));
            if constexpr (VPB == 4) mag = max(mag, __shfl_xor_sync(0xffffffffu, mag, 2));
            if (v < nvec) {
                BlockCode bc;
                if constexpr (FMT == kMXFP4) {
                    bc.byte = e8m0_byte_from_bf16_mag<FmtTraits<FMT>::kEmax>(mag);
                    // 2^-e * (1 - 2^-20): exact, also for the subnormal 2^-127
                    const float c = __fmul_rn(e8m0_inv(bc.byte), 0.99999904632568359375f);
                    reinterpret_cast<uint32_t*>(packed)[v] = cvt8_scaled(w[u], c);
                } else {
                    block_setup<FMT>(mag, gmax, alpha, bc);
                    reinterpret_cast<uint2*>(packed)[v] = encode8_fp8(w[u], bc);
                }
                if ((lane & (VPB - 1)) == 0) {
                    const int64_t blk = v / VPB;
                    int64_t off = blk;
                    if constexpr (SWZ) {  // the host guarantees < 2^31 blocks with SWZ
                        const uint32_t r = nb.div((uint32_t)blk);
                        off = swizzle_offset(r, (int64_t)((uint32_t)blk - r * nb.d), c4);
                    }
                    scale[off] = (uint8_t)bc.byte;
                }
            }
        }
    }
}

// NVFP4 fast path: one thread per 16-element block (two 16-byte loads, one
// 8-byte code store, one scale byte), so the per-block scale and threshold
// set-up is computed once per block.  U blocks per thread per iteration.
template <bool SWZ, int U>
__global__ void __launch_bounds__(256) nvfp4_flat_kernel(const uint4* __restrict__ x, int64_t nblk,
                                                         uint2* __restrict__ packed,
                                                         uint8_t* __restrict__ scale, FastDiv nb,
                                                         int64_t c4, const float* __restrict__ gmax_p,
                                                         const float* __restrict__ alpha_p) {
    const Nvfp4Tensor g = nvfp4_tensor(gmax_p, alpha_p);
    const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nblk; base += nthr * U) {
        uint4 w0[U], w1[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t b = base + u * nthr;
            if (b < nblk) {
                w0[u] = ldg_stream(x + 2 * b);
                w1[u] = ldg_stream(x + 2 * b + 1);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t b = base + u * nthr;
            if (b < nblk) {
                uint2 out;
                const uint32_t byte = nvfp4_block16(w0[u], w1[u], amax16(w0[u], w1[u]), g, out);
                packed[b] = out;
                int64_t off = b;
                if constexpr (SWZ) {  // the host guarantees < 2^31 blocks with SWZ
                    const uint32_t r = nb.div((uint32_t)b);
                    off = swizzle_offset(r, (int64_t)((uint32_t)b - r * nb.d), c4);
                }
                scale[off] = (uint8_t)byte;
            }
        }
    }
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Per-CTA table of everything an NVFP4 block needs besides its codes, indexed
// by the block's scale byte (1..126), built once per CTA after the barrier.
//
//   tt[j]  t_j, the largest bf16 value <= T_j, in both halves of a word: a
//          bf16 |x| has code > j iff |x| > t_j (exact; used by the packed
//          binary search below).
//   c      the encoder multiplier, when one separates every threshold: let
//          n_j be the bf16 value after t_j; if RN(t_j*c) < mid_j and
//          RN(n_j*c) > mid_j for all seven j, then, a -> RN(a*c) being
//          monotone, cvt.rn(RN(|x|*c)) equals cdl's code for every bf16 x and
//          no product lands on a midpoint.  The 14 products are evaluated with
//          the encoder's own rounding for a few c = RN(1/s)*(1 - nu).
//   kind   kCvt (c separates every threshold), kSearch (no candidate does:
//          thresholds pinched against the bf16 grid from both sides, which
//          happens for whole tensors because gmax/2688 has short periodic
//          binary expansions), kDivide (s below 2^-100 or not finite:
//          literal IEEE divide).
// The table is identical on every CTA, so the encoding mode chosen from it is
// uniform across the grid: cvt when no entry has exceptions, otherwise the
// packed search (and the divide for kDivide entries).
constexpr uint32_t kCvt = 0u, kSearch = 1u, kDivide = 2u;
struct ScaleEntry {
    float c, s;
    uint32_t kind, pad;
    uint32_t tt[8];
};

// Scale entry of `byte` built cooperatively by 4 adjacent lanes of a warp:
// lane i tries c = RN(1/s)*(1 - nu_i) (nu = 2^-20, 2^-21, 2^-19, 2^-22) and
// the first candidate that separates all seven thresholds wins.
__device__ __forceinline__ ScaleEntry make_scale_entry(uint32_t byte, float alpha, int cand) {
    ScaleEntry e;
    e.s = __fmul_rn(e4m3_to_f32(byte), alpha);
    e.c = 0.0f;
    e.pad = 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) e.tt[j] = 0u;
    const bool divide = !(e.s >= 0x1p-100f && e.s <= 3.4028234e38f);
    // T_0 = RD(0.25 s (1 + 2^-24)) = 0.25 s; T_4 = 2 T_2, T_5 = 2 T_3, T_6 = 4 T_2
    float T[7];
    T[0] = __fmul_rn(e.s, 0.25f);
    T[1] = __fmaf_rd(0.75f, e.s, __fmul_rn(e.s, 0x1p-25f));
    T[2] = __fmaf_rd(1.25f, e.s, __fmul_rn(e.s, 0x1p-24f));
    T[3] = __fmaf_rd(1.75f, e.s, __fmul_rn(e.s, 0x1p-24f));
    T[4] = __fmul_rn(T[2], 2.0f);
    T[5] = __fmul_rn(T[3], 2.0f);
    T[6] = __fmul_rn(T[2], 4.0f);
#pragma unroll
    for (int j = 0; j < 7; ++j) {
        const uint32_t t16 = f2u(T[j]) >> 16;
        e.tt[j] = t16 | (t16 << 16);
    }
    const float nu = cand == 0 ? 0x1p-20f : cand == 1 ? 0x1p-21f : cand == 2 ? 0x1p-19f : cand == 3 ? 0x1p-22f
                   : cand == 4 ? 0x1p-18f : cand == 5 ? 0x1p-23f : cand == 6 ? 0x1p-17f : 0x1p-24f;
    const float c = __fmul_rn(recip_nr(e.s), 1.0f - nu);
    bool ok = !divide;
#pragma unroll
    for (int j = 0; j < 7; ++j) {
        const uint32_t tb = f2u(T[j]) & 0xffff0000u;
        ok = ok && (__fmul_rn(u2f(tb), c) < mid_j(j)) && (__fmul_rn(u2f(tb + 0x10000u), c) > mid_j(j));
    }
    const uint32_t lane = threadIdx.x & 31, grp = lane & ~3u;
    const uint32_t votes = (__ballot_sync(0xffffffffu, ok) >> grp) & 0xfu;
    const int first = votes ? __ffs(votes) - 1 : -1;
    e.c = __shfl_sync(0xffffffffu, c, (int)grp + (first < 0 ? 0 : first));
    e.kind = divide ? kDivide : (first < 0 ? kSearch : kCvt);
    return e;
}

// NVFP4 fused path: global amax and encode in ONE persistent cooperative
// launch, two 512-thread CTAs per SM.  The input is cut into chunks of 512
// blocks (16 KiB), dealt round-robin to the CTAs so that each CTA streams
// from every part of the tensor.
//   phase 1  stream own chunks from HBM (four 32-byte blocks in flight per
//            thread), reduce max|x|, keep every block's amax in shared
//            memory, fold the CTA maximum into one global word (atomicMax)
//            and arrive on a grid barrier;
//   phase 2  every CTA reads the global amax, builds the 126-entry scale
//            table (4 lanes per entry), and re-encodes its chunks in reverse
//            order -- most recently streamed first, so they come from L2.
// The grid-barrier wait is bounded (cdlb200_set_wait_limit polls, by default
// 2^20, about a second): on a timeout the CTA writes a non-zero status word
// into the workspace (byte offset 8) and carries on with the maxima that have
// arrived, so a failed wait never hangs the GPU; the host reads and clears
// that word (cdl_b200._lib.check_status).  The last CTA to finish
// re-arms the barrier words for the next stream-ordered call.
constexpr int kFusedThreads = 512;  // threads of the fused NVFP4 kernel (two CTAs per SM)
constexpr int kChunkBlocks = kFusedThreads;  // one block per thread per chunk (16 KiB)
constexpr int kAmaxChunks = 16;  // chunks whose per-block amax phase 1 keeps for phase 2
constexpr int kMaxSearchEntries = 8;  // more kSearch table entries than this: search every block

// Codes of one block with the table entry of its scale byte: the hardware
// converter for a kCvt entry, else the exact search (kSearch, or every entry
// when `all_search`), or the literal divide (kDivide).
__device__ __forceinline__ uint2 encode_block(const uint4& a0, const uint4& a1, const ScaleEntry& e,
                                              bool all_search) {
    uint2 out;
    const uint32_t kind = e.kind;
    if (kind == kCvt && !all_search) {
        out.x = cvt8_scaled(a0, e.c);
        out.y = cvt8_scaled(a1, e.c);
    } else if (kind != kDivide) {
        uint32_t tt[7];
#pragma unroll
        for (int j = 0; j < 7; ++j) tt[j] = e.tt[j];
        out.x = search8(a0, tt);
        out.y = search8(a1, tt);
    } else {
        BlockCode bc;
        bc.s = e.s;
        bc.exact_div = true;
        out.x = encode8_fp4(a0, bc);
        out.y = encode8_fp4(a1, bc);
    }
    return out;
}

template <bool SWZ>
__global__ void __launch_bounds__(kFusedThreads, 2) nvfp4_fused_kernel(
    const uint4* __restrict__ x, int64_t nblk, uint2* __restrict__ packed, uint8_t* __restrict__ scale,
    FastDiv nb, int64_t c4, uint8_t* __restrict__ ws, float* __restrict__ gmax_out,
    float* __restrict__ alpha_out, uint32_t spin_limit) {
    __shared__ uint32_t red[kFusedThreads / 32];
    __shared__ ScaleEntry table[128];
    __shared__ float ctab[128];  // the cvt multiplier of a kCvt entry, else -1: one 4-byte lookup per block
    __shared__ float s_gmax;
    __shared__ int s_mode;
    __shared__ uint16_t amax_s[kAmaxChunks * kChunkBlocks];
    uint32_t* arrive = reinterpret_cast<uint32_t*>(ws + kWsCounterOff);
    uint32_t* depart = reinterpret_cast<uint32_t*>(ws + kWsDepartOff);
    uint32_t* status = reinterpret_cast<uint32_t*>(ws + kWsStatusOff);
    uint32_t* gmax_bits = reinterpret_cast<uint32_t*>(ws + kWsGmaxOff);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t G = gridDim.x;
    const int64_t nchunk = (nblk + kChunkBlocks - 1) / kChunkBlocks;
    const int nmine = nchunk > (int64_t)blockIdx.x ? (int)((nchunk - 1 - blockIdx.x) / G + 1) : 0;
    auto blk = [&](int q) { return ((int64_t)blockIdx.x + (int64_t)q * G) * kChunkBlocks + tid; };

    // ---- phase 1: stream own chunks (four blocks in flight per thread),
    //      reduce max|x|, keep each block's amax in shared memory
    uint32_t m = 0;
    for (int q0 = 0; q0 < nmine; q0 += 4) {
        uint4 v[8];
        bool ok[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t b = blk(q0 + u);
            ok[u] = q0 + u < nmine && b < nblk;
            if (ok[u]) {
                v[2 * u] = ldg_stream(x + 2 * b);
                v[2 * u + 1] = ldg_stream(x + 2 * b + 1);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (!ok[u]) continue;
            const uint32_t bm = amax16(v[2 * u], v[2 * u + 1]);
            if (q0 + u < kAmaxChunks) amax_s[(q0 + u) * kChunkBlocks + tid] = (uint16_t)bm;
            m = max(m, bm);
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
        uint32_t cm = 0;
        for (int w = 0; w < kFusedThreads / 32; ++w) cm = max(cm, red[w]);
        atomicMax(gmax_bits, cm);
        __threadfence();
        atomicAdd(arrive, 1u);
        uint32_t spins = 0;
        while (ld_acquire_u32(arrive) < G) {
            if (++spins > spin_limit) {
                atomicExch(status, 1u);
                break;
            }
            __nanosleep(32);
        }
        // ---- global amax: one word, folded in by every CTA before it arrived
        const uint32_t gm = __ldcg(gmax_bits);
        const float gmax = gm > 0x7f80u ? u2f(0x7fc00000u) : fmaxf(u2f(gm << 16), 1.1754943508222875e-38f);
        s_gmax = gmax;
        s_mode = 0;
        if (blockIdx.x == 0) {
            if (gmax_out) *gmax_out = gmax;
            *alpha_out = nvfp4_alpha(gmax);
        }
    }
    __syncthreads();
    Nvfp4Tensor t;
    t.gmax = s_gmax;
    t.alpha = nvfp4_alpha(t.gmax);
    t.markstein = t.gmax >= 0x1p-100f && t.gmax <= 1.0e35f;
    t.yg = t.markstein ? __frcp_rn(t.gmax) : 0.0f;
    {  // 4 lanes per scale byte, one candidate multiplier each
        const uint32_t byte = (uint32_t)(tid >> 2);
        const ScaleEntry e = make_scale_entry(byte < 1 ? 1u : (byte > 126 ? 126u : byte), t.alpha, tid & 3);
        if ((tid & 3) == 0 && byte >= 1 && byte <= 126) {
            table[byte] = e;
            ctab[byte] = e.kind == kCvt ? e.c : -1.0f;
            if (e.kind == kSearch) atomicAdd(&s_mode, 1);  // count of search entries
        }
    }
    __syncthreads();
    // A few kSearch entries: each block follows its own entry (the warps that
    // meet one diverge); many: every block takes the search, uniformly.
    const bool all_search = s_mode > kMaxSearchEntries;

    // ---- phase 2: encode own chunks, last-streamed first (they come from
    //      L2), four blocks per thread loaded together so that their L2
    //      round trips overlap
    for (int q1 = nmine - 1; q1 >= 0; q1 -= 4) {
        uint4 v[8];
        int64_t bb[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            bb[u] = q1 - u >= 0 ? blk(q1 - u) : nblk;
            if (bb[u] < nblk) {
                v[2 * u] = ldg_stream(x + 2 * bb[u]);
                v[2 * u + 1] = ldg_stream(x + 2 * bb[u] + 1);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int q = q1 - u;
            const int64_t b = bb[u];
            if (b >= nblk) continue;
            const uint4 a0 = v[2 * u], a1 = v[2 * u + 1];
            const uint32_t mag = q < kAmaxChunks ? (uint32_t)amax_s[q * kChunkBlocks + tid] : amax16(a0, a1);
            const uint32_t byte = nvfp4_scale_byte(mag, t);
            const float c = all_search ? -1.0f : ctab[byte];
            packed[b] = c > 0.0f ? make_uint2(cvt8_scaled(a0, c), cvt8_scaled(a1, c))
                                 : encode_block(a0, a1, table[byte], all_search);
            int64_t off = b;
            if constexpr (SWZ) {  // with SWZ the host guarantees nblk < 2^31
                const uint32_t r = nb.div((uint32_t)b);
                off = swizzle_offset(r, (int64_t)((uint32_t)b - r * nb.d), c4);
            }
            scale[off] = (uint8_t)byte;
        }
    }

    // ---- leave the grid barrier; the last CTA out re-arms it for the next call
    if (tid == 0 && atomicAdd(depart, 1u) == G - 1) {
        *arrive = 0u;
        *gmax_bits = 0u;
        *depart = 0u;
    }
}

// ---------------------------------------------------------------------------
// Multi-tensor NVFP4 encode with a known global amax (the weights of the QAT
// step, right after the optimizer wrote them): one pass over all tensors,
// work chunks of 512 blocks dealt over the grid, each block encoded exactly
// by nvfp4_block16 (no per-tensor table: consecutive chunks of a CTA belong
// to different tensors), scales written in the GEMM layout, and optionally
// the dequantized copy for the bf16 backward in the same pass.
// ---------------------------------------------------------------------------
constexpr int kEncThreads = 256;
constexpr int kEncPerThread = 4;                              // blocks per thread per chunk, loaded together
constexpr int kEncChunkBlocks = kEncPerThread * kEncThreads;  // 16-element blocks per work chunk
constexpr int kEncGroup = 256;                    // tensors per launch (table in the parameter block)

struct EncGroup {
    int count, pad;
    int64_t chunk0[kEncGroup + 1];  // global chunk index of each tensor's first chunk
    FastDiv nb[kEncGroup];          // k / 16 per tensor
    cdlb200_nvfp4_encode_tensor t[kEncGroup];
};

__device__ __forceinline__ int enc_tensor_of(const EncGroup& g, int64_t c) {
    int lo = 0, hi = g.count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (g.chunk0[mid] <= c) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// bf16((e2m1 * scale) * alpha) of the 8 codes in one word -> one uint4
__device__ __forceinline__ uint4 dequant8(uint32_t codes, float sc, float alpha) {
    uint32_t h[4], o[4];
    e2m1x8_to_f16x2(codes, h);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float lo, hi;
        f16x2_to_f32(h[j], lo, hi);
        o[j] = bf16x2_rn(__fmul_rn(__fmul_rn(lo, sc), alpha), __fmul_rn(__fmul_rn(hi, sc), alpha));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(kEncThreads) nvfp4_encode_multi_kernel(const __grid_constant__ EncGroup g) {
    const int tid = threadIdx.x;
    for (int64_t c = g.chunk0[0] + blockIdx.x; c < g.chunk0[g.count]; c += gridDim.x) {
        const int ti = enc_tensor_of(g, c);
        const cdlb200_nvfp4_encode_tensor& T = g.t[ti];
        const FastDiv nb = g.nb[ti];
        const int64_t nblk = T.rows * (int64_t)nb.d;
        const int64_t c4 = (nb.d + 3) / 4;
        // the tensor's global scale, as the fused quantizer derives it from its amax
        // (up to 64 amax words: two per lane at most, reduced across the warp)
        const int nw = T.amax_words > 1 ? T.amax_words : 1, lane = tid & 31;
        uint32_t gm = lane < nw ? __ldcg(T.amax + lane) : 0u;
        if (lane + 32 < nw) gm = max(gm, __ldcg(T.amax + lane + 32));
        gm = __reduce_max_sync(0xffffffffu, gm);
        Nvfp4Tensor tn;
        tn.gmax = gm > 0x7f80u ? u2f(0x7fc00000u) : fmaxf(u2f(gm << 16), 1.1754943508222875e-38f);
        tn.alpha = nvfp4_alpha(tn.gmax);
        tn.markstein = tn.gmax >= 0x1p-100f && tn.gmax <= 1.0e35f;
        tn.yg = tn.markstein ? __frcp_rn(tn.gmax) : 0.0f;
        if (c == g.chunk0[ti] && tid == 0) *T.alpha = tn.alpha;
        const int64_t base = (c - g.chunk0[ti]) * kEncChunkBlocks;
        const uint4* x = static_cast<const uint4*>(T.x);
        uint4 w[2 * kEncPerThread];
        int64_t b[kEncPerThread];
#pragma unroll
        for (int j = 0; j < kEncPerThread; ++j) {
            b[j] = base + j * kEncThreads + tid;
            if (b[j] < nblk) {
                w[2 * j] = ldg_stream(x + 2 * b[j]);
                w[2 * j + 1] = ldg_stream(x + 2 * b[j] + 1);
            }
        }
#pragma unroll
        for (int j = 0; j < kEncPerThread; ++j) {
            if (b[j] >= nblk) continue;
            uint2 out;
            const uint32_t byte = nvfp4_block16(w[2 * j], w[2 * j + 1], amax16(w[2 * j], w[2 * j + 1]),
                                                tn, out);
            static_cast<uint2*>(T.packed)[b[j]] = out;
            const uint32_t r = nb.div((uint32_t)b[j]);
            static_cast<uint8_t*>(T.scale)[swizzle_offset(r, (int64_t)((uint32_t)b[j] - r * nb.d), c4)] =
                (uint8_t)byte;
            if (T.deq) {
                const float sc = e4m3_to_f32(byte);
                uint4* d = static_cast<uint4*>(T.deq) + 2 * b[j];
                d[0] = dequant8(out.x, sc, tn.alpha);
                d[1] = dequant8(out.y, sc, tn.alpha);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Dual NVFP4 encode: x and x^T from one read of x (the operands of the
// quantized dgrad / wgrad GEMMs).  The tiles of all tensors of a launch form
// one list; a CTA walks its share of it.  Per 64 x 64 tile:
//   * 256 threads load the tile (two 16-byte vectors each, whole 128-byte
//     row segments) and stage it in shared memory; the next tile's loads are
//     issued right after, so they are in flight while this one is encoded;
//   * row-wise: thread (r, b) encodes row r's 16-element block b with the
//     exact block encoder (nvfp4_block16), stores its 8 code bytes (a warp
//     covers whole 32-byte row segments) and the four lanes of a row combine
//     their scale bytes into the one 4-byte word of the 128x4 layout;
//   * column-wise: thread (c, b) gathers column c's 16 values of block b from
//     shared memory (a warp reads 32 consecutive columns of one row per load:
//     conflict-free), encodes them the same way and stages codes and scale
//     bytes, which then leave as one 32-byte segment per output row and one
//     scale word per output row.
// ---------------------------------------------------------------------------
constexpr int kDualT = 64;                  // rows of a work item = columns of a sub-tile
constexpr int kDualW = 2 * kDualT;          // columns of a work item: two 64 x 64 sub-tiles
constexpr int kDualPitch = kDualW + 8;      // staged row: 128 bf16 + 16 bytes of padding
constexpr int kDualThreads = 256;
constexpr int kDualStages = 2;              // items in shared memory: one encoded, one loading
constexpr int kDualGroup = 128;             // tensors per launch (table in the parameter block)

struct DualGroup {
    int count, pad;
    int32_t item0[kDualGroup + 1];  // index of each tensor's first work item in the launch
    FastDiv items_c[kDualGroup];    // ceil(cols / 128)
    cdlb200_nvfp4_dual_tensor t[kDualGroup];
};

__device__ __forceinline__ int dual_tensor_of(const DualGroup& g, int32_t item) {
    int lo = 0, hi = g.count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (g.item0[mid] <= item) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// The tensor's NVFP4 constants from its amax words (warp-wide max) or gmax.
__device__ __forceinline__ Nvfp4Tensor dual_scale(const cdlb200_nvfp4_dual_tensor& T, int lane) {
    float gmax;
    if (T.amax != nullptr) {
        const int nw = T.amax_words > 1 ? T.amax_words : 1;
        uint32_t gm = lane < nw ? __ldcg(T.amax + lane) : 0u;
        if (lane + 32 < nw) gm = max(gm, __ldcg(T.amax + lane + 32));
        gm = __reduce_max_sync(0xffffffffu, gm);
        gmax = gm > 0x7f80u ? u2f(0x7fc00000u) : fmaxf(u2f(gm << 16), 1.1754943508222875e-38f);
    } else {
        gmax = __ldcg(T.gmax);
    }
    Nvfp4Tensor tn;
    tn.gmax = gmax;
    tn.alpha = nvfp4_alpha(gmax);
    tn.markstein = gmax >= 0x1p-100f && gmax <= 1.0e35f;
    tn.yg = tn.markstein ? __frcp_rn(gmax) : 0.0f;
    return tn;
}

struct DualItem {
    int ti;
    int64_t row0, col0;
};

__device__ __forceinline__ DualItem dual_locate(const DualGroup& g, int32_t item) {
    DualItem d;
    d.ti = dual_tensor_of(g, item);
    const uint32_t li = (uint32_t)(item - g.item0[d.ti]);
    const uint32_t ir = g.items_c[d.ti].div(li);
    d.row0 = (int64_t)ir * kDualT;
    d.col0 = (int64_t)(li - ir * g.items_c[d.ti].d) * kDualW;
    return d;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}

// One block with the tensor's scale table (see the fused kernel): the cvt
// multiplier of the block's scale byte when it separates every threshold,
// else the exact search (or the divide); `all_search` when the tensor has
// many search entries, so that the warps do not diverge.
__device__ __forceinline__ uint32_t table_block16(const uint4& a0, const uint4& a1, const Nvfp4Tensor& tn,
                                                  const ScaleEntry* table, const float* ctab, bool all_search,
                                                  uint2& out) {
    const uint32_t byte = nvfp4_scale_byte(amax16(a0, a1), tn) & 127u;
    const float c = all_search ? -1.0f : ctab[byte];
    if (c > 0.0f) {
        out.x = cvt8_scaled(a0, c);
        out.y = cvt8_scaled(a1, c);
    } else {
        out = encode_block(a0, a1, table[byte], all_search);
    }
    return byte;
}

// One column block of a staged tile: v[i] holds row i of columns 2p (low
// half) and 2p + 1 (high half); HI picks the column, `mag` is its block amax.
// Same encoding as table_block16; only the rare table paths regroup the
// halves into pairs.
template <bool HI>
__device__ __forceinline__ uint32_t table_col16(const uint32_t (&v)[16], uint32_t mag, const Nvfp4Tensor& tn,
                                                const ScaleEntry* table, const float* ctab, bool all_search,
                                                uint2& out) {
    const uint32_t byte = nvfp4_scale_byte(mag, tn) & 127u;
    const float c = all_search ? -1.0f : ctab[byte];
    if (c > 0.0f) {
        out.x = cvt8_halves_scaled<HI>(v, c);
        out.y = cvt8_halves_scaled<HI>(v + 8, c);
    } else {
        uint32_t e[8];  // rows (2i, 2i + 1) of the column
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = __byte_perm(v[2 * i], v[2 * i + 1], HI ? 0x7632 : 0x5410);
        out = encode_block(make_uint4(e[0], e[1], e[2], e[3]), make_uint4(e[4], e[5], e[6], e[7]), table[byte],
                           all_search);
    }
    return byte;
}

__global__ void __launch_bounds__(kDualThreads, 4) nvfp4_dual_multi_kernel(const __grid_constant__ DualGroup g) {
    extern __shared__ __align__(16) uint8_t dual_smem[];
    __shared__ ScaleEntry table[128];
    __shared__ float ctab[128];  // the cvt multiplier of a kCvt entry, else -1
    __shared__ int s_search;     // count of kSearch entries
    uint16_t* xs0 = reinterpret_cast<uint16_t*>(dual_smem);  // kDualStages items of kDualT x kDualPitch
    // staged column codes [h][b][c] (sub-tile h, block b, column c) and scale bytes [h][4c + b]
    uint2* ccodes = reinterpret_cast<uint2*>(dual_smem + kDualStages * kDualT * kDualPitch * 2);
    uint8_t* cscale = reinterpret_cast<uint8_t*>(ccodes + 2 * 4 * kDualT);
    const int tid = threadIdx.x, lane = tid & 31;
    const int32_t total = g.item0[g.count];
    const int32_t first = (int32_t)blockIdx.x, stride = (int32_t)gridDim.x;

    // copies of item `item` into stage `s`: four 16-byte pieces per thread,
    // whole 128-byte row segments per 8 lanes (a missing second sub-tile is
    // not loaded)
    auto issue = [&](int32_t item, const DualItem& d, int s) {
        if (item < total) {
            const cdlb200_nvfp4_dual_tensor& T = g.t[d.ti];
            const uint16_t* x = static_cast<const uint16_t*>(T.x) + d.row0 * T.cols + d.col0;
            const int ncols = T.cols - d.col0 < kDualW ? kDualT : kDualW;
            uint16_t* xs = xs0 + s * (kDualT * kDualPitch);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int e = tid + kDualThreads * j, r = e >> 4, c8 = (e & 15) * 8;
                if (c8 < ncols) cp_async16(&xs[r * kDualPitch + c8], x + r * T.cols + c8);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    // each item is located once, when its copies are issued, and kept for
    // its encode in the next iteration
    DualItem dnext{};
    if (first < total) dnext = dual_locate(g, first);
    issue(first, dnext, 0);
    int k = 0, cur_ti = -1;
    Nvfp4Tensor tn;
    bool all_search = false;
    for (int32_t item = first; item < total; item += stride, ++k) {
        const DualItem d = dnext;
        if (item + stride < total) dnext = dual_locate(g, item + stride);
        issue(item + stride, dnext, (k + 1) % kDualStages);
        asm volatile("cp.async.wait_group 1;" ::: "memory");  // this thread's copies of `item` landed
        __syncthreads();                                      // ... and every other thread's
        const uint16_t* xs = xs0 + (k % kDualStages) * (kDualT * kDualPitch);
        const cdlb200_nvfp4_dual_tensor& T = g.t[d.ti];
        const int64_t row0 = d.row0, col0 = d.col0;
        const int nsub = T.cols - col0 < kDualW ? 1 : 2;  // sub-tiles of this item
        if (d.ti != cur_ti) {  // the tensor's constants and scale table, once per tensor a CTA meets
            tn = dual_scale(T, lane);
            cur_ti = d.ti;
            if (tid == 0) s_search = 0;
            __syncthreads();  // the previous table is no longer read
#pragma unroll
            for (int half = 0; half < 2; ++half) {  // 4 lanes per scale byte, one candidate multiplier each
                const uint32_t byte = (uint32_t)((tid >> 2) + 64 * half);
                const ScaleEntry e = make_scale_entry(byte < 1 ? 1u : (byte > 126 ? 126u : byte), tn.alpha, tid & 3);
                if ((tid & 3) == 0) {
                    table[byte] = e;
                    ctab[byte] = e.kind == kCvt ? e.c : -1.0f;
                    if (e.kind == kSearch && byte >= 1 && byte <= 126) atomicAdd(&s_search, 1);
                }
            }
            __syncthreads();
            all_search = s_search > kMaxSearchEntries;
        }
        if (item == g.item0[d.ti] && tid == 0) *T.alpha = tn.alpha;

        if (tid < 128) {
            // ---- x, warps 0-3: row r of sub-tile h, its four blocks (64 contiguous values)
            const int r = tid >> 1, h = tid & 1;
            if (T.row_packed != nullptr && h < nsub) {
                const uint16_t* src = &xs[r * kDualPitch + kDualT * h];
                uint32_t word = 0;
                uint2 o[4];
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint4 w0 = *reinterpret_cast<const uint4*>(src + 16 * b);
                    const uint4 w1 = *reinterpret_cast<const uint4*>(src + 16 * b + 8);
                    word |= table_block16(w0, w1, tn, table, ctab, all_search, o[b]) << (8 * b);
                }
                uint8_t* dst = static_cast<uint8_t*>(T.row_packed) + (row0 + r) * (T.cols / 2) + col0 / 2 + 32 * h;
                *reinterpret_cast<uint4*>(dst) = make_uint4(o[0].x, o[0].y, o[1].x, o[1].y);
                *reinterpret_cast<uint4*>(dst + 16) = make_uint4(o[2].x, o[2].y, o[3].x, o[3].y);
                const int64_t so = (T.flags & CDLB200_DUAL_ROW_LINEAR)
                                       ? (row0 + r) * (T.cols / 16) + (col0 + kDualT * h) / 16
                                       : swizzle_offset(row0 + r, (col0 + kDualT * h) / 16, T.cols / 64);
                *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(T.row_scale) + so) = word;
            }
        } else if (T.col_packed != nullptr) {
            // ---- x^T, warps 4-7: columns 2p and 2p + 1 of each sub-tile, block b (tile rows 16b .. 16b + 15);
            // one 32-bit load holds both columns' values of a row
            const int t = tid - 128, p = t & 31, b = t >> 5;
            for (int h = 0; h < nsub; ++h) {
                const uint32_t* src = reinterpret_cast<const uint32_t*>(&xs[16 * b * kDualPitch + kDualT * h + 2 * p]);
                uint32_t v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = src[i * (kDualPitch / 2)];
                // both columns' block amax at once: the low / high halves of a pairwise tree
                uint32_t m[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) m[i] = absmax2(v[2 * i], v[2 * i + 1]);
#pragma unroll
                for (int i = 0; i < 4; ++i) m[i] = absmax2(m[2 * i], m[2 * i + 1]);
                const uint32_t mm = absmax2(absmax2(m[0], m[1]), absmax2(m[2], m[3])) & 0x7fff7fffu;
                uint2 ce, co;
                const uint32_t se = table_col16<false>(v, mm & 0xffffu, tn, table, ctab, all_search, ce);
                const uint32_t so = table_col16<true>(v, mm >> 16, tn, table, ctab, all_search, co);
                *reinterpret_cast<uint4*>(&ccodes[(4 * h + b) * kDualT + 2 * p]) = make_uint4(ce.x, ce.y, co.x, co.y);
                cscale[256 * h + 4 * (2 * p) + b] = (uint8_t)se;
                cscale[256 * h + 4 * (2 * p + 1) + b] = (uint8_t)so;
            }
        }
        __syncthreads();  // staged columns complete; the stage is free for the copies issued next
        if (T.col_packed != nullptr) {
            {  // output row col0 + 64h + c: 32 code bytes, blocks (2q, 2q + 1) per half q
                const int h = tid >> 7, c = (tid >> 1) & 63, qh = tid & 1;
                if (h < nsub) {
                    const uint2 q0 = ccodes[(4 * h + 2 * qh) * kDualT + c], q1 = ccodes[(4 * h + 2 * qh + 1) * kDualT + c];
                    *reinterpret_cast<uint4*>(static_cast<uint8_t*>(T.col_packed) +
                                              (col0 + kDualT * h + c) * (T.rows / 2) + row0 / 2 + 16 * qh) =
                        make_uint4(q0.x, q0.y, q1.x, q1.y);
                }
            }
            if (tid < 2 * kDualT) {  // its scale word (blocks row0/16 .. +3)
                const int h = tid >> 6, c = tid & 63;
                if (h < nsub) {
                    const int64_t so = (T.flags & CDLB200_DUAL_COL_LINEAR)
                                           ? (col0 + kDualT * h + c) * (T.rows / 16) + row0 / 16
                                           : swizzle_offset(col0 + kDualT * h + c, row0 / 16, T.rows / 64);
                    *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(T.col_scale) + so) =
                        *reinterpret_cast<const uint32_t*>(&cscale[256 * h + 4 * c]);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

constexpr int kDualSmem = kDualStages * kDualT * kDualPitch * 2 + 2 * kDualT * 4 * 8 + 2 * kDualT * 4;

// ---------------------------------------------------------------------------
// general path: any leading dimension, ragged k, transposed (dim-0) blocks.
// One thread per (output row r, block b); element (r, c) is x[r*sr + c*sc].
// Threads are ordered r-fastest so a transposed input is read coalesced.
// ---------------------------------------------------------------------------
template <int FMT, bool SWZ>
__global__ void __launch_bounds__(256) quant_strided_kernel(const uint16_t* __restrict__ x, int64_t R,
                                                            int64_t C, int64_t sr, int64_t sc,
                                                            uint8_t* __restrict__ packed,
                                                            int64_t pstride,
                                                            uint8_t* __restrict__ scale, int64_t nb,
                                                            int64_t c4,
                                                            const float* __restrict__ gmax_p,
                                                            const float* __restrict__ alpha_p) {
    constexpr int B = FmtTraits<FMT>::kBlock;
    float gmax = 0.f, alpha = 0.f;
    if constexpr (FMT == kNVFP4) {
        gmax = *gmax_p;
        alpha = *alpha_p;
    }
    const int64_t total = R * nb;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx % R, b = idx / R;
        uint32_t h[B];
        uint32_t mag = 0;
#pragma unroll
        for (int i = 0; i < B; ++i) {
            const int64_t c = b * B + i;
            h[i] = c < C ? (uint32_t)x[r * sr + c * sc] : 0u;
            mag = max(mag, h[i] & 0x7fffu);
        }
        BlockCode bc;
        block_setup<FMT>(mag, gmax, alpha, bc);
        uint8_t* prow = packed + r * pstride;
        if constexpr (FmtTraits<FMT>::kFp4) {
#pragma unroll
            for (int i = 0; i < B; i += 2)
                prow[(b * B + i) / 2] = (uint8_t)(e2m1_nibble(h[i], bc) | (e2m1_nibble(h[i + 1], bc) << 4));
        } else {
#pragma unroll
            for (int i = 0; i < B; i += 2) {
                uint32_t p = cvt_e4m3x2(__fmul_rn(u2f(h[i + 1] << 16), bc.s), __fmul_rn(u2f(h[i] << 16), bc.s));
                prow[b * B + i] = (uint8_t)(p & 0xffu);
                prow[b * B + i + 1] = (uint8_t)(p >> 8);
            }
        }
        const int64_t off = SWZ ? swizzle_offset(r, b, c4) : r * nb + b;
        scale[off] = (uint8_t)bc.byte;
    }
}

// ---------------------------------------------------------------------------
// transposed path (the wgrad requantize): blocks run along dim 0 of x[rows, k],
// output row r is input column r.  A CTA stages a [TR x 64] tile of x in
// shared memory with coalesced 16-byte loads, encodes one (column, block) pair
// per thread from the shared-memory columns, collects the codes of its 64
// output rows in shared memory and writes each row's segment contiguously.
// TR = 256 input rows for FP4 (16 NVFP4 / 8 MXFP4 blocks), 128 for MXFP8
// (4 blocks): 128 output bytes per row and tile either way.
// ---------------------------------------------------------------------------
constexpr int kTrCols = 64, kTrPitch = kTrCols + 8;  // staged row: 64 bf16 + 16 bytes of padding
template <int FMT>
struct TrTile {
    static constexpr int kRows = FmtTraits<FMT>::kFp4 ? 256 : 128;
    static constexpr int kBlocks = kRows / FmtTraits<FMT>::kBlock;
    static constexpr int kOutBytes = 128;  // codes per output row and tile
};

template <int FMT, bool SWZ>
__global__ void __launch_bounds__(256) quant_transpose_kernel(const uint16_t* __restrict__ x, int64_t rows, int64_t k,
                                                              int64_t ldx, uint8_t* __restrict__ packed,
                                                              int64_t pstride, uint8_t* __restrict__ scale,
                                                              int64_t nb, int64_t c4, const float* __restrict__ gmax_p,
                                                              const float* __restrict__ alpha_p) {
    using G = TrTile<FMT>;
    constexpr int B = FmtTraits<FMT>::kBlock, TR = G::kRows, NBT = G::kBlocks;
    constexpr int BB = FmtTraits<FMT>::kFp4 ? B / 2 : B;  // code bytes per block
    __shared__ __align__(16) uint16_t xs[TR * kTrPitch];
    __shared__ __align__(16) uint8_t os[kTrCols * (G::kOutBytes + 16)];
    constexpr int kOutPitch = G::kOutBytes + 16;
    float gmax = 0.f, alpha = 0.f;
    if constexpr (FMT == kNVFP4) {
        gmax = *gmax_p;
        alpha = *alpha_p;
    }
    const int tid = threadIdx.x;
    const int64_t tiles_c = (k + kTrCols - 1) / kTrCols, tiles_r = (rows + TR - 1) / TR;
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (ldx & 7) == 0;
    for (int64_t tile = blockIdx.x; tile < tiles_c * tiles_r; tile += gridDim.x) {
        const int64_t col0 = (tile % tiles_c) * kTrCols, row0 = (tile / tiles_c) * TR;
        // ---- stage x[row0 .. +TR, col0 .. +64) (zeros outside x)
        for (int e = tid; e < TR * (kTrCols / 8); e += 256) {
            const int r = e >> 3, c8 = (e & 7) * 8;
            const int64_t gr = row0 + r, gc = col0 + c8;
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (gr < rows) {
                const uint16_t* src = x + gr * ldx + gc;
                if (vec && gc + 8 <= k) {
                    v = ldg_stream(src);
                } else {
                    uint16_t h[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) h[i] = gc + i < k ? src[i] : (uint16_t)0;
                    v = make_uint4(h[0] | (uint32_t)h[1] << 16, h[2] | (uint32_t)h[3] << 16, h[4] | (uint32_t)h[5] << 16,
                                   h[6] | (uint32_t)h[7] << 16);
                }
            }
            *reinterpret_cast<uint4*>(&xs[r * kTrPitch + c8]) = v;
        }
        __syncthreads();
        // ---- encode: thread (j, b) = column col0 + j, block b of this tile (a warp shares b)
        for (int p = tid; p < kTrCols * NBT; p += 256) {
            const int j = p % kTrCols, b = p / kTrCols;
            uint32_t h[B];
            uint32_t mag = 0;
#pragma unroll
            for (int i = 0; i < B; ++i) {
                h[i] = xs[(b * B + i) * kTrPitch + j];
                mag = max(mag, h[i] & 0x7fffu);
            }
            BlockCode bc;
            block_setup<FMT>(mag, gmax, alpha, bc);
            uint8_t* o = os + j * kOutPitch + b * BB;
            if constexpr (FmtTraits<FMT>::kFp4) {
#pragma unroll
                for (int i = 0; i < B; i += 2)
                    o[i / 2] = (uint8_t)(e2m1_nibble(h[i], bc) | (e2m1_nibble(h[i + 1], bc) << 4));
            } else {
#pragma unroll
                for (int i = 0; i < B; i += 2) {
                    const uint32_t q2 =
                        cvt_e4m3x2(__fmul_rn(u2f(h[i + 1] << 16), bc.s), __fmul_rn(u2f(h[i] << 16), bc.s));
                    o[i] = (uint8_t)(q2 & 0xffu);
                    o[i + 1] = (uint8_t)(q2 >> 8);
                }
            }
            const int64_t r_out = col0 + j, blk = row0 / B + b;
            if (r_out < k && blk < nb) scale[SWZ ? swizzle_offset(r_out, blk, c4) : r_out * nb + blk] = (uint8_t)bc.byte;
        }
        __syncthreads();
        // ---- write each output row's segment: blocks row0/B .. (clipped to nb)
        const int64_t blk0 = row0 / B;
        const int nbytes = (int)((nb - blk0 < NBT ? nb - blk0 : NBT) * BB);
        for (int e = tid; e < kTrCols * (G::kOutBytes / 8); e += 256) {
            const int j = e / (G::kOutBytes / 8), o8 = (e % (G::kOutBytes / 8)) * 8;
            const int64_t r_out = col0 + j;
            if (r_out >= k || o8 >= nbytes) continue;
            uint8_t* dst = packed + r_out * pstride + blk0 * BB + o8;
            const uint8_t* srcb = os + j * kOutPitch + o8;
            if (o8 + 8 <= nbytes && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
                *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(srcb);
            } else {
                for (int i = 0; i < 8 && o8 + i < nbytes; ++i) dst[i] = srcb[i];
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// MX transposed (dim-0) quantize of a contiguous x[rows, k] with rows % 64 == 0
// and k % 128 == 0: output row c holds column c's blocks of 32 values.  A
// work item is a 64 x 128 tile staged by cp.async (two stages: the next
// tile loads while this one is encoded); thread t takes columns 2p, 2p + 1
// (p = t & 63) of block b = t >> 6: 32 shared-memory words, each holding both
// columns' values of one row, split with byte permutes into the two columns'
// packed pairs, then the block is encoded as the row-wise MX path encodes it
// (hardware conversion of x * 2^-e, nudged for MXFP4) and stored straight
// from registers: 16 (MXFP4) or 32 (MXFP8) bytes per column block.
// ---------------------------------------------------------------------------
constexpr int kMxcR = 64, kMxcC = 128, kMxcPitch = kMxcC + 8;  // staged row: 128 bf16 + 16 bytes of padding

template <int FMT, bool SWZ>
__device__ __forceinline__ void mx_col_block(const uint32_t (&w)[16], int64_t col, int64_t blk, uint8_t* packed,
                                             int64_t pstride, uint8_t* scale, int64_t nb, int64_t c4) {
    const uint32_t M = 0x7fff7fffu;
    uint32_t m = w[0] & M;
#pragma unroll
    for (int i = 1; i < 16; ++i) asm("max.u16x2 %0, %1, %2;" : "=r"(m) : "r"(m), "r"(w[i] & M));
    const uint32_t byte = e8m0_byte_from_bf16_mag<FmtTraits<FMT>::kEmax>(max(m & 0xffffu, m >> 16));
    if constexpr (FMT == kMXFP4) {
        const float c = __fmul_rn(e8m0_inv(byte), 0.99999904632568359375f);  // 2^-e (1 - 2^-20)
        uint32_t q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = cvt8_scaled(make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]), c);
        *reinterpret_cast<uint4*>(packed + col * pstride + blk * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    } else {
        BlockCode bc;
        bc.s = e8m0_inv(byte);  // RN(x / 2^e) == x * 2^-e exactly
        uint2 q[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) q[j] = encode8_fp8(make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]), bc);
        uint4* dst = reinterpret_cast<uint4*>(packed + col * pstride + blk * 32);
        dst[0] = make_uint4(q[0].x, q[0].y, q[1].x, q[1].y);
        dst[1] = make_uint4(q[2].x, q[2].y, q[3].x, q[3].y);
    }
    scale[SWZ ? swizzle_offset(col, blk, c4) : col * nb + blk] = (uint8_t)byte;
}

template <int FMT, bool SWZ>
__global__ void __launch_bounds__(128) mx_col_kernel(const uint16_t* __restrict__ x, int64_t rows, int64_t k,
                                                     uint8_t* __restrict__ packed, int64_t pstride,
                                                     uint8_t* __restrict__ scale, int64_t nb, int64_t c4) {
    __shared__ __align__(16) uint16_t xs[2][kMxcR * kMxcPitch];
    const int tid = threadIdx.x;
    const int64_t tiles_c = k / kMxcC, tiles = (rows / kMxcR) * tiles_c;
    auto issue = [&](int64_t tile, int s) {
        if (tile < tiles) {
            const int64_t r0 = (tile / tiles_c) * kMxcR, c0 = (tile % tiles_c) * kMxcC;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int e = tid + 128 * j, r = e >> 4, c8 = (e & 15) * 8;
                cp_async16(&xs[s][r * kMxcPitch + c8], x + (r0 + r) * k + c0 + c8);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(blockIdx.x, 0);
    int it = 0;
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
        issue(tile + gridDim.x, (it + 1) & 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        const int64_t r0 = (tile / tiles_c) * kMxcR, c0 = (tile % tiles_c) * kMxcC;
        const int p = tid & 63, b = tid >> 6;
        const uint32_t* src = reinterpret_cast<const uint32_t*>(&xs[it & 1][32 * b * kMxcPitch + 2 * p]);
        uint32_t e[16], o[16];  // columns 2p / 2p + 1, rows (2i, 2i + 1) of the block
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint32_t v0 = src[(2 * i) * (kMxcPitch / 2)], v1 = src[(2 * i + 1) * (kMxcPitch / 2)];
            e[i] = __byte_perm(v0, v1, 0x5410);
            o[i] = __byte_perm(v0, v1, 0x7632);
        }
        const int64_t blk = r0 / 32 + b;
        mx_col_block<FMT, SWZ>(e, c0 + 2 * p, blk, packed, pstride, scale, nb, c4);
        mx_col_block<FMT, SWZ>(o, c0 + 2 * p + 1, blk, packed, pstride, scale, nb, c4);
        __syncthreads();  // the stage is free for the copies issued next
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(a - 1)) == 0; }

int device_ok() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CDLB200_ERR_CUDA;
    static int cc_major[128] = {0};
    if (dev < 0 || dev >= 128) return CDLB200_ERR_CUDA;
    if (cc_major[dev] == 0) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
            return CDLB200_ERR_CUDA;
        cc_major[dev] = major;
    }
    return cc_major[dev] == 10 ? CDLB200_OK : CDLB200_ERR_UNSUPPORTED;
}

template <int FMT, bool SWZ>
int launch_encode(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose, void* packed,
                  void* scale, const float* gmax, const float* alpha, cudaStream_t st) {
    constexpr int B = FmtTraits<FMT>::kBlock;
    const int64_t R = transpose ? k : rows, C = transpose ? rows : k;
    const int64_t nb = (C + B - 1) / B;
    const int64_t c4 = (nb + 3) / 4;
    const int64_t pstride = FmtTraits<FMT>::kFp4 ? nb * B / 2 : nb * B;
    const int sms = num_sms();
    // the flat kernels locate a swizzled scale with 32-bit block indices
    const bool flat = !transpose && ldx == k && (k % B) == 0 && aligned(x, 16) &&
                      aligned(packed, (FmtTraits<FMT>::kFp4 && FMT != kNVFP4) ? 4 : 8) &&
                      (!SWZ || rows * nb < (1ll << 31));
    const FastDiv nbd((uint32_t)(nb < (1ll << 31) ? nb : 1));
    if (flat && FMT == kNVFP4) {
        constexpr int U = 2;
        const int64_t nblk = rows * k / 16;
        int64_t grid = (nblk + 256 * U - 1) / (256 * U);
        grid = grid < (int64_t)sms * 8 ? grid : (int64_t)sms * 8;
        nvfp4_flat_kernel<SWZ, U><<<(unsigned)grid, 256, 0, st>>>(
            reinterpret_cast<const uint4*>(x), nblk, static_cast<uint2*>(packed),
            static_cast<uint8_t*>(scale), nbd, c4, gmax, alpha);
    } else if (flat) {
        constexpr int U = 4;
        const int64_t nvec = rows * k / 8;
        int64_t grid = (nvec + 256 * U - 1) / (256 * U);
        grid = grid < (int64_t)sms * 8 ? grid : (int64_t)sms * 8;
        quant_flat_kernel<FMT, SWZ, U><<<(unsigned)grid, 256, 0, st>>>(
            reinterpret_cast<const uint4*>(x), nvec, static_cast<uint8_t*>(packed),
            static_cast<uint8_t*>(scale), nbd, c4, gmax, alpha);
    } else if (transpose && FMT != kNVFP4 && ldx == k && (rows % kMxcR) == 0 && (k % kMxcC) == 0 &&
               aligned(x, 16) && aligned(packed, 16)) {
        const int64_t tiles = (rows / kMxcR) * (k / kMxcC);
        int64_t grid = tiles < (int64_t)sms * 6 ? tiles : (int64_t)sms * 6;
        mx_col_kernel<FMT, SWZ><<<(unsigned)grid, 128, 0, st>>>(static_cast<const uint16_t*>(x), rows, k,
                                                                static_cast<uint8_t*>(packed), pstride,
                                                                static_cast<uint8_t*>(scale), nb, c4);
    } else if (transpose) {
        const int64_t tiles = ((k + kTrCols - 1) / kTrCols) * ((rows + TrTile<FMT>::kRows - 1) / TrTile<FMT>::kRows);
        int64_t grid = tiles < (int64_t)sms * 4 ? tiles : (int64_t)sms * 4;
        quant_transpose_kernel<FMT, SWZ><<<(unsigned)grid, 256, 0, st>>>(
            static_cast<const uint16_t*>(x), rows, k, ldx, static_cast<uint8_t*>(packed), pstride,
            static_cast<uint8_t*>(scale), nb, c4, gmax, alpha);
    } else {
        const int64_t sr = transpose ? 1 : ldx, sc = transpose ? ldx : 1;
        int64_t grid = (R * nb + 255) / 256;
        grid = grid < (int64_t)sms * 16 ? grid : (int64_t)sms * 16;
        quant_strided_kernel<FMT, SWZ><<<(unsigned)grid, 256, 0, st>>>(
            static_cast<const uint16_t*>(x), R, C, sr, sc, static_cast<uint8_t*>(packed), pstride,
            static_cast<uint8_t*>(scale), nb, c4, gmax, alpha);
    }
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

template <int FMT>
int quant_entry(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose, void* packed,
                void* scale, int scale_layout, const float* gmax, const float* alpha, cudaStream_t st) {
    constexpr int B = FmtTraits<FMT>::kBlock;
    if (scale_layout == CDLB200_SCALE_SWIZZLED) {
        const int64_t R = transpose ? k : rows, C = transpose ? rows : k;
        const int64_t nb = (C + B - 1) / B;
        if ((R % 128) != 0 || (nb % 4) != 0) {
            const size_t bytes = (size_t)((R + 127) / 128 * 128) * (size_t)((nb + 3) / 4 * 4);
            if (cudaMemsetAsync(scale, 0, bytes, st) != cudaSuccess) return CDLB200_ERR_CUDA;
        }
        return launch_encode<FMT, true>(x, rows, k, ldx, transpose, packed, scale, gmax, alpha, st);
    }
    return launch_encode<FMT, false>(x, rows, k, ldx, transpose, packed, scale, gmax, alpha, st);
}

int check_args(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose, const void* packed,
               const void* scale, int scale_layout) {
    if (rows < 0 || k < 0) return CDLB200_ERR_INVALID_ARG;
    if (transpose != 0 && transpose != 1) return CDLB200_ERR_INVALID_ARG;
    if (scale_layout != CDLB200_SCALE_LINEAR && scale_layout != CDLB200_SCALE_SWIZZLED)
        return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || k == 0) return CDLB200_OK;
    if (!x || !packed || !scale) return CDLB200_ERR_INVALID_ARG;
    if (ldx < k) return CDLB200_ERR_INVALID_ARG;
    if (!aligned(x, 2)) return CDLB200_ERR_ALIGNMENT;
    return CDLB200_OK;
}

}  // namespace

// Launches the global amax reduction; shared with the no-workspace variants.
int launch_amax(const void* x, int64_t rows, int64_t k, int64_t ldx, uint32_t* partial,
                uint32_t* counter, float* gmax, float* alpha, cudaStream_t st) {
    if (rows == 0 || k == 0) {
        empty_alpha_kernel<<<1, 1, 0, st>>>(gmax, alpha);
        CDLB200_CHECK_LAUNCH();
        return CDLB200_OK;
    }
    const int sms = num_sms();
    const int vec_ok = ldx == k && aligned(x, 16);
    int64_t want = vec_ok ? (rows * k / 8 + 512 * 4 - 1) / (512 * 4) : rows;
    int64_t cap = (int64_t)sms * 2 < kMaxAmaxGrid ? (int64_t)sms * 2 : kMaxAmaxGrid;
    int grid = (int)(want < 1 ? 1 : (want < cap ? want : cap));
    amax_kernel<<<grid, 512, 0, st>>>(static_cast<const uint16_t*>(x), rows, k, ldx, vec_ok, partial,
                                      counter, gmax, alpha);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

namespace {

template <bool SWZ>
int launch_fused_impl(const void* x, int64_t rows, int64_t k, void* packed, void* scale, float* gmax,
                      float* alpha, uint8_t* ws, cudaStream_t st) {
    static int occ_cache[128][2] = {{0}};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return CDLB200_ERR_CUDA;
    int& per_sm = occ_cache[dev][SWZ ? 1 : 0];
    if (per_sm == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, nvfp4_fused_kernel<SWZ>, kFusedThreads, 0) !=
                cudaSuccess || n < 1)
            return CDLB200_ERR_CUDA;
        per_sm = n > 2 ? 2 : n;
    }
    const int64_t nblk = rows * k / 16;
    const int64_t nchunk = (nblk + kChunkBlocks - 1) / kChunkBlocks;
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > kMaxAmaxGrid) grid = kMaxAmaxGrid;
    if (grid > nchunk) grid = nchunk;
    const int64_t nb = k / 16, c4 = (nb + 3) / 4;
    if (SWZ && nblk >= (1ll << 31)) return CDLB200_ERR_INVALID_ARG;
    const FastDiv nbd((uint32_t)(nb < (1ll << 31) ? nb : 1));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident, or the launch fails
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, nvfp4_fused_kernel<SWZ>, reinterpret_cast<const uint4*>(x),
                                             nblk, static_cast<uint2*>(packed), static_cast<uint8_t*>(scale),
                                             nbd, c4, ws, gmax, alpha, wait_limit());
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return CDLB200_ERR_LAUNCH;
    }
    return CDLB200_OK;
}

}  // namespace

// Fused single-launch NVFP4 quantize of a contiguous, 16-byte aligned bf16
// matrix with k % 16 == 0 (row-wise blocks).
int launch_nvfp4_fused(const void* x, int64_t rows, int64_t k, void* packed, void* scale,
                       int scale_layout, float* gmax, float* alpha, uint8_t* ws, cudaStream_t st) {
    if (scale_layout == CDLB200_SCALE_SWIZZLED) {
        const int64_t nb = k / 16;
        if ((rows % 128) != 0 || (nb % 4) != 0) {
            const size_t bytes = (size_t)((rows + 127) / 128 * 128) * (size_t)((nb + 3) / 4 * 4);
            if (cudaMemsetAsync(scale, 0, bytes, st) != cudaSuccess) return CDLB200_ERR_CUDA;
        }
        return launch_fused_impl<true>(x, rows, k, packed, scale, gmax, alpha, ws, st);
    }
    return launch_fused_impl<false>(x, rows, k, packed, scale, gmax, alpha, ws, st);
}

int launch_nvfp4_encode(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                        void* packed, void* scale, int scale_layout, const float* gmax,
                        const float* alpha, cudaStream_t st) {
    return quant_entry<kNVFP4>(x, rows, k, ldx, transpose, packed, scale, scale_layout, gmax, alpha,
                               st);
}

}  // namespace cdlb200

namespace cdlb200 {
namespace {
// Launches the dual NVFP4 encoder over validated tensors (defined with its
// entry point, cdlb200_nvfp4_dual_multi).
int launch_dual(const cdlb200_nvfp4_dual_tensor* tensors, int count, cudaStream_t st);
}  // namespace
}  // namespace cdlb200

using namespace cdlb200;

extern "C" size_t cdlb200_nvfp4_quant_workspace_bytes(int64_t, int64_t) {
    return (size_t)kWsPartialOff + sizeof(uint32_t) * kMaxAmaxGrid + sizeof(float);
}

extern "C" int cdlb200_nvfp4_quant(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                                   void* packed, void* scale, int scale_layout, float* gmax,
                                   float* alpha, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    int rc = check_args(x, rows, k, ldx, transpose, packed, scale, scale_layout);
    if (rc != CDLB200_OK) return rc;
    if (!alpha) return CDLB200_ERR_INVALID_ARG;
    if (!workspace || workspace_bytes < cdlb200_nvfp4_quant_workspace_bytes(rows, k))
        return CDLB200_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return CDLB200_ERR_ALIGNMENT;
    if ((rc = device_ok()) != CDLB200_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint32_t* counter = reinterpret_cast<uint32_t*>(ws + kWsCounterOff);
    uint32_t* partial = reinterpret_cast<uint32_t*>(ws + kWsPartialOff);
    // gmax goes to the caller's buffer if given, else to the workspace tail
    float* g = gmax ? gmax : reinterpret_cast<float*>(ws + kWsPartialOff + sizeof(uint32_t) * kMaxAmaxGrid);
    if (!transpose && rows > 0 && k > 0 && ldx == k && (k % 16) == 0 && aligned(x, 16) && aligned(packed, 8))
        return launch_nvfp4_fused(x, rows, k, packed, scale, scale_layout, gmax, alpha, ws, st);
    rc = launch_amax(x, rows, k, ldx, partial, counter, g, alpha, st);
    if (rc != CDLB200_OK || rows == 0 || k == 0) return rc;
    if (transpose && ldx == k && (rows % 64) == 0 && (k % 64) == 0 && aligned(x, 16) && aligned(packed, 16) &&
        aligned(scale, 4) && (rows / 64) * ((k + 127) / 128) < (1ll << 31)) {
        // the transposed encode of the dual encoder (its column pass alone):
        // x is staged in shared memory tile by tile and each column block
        // encoded from there
        cdlb200_nvfp4_dual_tensor t{};
        t.x = x;
        t.rows = rows;
        t.cols = k;
        t.gmax = g;
        t.alpha = alpha;
        t.col_packed = packed;
        t.col_scale = scale;
        t.flags = scale_layout == CDLB200_SCALE_SWIZZLED ? 0 : CDLB200_DUAL_COL_LINEAR;
        return launch_dual(&t, 1, st);
    }
    return launch_nvfp4_encode(x, rows, k, ldx, transpose, packed, scale, scale_layout, g, alpha, st);
}

extern "C" int cdlb200_nvfp4_amax(const void* x, int64_t rows, int64_t k, int64_t ldx, float* gmax, float* alpha,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    if (rows < 0 || k < 0 || !gmax || !alpha) return CDLB200_ERR_INVALID_ARG;
    if (rows > 0 && k > 0 && (!x || ldx < k)) return CDLB200_ERR_INVALID_ARG;
    if (x && !aligned(x, 2)) return CDLB200_ERR_ALIGNMENT;
    if (!workspace || workspace_bytes < cdlb200_nvfp4_quant_workspace_bytes(rows, k)) return CDLB200_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return CDLB200_ERR_ALIGNMENT;
    int rc;
    if ((rc = device_ok()) != CDLB200_OK) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    return launch_amax(x, rows, k, ldx, reinterpret_cast<uint32_t*>(ws + kWsPartialOff),
                       reinterpret_cast<uint32_t*>(ws + kWsCounterOff), gmax, alpha, static_cast<cudaStream_t>(stream));
}

extern "C" int cdlb200_mxfp4_quant(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                                   void* packed, void* scale, int scale_layout, void* stream) {
    int rc = check_args(x, rows, k, ldx, transpose, packed, scale, scale_layout);
    if (rc != CDLB200_OK || rows == 0 || k == 0) return rc;
    if ((rc = device_ok()) != CDLB200_OK) return rc;
    return quant_entry<kMXFP4>(x, rows, k, ldx, transpose, packed, scale, scale_layout, nullptr,
                               nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int cdlb200_mxfp8_quant(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                                   void* packed, void* scale, int scale_layout, void* stream) {
    int rc = check_args(x, rows, k, ldx, transpose, packed, scale, scale_layout);
    if (rc != CDLB200_OK || rows == 0 || k == 0) return rc;
    if ((rc = device_ok()) != CDLB200_OK) return rc;
    return quant_entry<kMXFP8>(x, rows, k, ldx, transpose, packed, scale, scale_layout, nullptr,
                               nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int cdlb200_nvfp4_encode_multi(const cdlb200_nvfp4_encode_tensor* tensors, int count, void* stream) {
    if (count < 0 || (count > 0 && !tensors)) return CDLB200_ERR_INVALID_ARG;
    for (int i = 0; i < count; ++i) {
        const cdlb200_nvfp4_encode_tensor& t = tensors[i];
        if (t.rows < 0 || t.k < 0 || (t.k % 16) != 0) return CDLB200_ERR_INVALID_ARG;
        if (t.rows == 0 || t.k == 0) continue;
        if (!t.x || !t.amax || !t.packed || !t.scale || !t.alpha || t.amax_words < 0 || t.amax_words > 64)
            return CDLB200_ERR_INVALID_ARG;
        if ((t.rows % 128) != 0 || ((t.k / 16) % 4) != 0 || t.rows * (t.k / 16) >= (1ll << 31))
            return CDLB200_ERR_INVALID_ARG;
        if (!aligned(t.x, 16) || !aligned(t.packed, 8) || (t.deq && !aligned(t.deq, 16))) return CDLB200_ERR_ALIGNMENT;
    }
    int rc;
    if ((rc = device_ok()) != CDLB200_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    std::vector<EncGroup> groups;
    int64_t chunk = 0;
    for (int i = 0; i < count; ++i) {
        const cdlb200_nvfp4_encode_tensor& t = tensors[i];
        if (t.rows == 0 || t.k == 0) continue;
        if (groups.empty() || groups.back().count == kEncGroup) {
            groups.emplace_back();
            groups.back().count = 0;
            groups.back().pad = 0;
        }
        EncGroup& g = groups.back();
        g.t[g.count] = t;
        g.nb[g.count] = FastDiv((uint32_t)(t.k / 16));
        g.chunk0[g.count] = chunk;
        chunk += (t.rows * (t.k / 16) + kEncChunkBlocks - 1) / kEncChunkBlocks;
        g.chunk0[++g.count] = chunk;
    }
    const int64_t cap = (int64_t)num_sms() * 8;
    for (const EncGroup& g : groups) {
        const int64_t n = g.chunk0[g.count] - g.chunk0[0];
        nvfp4_encode_multi_kernel<<<(unsigned)(n < cap ? n : cap), kEncThreads, 0, st>>>(g);
        CDLB200_CHECK_LAUNCH();
    }
    return CDLB200_OK;
}

namespace {
// Zero the last 128-row block of a 128x4-layout scale matrix of `rows` rows
// and `nb` blocks when rows is not a multiple of 128 (its padding rows are
// interleaved with the valid ones; the kernel then writes the valid rows).
int zero_scale_tail(void* scale, int64_t rows, int64_t nb, cudaStream_t st) {
    if ((rows % 128) == 0) return CDLB200_OK;
    const int64_t c4 = (nb + 3) / 4;
    const int64_t off = (rows / 128) * c4 * 512;
    return cudaMemsetAsync(static_cast<uint8_t*>(scale) + off, 0, (size_t)(c4 * 512), st) == cudaSuccess
               ? CDLB200_OK
               : CDLB200_ERR_CUDA;
}
}  // namespace

extern "C" int cdlb200_nvfp4_dual_multi(const cdlb200_nvfp4_dual_tensor* tensors, int count, void* stream) {
    if (count < 0 || (count > 0 && !tensors)) return CDLB200_ERR_INVALID_ARG;
    for (int i = 0; i < count; ++i) {
        const cdlb200_nvfp4_dual_tensor& t = tensors[i];
        if (t.rows < 0 || t.cols < 0 || (t.rows % kDualT) != 0 || (t.cols % kDualT) != 0) return CDLB200_ERR_INVALID_ARG;
        if (t.rows == 0 || t.cols == 0) continue;
        if (!t.x || !t.alpha || (!t.amax && !t.gmax) || (t.amax && (t.amax_words < 1 || t.amax_words > 64)))
            return CDLB200_ERR_INVALID_ARG;
        if ((t.row_packed && !t.row_scale) || (t.col_packed && !t.col_scale)) return CDLB200_ERR_INVALID_ARG;
        if ((t.flags & ~(CDLB200_DUAL_ROW_LINEAR | CDLB200_DUAL_COL_LINEAR)) != 0) return CDLB200_ERR_INVALID_ARG;
        if ((t.rows / kDualT) * (t.cols / kDualT) >= (1ll << 31)) return CDLB200_ERR_INVALID_ARG;
        if (!aligned(t.x, 16) || (t.row_packed && !aligned(t.row_packed, 8)) ||
            (t.col_packed && !aligned(t.col_packed, 16)) || (t.row_scale && !aligned(t.row_scale, 4)) ||
            (t.col_scale && !aligned(t.col_scale, 4)))
            return CDLB200_ERR_ALIGNMENT;
    }
    int rc;
    if ((rc = device_ok()) != CDLB200_OK) return rc;
    return launch_dual(tensors, count, static_cast<cudaStream_t>(stream));
}

namespace cdlb200 {
namespace {
int launch_dual(const cdlb200_nvfp4_dual_tensor* tensors, int count, cudaStream_t st) {
    int rc;
    std::vector<DualGroup> groups;
    int64_t tiles = 0;
    for (int i = 0; i < count; ++i) {
        const cdlb200_nvfp4_dual_tensor& t = tensors[i];
        if (t.rows == 0 || t.cols == 0) continue;
        if (t.row_packed && !(t.flags & CDLB200_DUAL_ROW_LINEAR) &&
            (rc = zero_scale_tail(t.row_scale, t.rows, t.cols / 16, st)) != CDLB200_OK)
            return rc;
        if (t.col_packed && !(t.flags & CDLB200_DUAL_COL_LINEAR) &&
            (rc = zero_scale_tail(t.col_scale, t.cols, t.rows / 16, st)) != CDLB200_OK)
            return rc;
        const int64_t nt = (t.rows / kDualT) * ((t.cols + kDualW - 1) / kDualW);
        if (groups.empty() || groups.back().count == kDualGroup || tiles + nt >= (1ll << 31)) {
            groups.emplace_back();
            groups.back().count = 0;
            groups.back().pad = 0;
            tiles = 0;
        }
        DualGroup& g = groups.back();
        g.t[g.count] = t;
        g.items_c[g.count] = FastDiv((uint32_t)((t.cols + kDualW - 1) / kDualW));
        g.item0[g.count] = (int32_t)tiles;
        tiles += nt;
        g.item0[++g.count] = (int32_t)tiles;
    }
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(nvfp4_dual_multi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDualSmem) !=
            cudaSuccess)
            return CDLB200_ERR_CUDA;
        attr_set = true;
    }
    const int64_t cap = (int64_t)persistent_sms() * 4;  // four resident CTAs per SM
    for (const DualGroup& g : groups) {
        const int64_t n = g.item0[g.count];
        nvfp4_dual_multi_kernel<<<(unsigned)(n < cap ? n : cap), kDualThreads, kDualSmem, st>>>(g);
        CDLB200_CHECK_LAUNCH();
    }
    return CDLB200_OK;
}
}  // namespace
}  // namespace cdlb200
