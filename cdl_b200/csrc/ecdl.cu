// ecdl.cu -- the ECDL ("extended CDL") stochastic block-scaled quantizer of
// cdl (cdl/core/kernel/ecdl/{kernel,launch,autograd}.py) for NVFP4 (nvidia
// scales: per-block UE4M3 from the global amax) and MXFP4 / MXFP8 (OCP
// scales: per-block E8M0 from the block's exponent).
//
// Forward, per element x of a block with scale s:  v = x / s; the element's
// level index is SAMPLED from the top-k window of levels around v with
// weights exp(-kappa (c - t)^2) relative to the nearest level (c is v's
// position in level-index units, linear between neighbouring levels); the
// uniform number is Triton's tl.rand(seed, flat index), i.e. Philox4x32-10
// on counter (index, 0, 0, 0) and key (seed, sign extension), so the stream
// is the reference's.  Backward: the gradient of the sampled level's
// expectation (the CDL proxy): dtheta = g * d E[level] / dx, plus the sums
// d kappa = sum g s dk and d alpha = sum g ds q.
//
// One thread per two consecutive elements; a block's 16 (NVFP4) or 32 (MX)
// elements are 8 or 16 adjacent lanes, which reduce the block amax with
// shuffles.  Level and gap tables sit in shared memory.
#include "cdlb200_step.h"
#include "common.cuh"

namespace cdlb200 {
namespace {

constexpr int kEcdlThreads = 256;
constexpr float kTiny = 1.1754943508222875e-38f;
constexpr float kLog2e = 1.4426950408889634f;

struct EcdlFormat {
    int tn;    // theta levels: 16 (e2m1) or 254 (e4m3)
    int tpb;   // elements per block: 16 (NVFP4) or 32 (MX)
    int bias;  // scale byte = scale index + bias (1 for UE4M3 without zero)
    int emax;  // floor(log2(max level)): 2 (e2m1), 8 (e4m3)
};

__host__ __device__ inline EcdlFormat ecdl_format(int fmt) {
    if (fmt == CDLB200_ECDL_NVFP4) return {16, 16, 1, 2};
    if (fmt == CDLB200_ECDL_MXFP4) return {16, 32, 0, 2};
    return {254, 32, 0, 8};
}

// level of index `key` (ascending; -0 sits just below +0)
__device__ float theta_level(int tn, int key) {
    if (tn == 126) return e4m3_to_f32((uint32_t)(key + 1));                     // UE4M3 without zero
    if (tn == 255) return u2f(key == 0 ? 0x00400000u : ((uint32_t)key << 23));  // E8M0, byte 0 = 2^-127
    if (tn == 16) {
        const int m = key >= 8 ? key - 8 : 7 - key;
        const float mag = m < 4 ? 0.5f * (float)m : (float)(1 << ((m >> 1) - 1)) * ((m & 1) ? 1.5f : 1.0f);
        return key >= 8 ? mag : -mag;
    }
    return e4m3_to_f32((uint32_t)(key >= 127 ? key - 127 : 254 - key));
}

// level / gap tables: gap[k] = level[k+1] - level[k], the last repeated, a
// zero gap (between -0 and +0) replaced by the one before (cdl/api/format.py)
__device__ void build_tables(int tn, float* lev, float* gap) {
    for (int k = threadIdx.x; k < tn; k += blockDim.x) lev[k] = theta_level(tn, k);
    __syncthreads();
    for (int k = threadIdx.x; k < tn; k += blockDim.x) {
        auto raw = [&](int i) { return i < tn - 1 ? lev[i + 1] - lev[i] : lev[tn - 1] - lev[tn - 2]; };
        float gk = raw(k);
        if (gk == 0.0f) gk = raw(k > 0 ? k - 1 : tn - 1);
        gap[k] = gk;
    }
    __syncthreads();
}

// fp32 -> e4m3 byte, round to nearest even, saturating (sign kept)
__device__ __forceinline__ uint32_t ue4m3_cvt(float v) { return cvt_e4m3x2(0.0f, v) & 0xffu; }

// nearest-level ordinal (cdl/core/kernel/formats/ordinals.py) of a theta grid
// (16: e2m1, 254: e4m3) or a scale grid (126: UE4M3 without zero, 255: E8M0)
__device__ __forceinline__ int theta_ordinal(int tn, float v) {
    if (tn == 126) {
        const int b = (int)ue4m3_cvt(fminf(fmaxf(v, 0.001953125f), 448.0f)) - 1;
        return b < 0 ? 0 : (b > 125 ? 125 : b);
    }
    if (tn == 255) {
        const uint32_t bits = f2u(fminf(fmaxf(v, 0x1p-127f), 0x1p127f));
        const int e8 = (int)(bits >> 23), mant = (int)(bits & 0x7fffff);
        if (e8 == 0) return mant > 4194304 ? 1 : 0;
        const int k = e8 + (mant >= 4194304);
        return k < 254 ? k : 254;
    }
    if (tn == 16) {
        const bool neg = (f2u(v) >> 31) != 0;
        const float av = fminf(fabsf(v), 6.0f);
        const int mag = (av > 0.25f) + (av > 0.75f) + (av > 1.25f) + (av > 1.75f) + (av > 2.5f) + (av > 3.5f) +
                        (av > 5.0f);
        return neg ? 7 - mag : 8 + mag;
    }
    const int b = (int)(ue4m3_cvt(fminf(fmaxf(v, -448.0f), 448.0f)));
    const int key = b < 128 ? b + 127 : 254 - b;
    return key < 0 ? 0 : (key > tn - 1 ? tn - 1 : key);
}

// Philox4x32-10, first output word (Salmon et al., SC 2011)
__device__ __forceinline__ uint32_t philox_x0(uint32_t c0, uint32_t k0, uint32_t k1) {
    uint32_t c1 = 0, c2 = 0, c3 = 0;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c0;
}

// tl.rand: the int32 view x of the word, (x < 0 ? -x - 1 : x) * 4.6566127342e-10
__device__ __forceinline__ float rand_uniform(uint32_t offset, int32_t seed) {
    const int32_t x = (int32_t)philox_x0(offset, (uint32_t)seed, seed < 0 ? 0xFFFFFFFFu : 0u);
    const int32_t y = x < 0 ? -x - 1 : x;
    return __fmul_rn(__int2float_rn(y), 4.6566127342e-10f);
}

struct Window {
    float c, kgap;
    int start;
};

__device__ __forceinline__ Window cdl_window(float v, const float* lev, const float* gap, int tn, int topk) {
    const int key = theta_ordinal(tn, v);
    const float klev = lev[key];
    const int left = key > 0 ? key - 1 : 0;
    Window w;
    w.kgap = v >= klev ? gap[key] : gap[left];
    // every gap of e2m1 and e4m3 is a power of two: the quotient is the
    // product with the exact reciprocal
    w.c = __fadd_rn((float)key, __fmul_rn(__fsub_rn(v, klev), __frcp_rn(w.kgap)));
    const int st = key - topk / 2;
    w.start = st < 0 ? 0 : (st > tn - topk ? tn - topk : st);
    return w;
}

__device__ __forceinline__ float cdl_weight(float c, float t, float t_near, float m, float kappa) {
    if (t == t_near) return 1.0f;
    const float d = __fsub_rn(c, t);
    return exp2f(__fmul_rn(fminf(__fsub_rn(__fmul_rn(__fmul_rn(-kappa, d), d), m), 0.0f), kLog2e));
}

__device__ __forceinline__ int cdl_sample(float v, float kappa, float u, const float* lev, const float* gap, int tn,
                                          int topk) {
    const Window w = cdl_window(v, lev, gap, tn, topk);
    const float fs = (float)w.start;
    const float t_near = fminf(fmaxf(floorf(__fadd_rn(w.c, 0.5f)), fs), (float)(w.start + topk - 1));
    const float dn = __fsub_rn(t_near, w.c);
    const float m = __fmul_rn(__fmul_rn(-kappa, dn), dn);
    float z = 0.0f;
    for (int j = 0; j < topk; ++j) z = __fadd_rn(z, cdl_weight(w.c, fs + (float)j, t_near, m, kappa));
    const float uz = __fmul_rn(u, z);
    float acc = 0.0f;
    int cnt = 0;
    for (int j = 0; j < topk; ++j) {
        acc = __fadd_rn(acc, cdl_weight(w.c, fs + (float)j, t_near, m, kappa));
        cnt += acc <= uz;
    }
    return w.start + (cnt < topk - 1 ? cnt : topk - 1);
}

// the same sampler for a window width K known at compile time: the weights
// are computed once and kept in registers
template <int K>
__device__ __forceinline__ int cdl_sample_k(float v, float kappa, float u, const float* lev, const float* gap,
                                            int tn) {
    const Window w = cdl_window(v, lev, gap, tn, K);
    const float fs = (float)w.start;
    const float t_near = fminf(fmaxf(floorf(__fadd_rn(w.c, 0.5f)), fs), (float)(w.start + K - 1));
    const float dn = __fsub_rn(t_near, w.c);
    const float m = __fmul_rn(__fmul_rn(-kappa, dn), dn);
    float wt[K];
    float z = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
        wt[j] = cdl_weight(w.c, fs + (float)j, t_near, m, kappa);
        z = __fadd_rn(z, wt[j]);
    }
    const float uz = __fmul_rn(u, z);
    float acc = 0.0f;
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < K; ++j) {
        acc = __fadd_rn(acc, wt[j]);
        cnt += acc <= uz;
    }
    return w.start + (cnt < K - 1 ? cnt : K - 1);
}

template <int K>
__device__ __forceinline__ int sample_dispatch(float v, float kappa, float u, const float* lev, const float* gap,
                                               int tn, int topk) {
    if constexpr (K > 0) return cdl_sample_k<K>(v, kappa, u, lev, gap, tn);
    else return cdl_sample(v, kappa, u, lev, gap, tn, topk);
}

// half-width of the truncated (scale-side) window: most of the weight of a
// sharp window lies within sqrt(60 / kappa) levels of the nearest one
__device__ __forceinline__ int half_window(int topk, float kappa) {
    int hq = topk / 2;
    if (kappa > 0.05f) hq = (int)fminf((float)(topk / 2), sqrtf(__fdiv_rn(60.0f, kappa))) + 1;
    return hq;
}

// cdl_sample_truncated (primitives.py:73-135): the window [t_lo, t_lo + 2 hq]
// around the nearest level, the left tail folded into one jump
__device__ __forceinline__ int cdl_sample_truncated(float v, float kappa, float u, const float* lev,
                                                    const float* gap, int tn, int topk) {
    const Window w = cdl_window(v, lev, gap, tn, topk);
    const float t_near = fminf(fmaxf(floorf(__fadd_rn(w.c, 0.5f)), (float)w.start), (float)(w.start + topk - 1));
    const float dn = __fsub_rn(t_near, w.c);
    const float m = __fmul_rn(__fmul_rn(-kappa, dn), dn);
    const int hq = half_window(topk, kappa);
    const int tn_i = (int)t_near;
    const int t_lo = tn_i - hq > w.start ? tn_i - hq : w.start;
    const int last = w.start + topk - 1;
    float z = 0.0f;
    for (int j = 0; j <= 2 * hq; ++j) {
        const int t = t_lo + j;
        if (t >= w.start && t <= last) z = __fadd_rn(z, cdl_weight(w.c, (float)t, t_near, m, kappa));
    }
    const float dl = __fsub_rn((float)(t_lo - 1), w.c);
    const float e_left =
        exp2f(__fmul_rn(fminf(__fsub_rn(__fmul_rn(__fmul_rn(-kappa, dl), dl), m), 0.0f), kLog2e));
    const float uz = __fmul_rn(u, z);
    const int off = uz >= __fmul_rn(e_left, __fadd_rn((float)(t_lo - w.start), 1.0f)) ? t_lo - w.start : 0;
    float acc = 0.0f;
    int cnt = 0;
    for (int j = 0; j <= 2 * hq; ++j) {
        const int t = t_lo + j;
        if (t >= w.start && t <= last) {
            acc = __fadd_rn(acc, cdl_weight(w.c, (float)t, t_near, m, kappa));
            cnt += acc <= uz;
        }
    }
    const int sub = off + cnt;
    return w.start + (sub < topk - 1 ? sub : topk - 1);
}

struct Coeffs {
    float dth, ds, dk;
};

// cdl_proxy_coeffs_truncated (primitives.py:190-240)
__device__ __forceinline__ Coeffs cdl_proxy_coeffs_truncated(float v, float kappa, const float* lev,
                                                             const float* gap, int tn, int topk) {
    const Window w = cdl_window(v, lev, gap, tn, topk);
    const float t_near = fminf(fmaxf(floorf(__fadd_rn(w.c, 0.5f)), (float)w.start), (float)(w.start + topk - 1));
    const float dn = __fsub_rn(t_near, w.c);
    const float m = __fmul_rn(__fmul_rn(-kappa, dn), dn);
    const int hq = half_window(topk, kappa);
    const int tn_i = (int)t_near;
    const int t_lo = tn_i - hq > w.start ? tn_i - hq : w.start;
    const int last = w.start + topk - 1;
    float z = 0.f, sl = 0.f, sa = 0.f, sal = 0.f, sb = 0.f, sbl = 0.f;
    for (int j = 0; j <= 2 * hq; ++j) {
        const int t = t_lo + j;
        if (t < w.start || t > last) continue;
        const float d = __fsub_rn(w.c, (float)t);
        const float e = cdl_weight(w.c, (float)t, t_near, m, kappa);
        const float lv = lev[t];
        const float a = __fmul_rn(__fmul_rn(-2.0f, kappa), d);
        const float dd = __fmul_rn(d, d);
        z += e;
        sl += e * lv;
        sa += e * a;
        sal += e * a * lv;
        sb += e * dd;
        sbl += e * dd * lv;
    }
    Coeffs r;
    const float p = sl / z;
    r.dth = (sal / z - p * (sa / z)) / w.kgap;
    r.ds = p - v * r.dth;
    r.dk = p * (sb / z) - sbl / z;
    return r;
}

__device__ __forceinline__ Coeffs cdl_proxy_coeffs(float v, float kappa, const float* lev, const float* gap, int tn,
                                                   int topk) {
    const Window w = cdl_window(v, lev, gap, tn, topk);
    const float fs = (float)w.start;
    const float t_near = fminf(fmaxf(floorf(__fadd_rn(w.c, 0.5f)), fs), (float)(w.start + topk - 1));
    const float dn = __fsub_rn(t_near, w.c);
    const float m = __fmul_rn(__fmul_rn(-kappa, dn), dn);
    float z = 0.f, sl = 0.f, sa = 0.f, sal = 0.f, sb = 0.f, sbl = 0.f;
    for (int j = 0; j < topk; ++j) {
        const float t = fs + (float)j;
        const float d = __fsub_rn(w.c, t);
        const float e = cdl_weight(w.c, t, t_near, m, kappa);
        const float lv = lev[w.start + j];
        const float a = __fmul_rn(__fmul_rn(-2.0f, kappa), d);
        const float dd = __fmul_rn(d, d);
        z += e;
        sl += e * lv;
        sa += e * a;
        sal += e * a * lv;
        sb += e * dd;
        sbl += e * dd * lv;
    }
    Coeffs r;
    const float p = sl / z;
    r.dth = (sal / z - p * (sa / z)) / w.kgap;
    r.ds = p - v * r.dth;
    r.dk = p * (sb / z) - sbl / z;
    return r;
}

template <typename T>
__device__ __forceinline__ void load2(const T* x, int64_t i, float& a, float& b);
template <>
__device__ __forceinline__ void load2<uint16_t>(const uint16_t* x, int64_t i, float& a, float& b) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(x + i);
    a = u2f(w << 16);
    b = u2f(w & 0xffff0000u);
}
template <>
__device__ __forceinline__ void load2<float>(const float* x, int64_t i, float& a, float& b) {
    const float2 w = *reinterpret_cast<const float2*>(x + i);
    a = w.x;
    b = w.y;
}

template <typename T>
__device__ __forceinline__ void store2(T* x, int64_t i, float a, float b);
template <>
__device__ __forceinline__ void store2<uint16_t>(uint16_t* x, int64_t i, float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    *reinterpret_cast<uint32_t*>(x + i) = r;
}
template <>
__device__ __forceinline__ void store2<float>(float* x, int64_t i, float a, float b) {
    *reinterpret_cast<float2*>(x + i) = make_float2(a, b);
}

// block amax over the `lanes` adjacent lanes holding one block
__device__ __forceinline__ float group_max(float a, int lanes) {
    for (int o = lanes >> 1; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    return a;
}

// global amax of |x| as float bits (non-negative floats order as integers)
template <typename T>
__global__ void __launch_bounds__(kEcdlThreads) ecdl_amax_kernel(const T* __restrict__ x, int64_t npairs,
                                                                 uint32_t* __restrict__ gmax_bits) {
    float a = 0.0f;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < npairs; p += (int64_t)gridDim.x * blockDim.x) {
        float x0, x1;
        load2(x, 2 * p, x0, x1);
        a = fmaxf(a, fmaxf(fabsf(x0), fabsf(x1)));
    }
    a = group_max(a, 32);
    __shared__ float red[kEcdlThreads / 32];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kEcdlThreads / 32; ++w) a = fmaxf(a, red[w]);
        atomicMax(gmax_bits, f2u(a));
    }
}

// scale of a block: (scale index, s) for the nvidia (0) or OCP (1) mode
__device__ __forceinline__ void block_scale(int mode, const EcdlFormat& f, float bamax, float gmax, float alpha,
                                            int& qi, float& s) {
    if (mode == CDLB200_ECDL_NVIDIA) {
        const float qv = __fdiv_rn(__fmul_rn(bamax, 448.0f), gmax);
        const int b = (int)ue4m3_cvt(fminf(fmaxf(qv, 0.001953125f), 448.0f));
        qi = b - 1 < 0 ? 0 : (b - 1 > 125 ? 125 : b - 1);
        s = __fmul_rn(e4m3_to_f32((uint32_t)(qi + 1)), alpha);
    } else {
        const int fl = (int)(f2u(fmaxf(bamax, kTiny)) >> 23) - 127;
        const int e = fl - f.emax + 127;
        qi = e < 0 ? 0 : (e > 254 ? 254 : e);
        s = u2f(qi == 0 ? 0x00400000u : ((uint32_t)qi << 23));  // alpha is 1 in this mode
    }
}

template <typename T, int K>
__global__ void __launch_bounds__(kEcdlThreads) ecdl_fwd_kernel(const T* __restrict__ theta, int64_t npairs, int fmt,
                                                                int mode, int topk, const float* __restrict__ kappa_p,
                                                                const int64_t* __restrict__ seed_p,
                                                                const uint32_t* __restrict__ gmax_bits,
                                                                uint8_t* __restrict__ packed,
                                                                uint8_t* __restrict__ scale, float* __restrict__ alpha_out) {
    __shared__ float lev[256], gap[256];
    const EcdlFormat f = ecdl_format(fmt);
    build_tables(f.tn, lev, gap);
    const float kappa = *kappa_p;
    const int32_t seed = (int32_t)(uint32_t)(*seed_p & 0xffffffffll);
    float gmax = 1.0f, alpha = 1.0f;
    if (mode == CDLB200_ECDL_NVIDIA) {
        gmax = fmaxf(u2f(*gmax_bits), kTiny);
        alpha = nvfp4_alpha(gmax);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *alpha_out = alpha;
    const int lanes = f.tpb / 2;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // whole warps iterate together (the block shuffles need all lanes)
    for (int64_t p0 = (int64_t)blockIdx.x * blockDim.x; p0 < npairs; p0 += stride) {
        const int64_t p = p0 + threadIdx.x;
        const bool ok = p < npairs;
        float x0 = 0.f, x1 = 0.f;
        if (ok) load2(theta, 2 * p, x0, x1);
        const float bamax = group_max(fmaxf(fabsf(x0), fabsf(x1)), lanes);
        if (!ok) continue;
        int qi;
        float s;
        block_scale(mode, f, bamax, gmax, alpha, qi, s);
        const float u0 = rand_uniform((uint32_t)(2 * p), seed), u1 = rand_uniform((uint32_t)(2 * p + 1), seed);
        const int i0 = sample_dispatch<K>(__fdiv_rn(x0, s), kappa, u0, lev, gap, f.tn, topk);
        const int i1 = sample_dispatch<K>(__fdiv_rn(x1, s), kappa, u1, lev, gap, f.tn, topk);
        if (f.tn == 16) {
            const uint32_t c0 = i0 < 8 ? 15 - i0 : i0 - 8, c1 = i1 < 8 ? 15 - i1 : i1 - 8;
            packed[p] = (uint8_t)(c0 | (c1 << 4));
        } else {
            const uint32_t b0 = i0 < 127 ? 254 - i0 : i0 - 127, b1 = i1 < 127 ? 254 - i1 : i1 - 127;
            reinterpret_cast<uint16_t*>(packed)[p] = (uint16_t)(b0 | (b1 << 8));
        }
        if ((p % lanes) == 0) scale[(2 * p) / f.tpb] = (uint8_t)(qi + f.bias);
    }
}

template <typename T>
__global__ void __launch_bounds__(kEcdlThreads) ecdl_bwd_kernel(const T* __restrict__ grad, const T* __restrict__ theta,
                                                                int64_t npairs, int fmt, int topk,
                                                                const uint8_t* __restrict__ scale,
                                                                const float* __restrict__ kappa_p,
                                                                const float* __restrict__ alpha_p,
                                                                T* __restrict__ dtheta, float* __restrict__ part) {
    __shared__ float lev[256], gap[256];
    __shared__ float red[2][kEcdlThreads / 32];
    const EcdlFormat f = ecdl_format(fmt);
    build_tables(f.tn, lev, gap);
    const float kappa = *kappa_p, alpha = *alpha_p;
    float dkt = 0.f, dal = 0.f;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < npairs; p += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)scale[(2 * p) / f.tpb];
        int qi = b - f.bias;
        qi = qi < 0 ? 0 : qi;
        const float q_hat = f.bias ? e4m3_to_f32((uint32_t)(qi + 1)) : u2f(qi == 0 ? 0x00400000u : ((uint32_t)qi << 23));
        const float s = __fmul_rn(q_hat, alpha);
        float g0, g1, x0, x1;
        load2(grad, 2 * p, g0, g1);
        load2(theta, 2 * p, x0, x1);
        const float v0 = __fdiv_rn(x0, s), v1 = __fdiv_rn(x1, s);
        const Coeffs c0 = cdl_proxy_coeffs(v0, kappa, lev, gap, f.tn, topk);
        const Coeffs c1 = cdl_proxy_coeffs(v1, kappa, lev, gap, f.tn, topk);
        store2(dtheta, 2 * p, g0 * c0.dth, g1 * c1.dth);
        dkt += g0 * s * c0.dk + g1 * s * c1.dk;
        dal += (g0 * c0.ds + g1 * c1.ds) * q_hat;
    }
    if (!part) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        dkt += __shfl_xor_sync(0xffffffffu, dkt, o);
        dal += __shfl_xor_sync(0xffffffffu, dal, o);
    }
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = dkt;
        red[1][threadIdx.x >> 5] = dal;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.f, c = 0.f;
        for (int w = 0; w < kEcdlThreads / 32; ++w) {
            a += red[0][w];
            c += red[1][w];
        }
        part[2 * blockIdx.x] = a;
        part[2 * blockIdx.x + 1] = c;
    }
}

// fixed-order sum of the per-CTA partials -> scalars[2]
__global__ void ecdl_sum_kernel(const float* __restrict__ part, int n, float* __restrict__ scalars) {
    __shared__ float red[2][32];
    float a = 0.f, c = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        a += part[2 * i];
        c += part[2 * i + 1];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = a;
        red[1][threadIdx.x >> 5] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        a = c = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
            a += red[0][w];
            c += red[1][w];
        }
        scalars[0] = a;
        scalars[1] = c;
    }
}

// ---------------------------------------------------------------------------
// CCDL (cdl/core/kernel/ccdl/kernel.py): the block scale is a learnable
// value q (one per block, or one row of q shared by every theta row when
// q_stride is 0), sampled on the scale grid with the truncated window and
// its own kappa from tl.rand(seed, rows * K + r * q_stride + b); then theta
// is sampled as in ECDL with s = q_level * alpha.
// ---------------------------------------------------------------------------
struct CcdlArgs {
    int64_t npairs, k, rows;
    int fmt, topk, q_topk;
    const float* q;
    int64_t q_stride;
    const float* kappa_t;
    const float* kappa_q;
    const float* alpha;
};

__device__ __forceinline__ int q_grid(int fmt) { return fmt == CDLB200_ECDL_NVFP4 ? 126 : 255; }

template <typename T, int K>
__global__ void __launch_bounds__(kEcdlThreads) ccdl_fwd_kernel(const T* __restrict__ theta, CcdlArgs a,
                                                                const int64_t* __restrict__ seed_p,
                                                                uint8_t* __restrict__ packed,
                                                                uint8_t* __restrict__ scale) {
    __shared__ float lev[256], gap[256], qlev[256], qgap[256];
    const EcdlFormat f = ecdl_format(a.fmt);
    const int qn = q_grid(a.fmt);
    build_tables(f.tn, lev, gap);
    build_tables(qn, qlev, qgap);
    const float kt = *a.kappa_t, kq = *a.kappa_q, alpha = *a.alpha;
    const int32_t seed = (int32_t)(uint32_t)(*seed_p & 0xffffffffll);
    const int lanes = f.tpb / 2;
    const int lane = threadIdx.x & 31, leader = lane & ~(lanes - 1);
    const int64_t nb = a.k / f.tpb;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p0 = (int64_t)blockIdx.x * blockDim.x; p0 < a.npairs; p0 += stride) {
        const int64_t p = p0 + threadIdx.x;
        const bool ok = p < a.npairs;
        int qi = 0;
        if (ok && lane == leader) {  // the block's scale, sampled once
            const int64_t e = 2 * p, r = e / a.k, b = (e - r * a.k) / f.tpb;
            const float qv = a.q[r * a.q_stride + b];
            const float uq = rand_uniform((uint32_t)(a.rows * a.k + r * a.q_stride + b), seed);
            qi = cdl_sample_truncated(qv, kq, uq, qlev, qgap, qn, a.q_topk);
            scale[r * nb + b] = (uint8_t)(qi + f.bias);
        }
        qi = __shfl_sync(0xffffffffu, qi, leader);
        if (!ok) continue;
        const float s = __fmul_rn(qlev[qi], alpha);
        float x0, x1;
        load2(theta, 2 * p, x0, x1);
        const float u0 = rand_uniform((uint32_t)(2 * p), seed), u1 = rand_uniform((uint32_t)(2 * p + 1), seed);
        const int i0 = sample_dispatch<K>(__fdiv_rn(x0, s), kt, u0, lev, gap, f.tn, a.topk);
        const int i1 = sample_dispatch<K>(__fdiv_rn(x1, s), kt, u1, lev, gap, f.tn, a.topk);
        if (f.tn == 16) {
            const uint32_t c0 = i0 < 8 ? 15 - i0 : i0 - 8, c1 = i1 < 8 ? 15 - i1 : i1 - 8;
            packed[p] = (uint8_t)(c0 | (c1 << 4));
        } else {
            const uint32_t b0 = i0 < 127 ? 254 - i0 : i0 - 127, b1 = i1 < 127 ? 254 - i1 : i1 - 127;
            reinterpret_cast<uint16_t*>(packed)[p] = (uint16_t)(b0 | (b1 << 8));
        }
    }
}

// fp32 -> bf16 -> fp32, round to nearest even
__device__ __forceinline__ float bf16_round(float v) {
    uint32_t h;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(0.0f), "f"(v));
    return u2f(h << 16);
}

// CCDL eval forward (cdl/core/ccdl.py:78-89 cascaded_nearest_round): q's
// nearest scale level, s = level * alpha in the level dtype, each element's
// nearest theta level of theta / s in the promoted dtype of theta and levels.
// lev_bf16: the levels are bf16, so s is rounded to bf16, and so is the
// quotient when theta is bf16 as well (torch's bf16 arithmetic).
template <typename T>
__global__ void __launch_bounds__(kEcdlThreads) ccdl_round_kernel(const T* __restrict__ theta, CcdlArgs a,
                                                                  int lev_bf16, uint8_t* __restrict__ packed,
                                                                  uint8_t* __restrict__ scale) {
    const EcdlFormat f = ecdl_format(a.fmt);
    const int qn = q_grid(a.fmt);
    const float alpha = *a.alpha;
    const bool bf_quot = lev_bf16 && sizeof(T) == 2;
    const int lanes = f.tpb / 2;
    const int64_t nb = a.k / f.tpb;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < a.npairs; p += stride) {
        const int64_t e = 2 * p, r = e / a.k, b = (e - r * a.k) / f.tpb;
        const int qi = theta_ordinal(qn, a.q[r * a.q_stride + b]);
        float s = __fmul_rn(theta_level(qn, qi), alpha);
        if (lev_bf16) s = bf16_round(s);
        float x0, x1;
        load2(theta, e, x0, x1);
        float v0 = __fdiv_rn(x0, s), v1 = __fdiv_rn(x1, s);
        if (bf_quot) {
            v0 = bf16_round(v0);
            v1 = bf16_round(v1);
        }
        const int i0 = theta_ordinal(f.tn, v0), i1 = theta_ordinal(f.tn, v1);
        if (f.tn == 16) {
            const uint32_t c0 = i0 < 8 ? 15 - i0 : i0 - 8, c1 = i1 < 8 ? 15 - i1 : i1 - 8;
            packed[p] = (uint8_t)(c0 | (c1 << 4));
        } else {
            const uint32_t b0 = i0 < 127 ? 254 - i0 : i0 - 127, b1 = i1 < 127 ? 254 - i1 : i1 - 127;
            reinterpret_cast<uint16_t*>(packed)[p] = (uint16_t)(b0 | (b1 << 8));
        }
        if ((p % lanes) == 0) scale[r * nb + b] = (uint8_t)(qi + f.bias);
    }
}

template <typename T>
__global__ void __launch_bounds__(kEcdlThreads) ccdl_bwd_kernel(const T* __restrict__ grad, const T* __restrict__ theta,
                                                                CcdlArgs a, const uint8_t* __restrict__ scale,
                                                                int64_t scale_stride, T* __restrict__ dtheta,
                                                                float* __restrict__ dq, float* __restrict__ part) {
    __shared__ float lev[256], gap[256], qlev[256], qgap[256];
    __shared__ float red[3][kEcdlThreads / 32];
    const EcdlFormat f = ecdl_format(a.fmt);
    const int qn = q_grid(a.fmt);
    build_tables(f.tn, lev, gap);
    build_tables(qn, qlev, qgap);
    const float kt = *a.kappa_t, kq = *a.kappa_q, alpha = *a.alpha;
    const int lanes = f.tpb / 2;
    const int lane = threadIdx.x & 31, leader = lane & ~(lanes - 1);
    const int64_t nb = a.k / f.tpb;
    float dkt = 0.f, dkq = 0.f, dal = 0.f;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t p0 = (int64_t)blockIdx.x * blockDim.x; p0 < a.npairs; p0 += stride) {
        const int64_t p = p0 + threadIdx.x;
        const bool ok = p < a.npairs;
        const int64_t e = 2 * p, r = e / a.k, b = (e - r * a.k) / f.tpb;
        float ds_sum = 0.f;
        if (ok) {
            int qi = (int)scale[r * scale_stride + b] - f.bias;
            qi = qi < 0 ? 0 : qi;
            const float q_hat = qlev[qi];
            const float s = __fmul_rn(q_hat, alpha);
            float g0, g1, x0, x1;
            load2(grad, 2 * p, g0, g1);
            load2(theta, 2 * p, x0, x1);
            const float v0 = __fdiv_rn(x0, s), v1 = __fdiv_rn(x1, s);
            const Coeffs c0 = cdl_proxy_coeffs(v0, kt, lev, gap, f.tn, a.topk);
            const Coeffs c1 = cdl_proxy_coeffs(v1, kt, lev, gap, f.tn, a.topk);
            store2(dtheta, 2 * p, g0 * c0.dth, g1 * c1.dth);
            dkt += g0 * s * c0.dk + g1 * s * c1.dk;
            const float ds0 = g0 * c0.ds, ds1 = g1 * c1.ds;
            dal += (ds0 + ds1) * q_hat;
            ds_sum = ds0 + ds1;
        }
        // the block's d s, then its q gradient (one lane per block)
        for (int o = lanes >> 1; o > 0; o >>= 1) ds_sum += __shfl_xor_sync(0xffffffffu, ds_sum, o);
        if (ok && lane == leader) {
            const float gq = alpha * ds_sum;
            const Coeffs cq = cdl_proxy_coeffs_truncated(a.q[r * a.q_stride + b], kq, qlev, qgap, qn, a.q_topk);
            if (dq) dq[r * nb + b] = gq * cq.dth;
            dkq += gq * cq.dk;
        }
    }
    if (!part) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        dkt += __shfl_xor_sync(0xffffffffu, dkt, o);
        dkq += __shfl_xor_sync(0xffffffffu, dkq, o);
        dal += __shfl_xor_sync(0xffffffffu, dal, o);
    }
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = dkt;
        red[1][threadIdx.x >> 5] = dkq;
        red[2][threadIdx.x >> 5] = dal;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float x = 0.f, y = 0.f, z = 0.f;
        for (int w = 0; w < kEcdlThreads / 32; ++w) {
            x += red[0][w];
            y += red[1][w];
            z += red[2][w];
        }
        part[3 * blockIdx.x] = x;
        part[3 * blockIdx.x + 1] = y;
        part[3 * blockIdx.x + 2] = z;
    }
}

// fixed-order sum of n partial triples -> scalars[3]
__global__ void ccdl_sum_kernel(const float* __restrict__ part, int n, float* __restrict__ scalars) {
    if (threadIdx.x >= 3) return;
    float acc = 0.f;
    for (int i = 0; i < n; ++i) acc += part[3 * i + threadIdx.x];
    scalars[threadIdx.x] = acc;
}

template <int K>
void launch_fwd(const void* theta, int theta_f32, int64_t npairs, int format, int scale_mode, int topk,
                const float* kappa, const int64_t* seed, const uint32_t* gbits, void* packed, void* scale,
                float* alpha, int grid, cudaStream_t st) {
    if (theta_f32)
        ecdl_fwd_kernel<float, K><<<grid, kEcdlThreads, 0, st>>>(static_cast<const float*>(theta), npairs, format,
                                                                 scale_mode, topk, kappa, seed, gbits,
                                                                 static_cast<uint8_t*>(packed),
                                                                 static_cast<uint8_t*>(scale), alpha);
    else
        ecdl_fwd_kernel<uint16_t, K><<<grid, kEcdlThreads, 0, st>>>(static_cast<const uint16_t*>(theta), npairs,
                                                                    format, scale_mode, topk, kappa, seed, gbits,
                                                                    static_cast<uint8_t*>(packed),
                                                                    static_cast<uint8_t*>(scale), alpha);
}

template <int K>
void launch_ccdl_fwd(const void* theta, int theta_f32, const CcdlArgs& a, const int64_t* seed, void* packed,
                     void* scale, int grid, cudaStream_t st) {
    if (theta_f32)
        ccdl_fwd_kernel<float, K><<<grid, kEcdlThreads, 0, st>>>(static_cast<const float*>(theta), a, seed,
                                                                 static_cast<uint8_t*>(packed),
                                                                 static_cast<uint8_t*>(scale));
    else
        ccdl_fwd_kernel<uint16_t, K><<<grid, kEcdlThreads, 0, st>>>(static_cast<const uint16_t*>(theta), a, seed,
                                                                    static_cast<uint8_t*>(packed),
                                                                    static_cast<uint8_t*>(scale));
}

int ecdl_grid(int64_t npairs) {
    const int64_t cap = (int64_t)num_sms() * 8;
    const int64_t g = (npairs + kEcdlThreads - 1) / kEcdlThreads;
    return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

bool ecdl_aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(a - 1)) == 0; }

int ecdl_check(int64_t rows, int64_t nb, int fmt, int topk) {
    if (rows < 0 || nb < 0 || (fmt != CDLB200_ECDL_NVFP4 && fmt != CDLB200_ECDL_MXFP4 && fmt != CDLB200_ECDL_MXFP8))
        return CDLB200_ERR_INVALID_ARG;
    const EcdlFormat f = ecdl_format(fmt);
    if (topk < 1 || topk > f.tn) return CDLB200_ERR_INVALID_ARG;
    if (rows * nb * f.tpb >= (1ll << 31)) return CDLB200_ERR_INVALID_ARG;  // the random stream's counter is 32-bit
    return CDLB200_OK;
}

}  // namespace
}  // namespace cdlb200

using namespace cdlb200;

extern "C" int cdlb200_ecdl_fwd(const void* theta, int theta_f32, int64_t rows, int64_t nb, int format, int scale_mode,
                                const float* kappa, const int64_t* seed, int topk, void* packed, void* scale,
                                float* alpha, void* workspace, void* stream) {
    int rc = ecdl_check(rows, nb, format, topk);
    if (rc != CDLB200_OK) return rc;
    if (scale_mode != CDLB200_ECDL_NVIDIA && scale_mode != CDLB200_ECDL_OCP) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || nb == 0) return CDLB200_OK;
    if (!theta || !kappa || !seed || !packed || !scale || !alpha || !workspace) return CDLB200_ERR_INVALID_ARG;
    const EcdlFormat f = ecdl_format(format);
    if (!ecdl_aligned(theta, theta_f32 ? 8 : 4) || !ecdl_aligned(packed, 2) || !ecdl_aligned(workspace, 4))
        return CDLB200_ERR_ALIGNMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t npairs = rows * nb * f.tpb / 2;
    uint32_t* gbits = static_cast<uint32_t*>(workspace);
    const int grid = ecdl_grid(npairs);
    if (scale_mode == CDLB200_ECDL_NVIDIA) {
        if (cudaMemsetAsync(gbits, 0, sizeof(uint32_t), st) != cudaSuccess) return CDLB200_ERR_CUDA;
        if (theta_f32)
            ecdl_amax_kernel<float><<<grid, kEcdlThreads, 0, st>>>(static_cast<const float*>(theta), npairs, gbits);
        else
            ecdl_amax_kernel<uint16_t><<<grid, kEcdlThreads, 0, st>>>(static_cast<const uint16_t*>(theta), npairs,
                                                                      gbits);
        CDLB200_CHECK_LAUNCH();
    }
    // common window widths get a sampler unrolled for them (cdl's training
    // default is 5; weights use the whole e2m1 grid, 16)
    switch (topk) {
        case 4: launch_fwd<4>(theta, theta_f32, npairs, format, scale_mode, topk, kappa, seed, gbits, packed, scale, alpha, grid, st); break;
        case 5: launch_fwd<5>(theta, theta_f32, npairs, format, scale_mode, topk, kappa, seed, gbits, packed, scale, alpha, grid, st); break;
        case 6: launch_fwd<6>(theta, theta_f32, npairs, format, scale_mode, topk, kappa, seed, gbits, packed, scale, alpha, grid, st); break;
        case 8: launch_fwd<8>(theta, theta_f32, npairs, format, scale_mode, topk, kappa, seed, gbits, packed, scale, alpha, grid, st); break;
        case 16: launch_fwd<16>(theta, theta_f32, npairs, format, scale_mode, topk, kappa, seed, gbits, packed, scale, alpha, grid, st); break;
        default: launch_fwd<0>(theta, theta_f32, npairs, format, scale_mode, topk, kappa, seed, gbits, packed, scale, alpha, grid, st); break;
    }
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int64_t cdlb200_ecdl_bwd_workspace_bytes(int64_t rows, int64_t nb, int format) {
    if (ecdl_check(rows, nb, format, 1) != CDLB200_OK || rows == 0 || nb == 0) return 0;
    const EcdlFormat f = ecdl_format(format);
    return (int64_t)ecdl_grid(rows * nb * f.tpb / 2) * 2 * (int64_t)sizeof(float);
}

extern "C" int cdlb200_ecdl_bwd(const void* grad, const void* theta, int theta_f32, int64_t rows, int64_t nb,
                                int format, const void* scale, const float* kappa, const float* alpha, int topk,
                                void* dtheta, float* scalars, void* workspace, int64_t workspace_bytes,
                                void* stream) {
    int rc = ecdl_check(rows, nb, format, topk);
    if (rc != CDLB200_OK) return rc;
    if (rows == 0 || nb == 0) return CDLB200_OK;
    if (!grad || !theta || !scale || !kappa || !alpha || !dtheta) return CDLB200_ERR_INVALID_ARG;
    const int a = theta_f32 ? 8 : 4;
    if (!ecdl_aligned(grad, a) || !ecdl_aligned(theta, a) || !ecdl_aligned(dtheta, a)) return CDLB200_ERR_ALIGNMENT;
    if (scalars && (!workspace || workspace_bytes < cdlb200_ecdl_bwd_workspace_bytes(rows, nb, format)))
        return CDLB200_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const EcdlFormat f = ecdl_format(format);
    const int64_t npairs = rows * nb * f.tpb / 2;
    const int grid = ecdl_grid(npairs);
    float* part = scalars ? static_cast<float*>(workspace) : nullptr;
    if (theta_f32)
        ecdl_bwd_kernel<float><<<grid, kEcdlThreads, 0, st>>>(
            static_cast<const float*>(grad), static_cast<const float*>(theta), npairs, format, topk,
            static_cast<const uint8_t*>(scale), kappa, alpha, static_cast<float*>(dtheta), part);
    else
        ecdl_bwd_kernel<uint16_t><<<grid, kEcdlThreads, 0, st>>>(
            static_cast<const uint16_t*>(grad), static_cast<const uint16_t*>(theta), npairs, format, topk,
            static_cast<const uint8_t*>(scale), kappa, alpha, static_cast<uint16_t*>(dtheta), part);
    CDLB200_CHECK_LAUNCH();
    if (scalars) {
        ecdl_sum_kernel<<<1, 256, 0, st>>>(part, grid, scalars);
        CDLB200_CHECK_LAUNCH();
    }
    return CDLB200_OK;
}

extern "C" int cdlb200_ccdl_fwd(const void* theta, int theta_f32, int64_t rows, int64_t nb, int format, const float* q,
                                int64_t q_stride, const float* kappa_t, const float* kappa_q, const float* alpha,
                                const int64_t* seed, int theta_topk, int q_topk, void* packed, void* scale,
                                void* stream) {
    int rc = ecdl_check(rows, nb, format, theta_topk);
    if (rc != CDLB200_OK) return rc;
    if (q_topk < 1 || q_topk > (format == CDLB200_ECDL_NVFP4 ? 126 : 255)) return CDLB200_ERR_INVALID_ARG;
    if (q_stride != 0 && q_stride != nb) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || nb == 0) return CDLB200_OK;
    if (!theta || !q || !kappa_t || !kappa_q || !alpha || !seed || !packed || !scale) return CDLB200_ERR_INVALID_ARG;
    if (!ecdl_aligned(theta, theta_f32 ? 8 : 4) || !ecdl_aligned(packed, 2)) return CDLB200_ERR_ALIGNMENT;
    const EcdlFormat f = ecdl_format(format);
    CcdlArgs a;
    a.npairs = rows * nb * f.tpb / 2;
    a.k = nb * f.tpb;
    a.rows = rows;
    a.fmt = format;
    a.topk = theta_topk;
    a.q_topk = q_topk;
    a.q = q;
    a.q_stride = q_stride;
    a.kappa_t = kappa_t;
    a.kappa_q = kappa_q;
    a.alpha = alpha;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = ecdl_grid(a.npairs);
    switch (theta_topk) {  // the theta window width as a compile-time constant where common
        case 4: launch_ccdl_fwd<4>(theta, theta_f32, a, seed, packed, scale, grid, st); break;
        case 5: launch_ccdl_fwd<5>(theta, theta_f32, a, seed, packed, scale, grid, st); break;
        case 6: launch_ccdl_fwd<6>(theta, theta_f32, a, seed, packed, scale, grid, st); break;
        case 8: launch_ccdl_fwd<8>(theta, theta_f32, a, seed, packed, scale, grid, st); break;
        case 16: launch_ccdl_fwd<16>(theta, theta_f32, a, seed, packed, scale, grid, st); break;
        default: launch_ccdl_fwd<0>(theta, theta_f32, a, seed, packed, scale, grid, st); break;
    }
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int cdlb200_ccdl_round(const void* theta, int theta_f32, int64_t rows, int64_t nb, int format,
                                  const float* q, int64_t q_stride, const float* alpha, int levels_bf16,
                                  void* packed, void* scale, void* stream) {
    int rc = ecdl_check(rows, nb, format, 1);
    if (rc != CDLB200_OK) return rc;
    if (q_stride != 0 && q_stride != nb) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || nb == 0) return CDLB200_OK;
    if (!theta || !q || !alpha || !packed || !scale) return CDLB200_ERR_INVALID_ARG;
    if (!ecdl_aligned(theta, theta_f32 ? 8 : 4) || !ecdl_aligned(packed, 2)) return CDLB200_ERR_ALIGNMENT;
    const EcdlFormat f = ecdl_format(format);
    CcdlArgs a{};
    a.npairs = rows * nb * f.tpb / 2;
    a.k = nb * f.tpb;
    a.rows = rows;
    a.fmt = format;
    a.q = q;
    a.q_stride = q_stride;
    a.alpha = alpha;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = ecdl_grid(a.npairs);
    if (theta_f32)
        ccdl_round_kernel<float><<<grid, kEcdlThreads, 0, st>>>(static_cast<const float*>(theta), a, levels_bf16 != 0,
                                                                static_cast<uint8_t*>(packed),
                                                                static_cast<uint8_t*>(scale));
    else
        ccdl_round_kernel<uint16_t><<<grid, kEcdlThreads, 0, st>>>(static_cast<const uint16_t*>(theta), a,
                                                                   levels_bf16 != 0, static_cast<uint8_t*>(packed),
                                                                   static_cast<uint8_t*>(scale));
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int64_t cdlb200_ccdl_bwd_workspace_bytes(int64_t rows, int64_t nb, int format) {
    if (ecdl_check(rows, nb, format, 1) != CDLB200_OK || rows == 0 || nb == 0) return 0;
    const EcdlFormat f = ecdl_format(format);
    return (int64_t)ecdl_grid(rows * nb * f.tpb / 2) * 3 * (int64_t)sizeof(float);
}

extern "C" int cdlb200_ccdl_bwd(const void* grad, const void* theta, int theta_f32, int64_t rows, int64_t nb,
                                int format, const float* q, int64_t q_stride, const void* scale,
                                int64_t scale_stride, const float* kappa_t, const float* kappa_q, const float* alpha,
                                int theta_topk, int q_topk, void* dtheta, float* dq, float* scalars,
                                void* workspace, int64_t workspace_bytes, void* stream) {
    int rc = ecdl_check(rows, nb, format, theta_topk);
    if (rc != CDLB200_OK) return rc;
    if (q_topk < 1 || q_topk > (format == CDLB200_ECDL_NVFP4 ? 126 : 255)) return CDLB200_ERR_INVALID_ARG;
    if ((q_stride != 0 && q_stride != nb) || (scale_stride != 0 && scale_stride != nb)) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0 || nb == 0) return CDLB200_OK;
    if (!grad || !theta || !q || !scale || !kappa_t || !kappa_q || !alpha || !dtheta) return CDLB200_ERR_INVALID_ARG;
    const int al = theta_f32 ? 8 : 4;
    if (!ecdl_aligned(grad, al) || !ecdl_aligned(theta, al) || !ecdl_aligned(dtheta, al)) return CDLB200_ERR_ALIGNMENT;
    if (scalars && (!workspace || workspace_bytes < cdlb200_ccdl_bwd_workspace_bytes(rows, nb, format)))
        return CDLB200_ERR_WORKSPACE;
    const EcdlFormat f = ecdl_format(format);
    CcdlArgs a;
    a.npairs = rows * nb * f.tpb / 2;
    a.k = nb * f.tpb;
    a.rows = rows;
    a.fmt = format;
    a.topk = theta_topk;
    a.q_topk = q_topk;
    a.q = q;
    a.q_stride = q_stride;
    a.kappa_t = kappa_t;
    a.kappa_q = kappa_q;
    a.alpha = alpha;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = ecdl_grid(a.npairs);
    float* part = scalars ? static_cast<float*>(workspace) : nullptr;
    if (theta_f32)
        ccdl_bwd_kernel<float><<<grid, kEcdlThreads, 0, st>>>(
            static_cast<const float*>(grad), static_cast<const float*>(theta), a, static_cast<const uint8_t*>(scale),
            scale_stride, static_cast<float*>(dtheta), dq, part);
    else
        ccdl_bwd_kernel<uint16_t><<<grid, kEcdlThreads, 0, st>>>(
            static_cast<const uint16_t*>(grad), static_cast<const uint16_t*>(theta), a,
            static_cast<const uint8_t*>(scale), scale_stride, static_cast<uint16_t*>(dtheta), dq, part);
    CDLB200_CHECK_LAUNCH();
    if (scalars) {
        ccdl_sum_kernel<<<1, 32, 0, st>>>(part, grid, scalars);
        CDLB200_CHECK_LAUNCH();
    }
    return CDLB200_OK;
}
