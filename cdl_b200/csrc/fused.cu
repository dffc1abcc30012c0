// fused.cu -- the elementwise parts of the SmolLM2 (Llama) QAT step, one
// memory pass each, following the rounding steps of the eager reference
// modules so that the results stay within bf16 rounding of them:
//
//   RMSNorm   y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))        (x -> fp32 first)
//   RoPE      out = bf16(bf16(q * cos) + bf16(rot(q) * sin)),  rot(q) = (-q[D/2:], q[:D/2])
//   SwiGLU    h = bf16(bf16(silu(g)) * u)
//
// and their backward passes (the gradients autograd forms for those modules,
// with fp32 intermediates).  All tensors are bf16, row-major, 16-byte aligned
// rows; each thread moves 8 values (16 bytes) at a time.
#include "cdlb200_step.h"
#include "common.cuh"

namespace cdlb200 {
namespace {

__device__ __forceinline__ float bf_lo(uint32_t w) { return u2f(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return u2f(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ float rbf(float v) {  // round to bf16 and back
    return u2f(pack_bf2(v, 0.f) << 16);
}
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
    f[0] = bf_lo(v.x), f[1] = bf_hi(v.x), f[2] = bf_lo(v.y), f[3] = bf_hi(v.y);
    f[4] = bf_lo(v.z), f[5] = bf_hi(v.z), f[6] = bf_lo(v.w), f[7] = bf_hi(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(pack_bf2(f[0], f[1]), pack_bf2(f[2], f[3]), pack_bf2(f[4], f[5]), pack_bf2(f[6], f[7]));
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// running max of bf16 magnitudes, two lanes per word: acc = max(acc, |v|)
__device__ __forceinline__ uint32_t mag8(uint32_t acc, const uint4& v) {
    uint32_t a, b;
    asm("max.u16x2 %0, %1, %2;" : "=r"(a) : "r"(v.x & 0x7fff7fffu), "r"(v.y & 0x7fff7fffu));
    asm("max.u16x2 %0, %1, %2;" : "=r"(b) : "r"(v.z & 0x7fff7fffu), "r"(v.w & 0x7fff7fffu));
    asm("max.u16x2 %0, %1, %2;" : "=r"(a) : "r"(a), "r"(b));
    asm("max.u16x2 %0, %1, %2;" : "=r"(acc) : "r"(acc), "r"(a));
    return acc;
}

// Folds each thread's two-lane running max `m2` into *amax (one atomic per
// CTA); all threads call it.
__device__ __forceinline__ void cta_amax(uint32_t m2, uint32_t* amax) {
    __shared__ uint32_t red[32];
    uint32_t m = __reduce_max_sync(0xffffffffu, max(m2 & 0xffffu, m2 >> 16));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = max(m, red[w]);
        atomicMax(amax + (blockIdx.x % CDLB200_AMAX_WORDS), m);  // spread: same-address atomics serialize
    }
}

// cta_amax for two outputs at once (one shared round trip); null pointers skip
__device__ __forceinline__ void cta_amax2(uint32_t m2a, uint32_t* amax_a, uint32_t m2b, uint32_t* amax_b) {
    __shared__ uint32_t red[2][32];
    uint32_t ma = __reduce_max_sync(0xffffffffu, max(m2a & 0xffffu, m2a >> 16));
    uint32_t mb = __reduce_max_sync(0xffffffffu, max(m2b & 0xffffu, m2b >> 16));
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = ma;
        red[1][threadIdx.x >> 5] = mb;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            ma = max(ma, red[0][w]);
            mb = max(mb, red[1][w]);
        }
        if (amax_a) atomicMax(amax_a + (blockIdx.x % CDLB200_AMAX_WORDS), ma);
        if (amax_b) atomicMax(amax_b + (blockIdx.x % CDLB200_AMAX_WORDS), mb);
    }
}

// ---------------------------------------------------------------------------
// RMSNorm over rows of d = 8 * nvec bf16 values.  W warps (1, 2 or 4) share a
// row: lane l of warp w owns the 8-value vectors (32 w + l) + 32 W j, j < VPL;
// a 256-thread CTA holds R = 8 / W rows at a time.  Few registers per thread,
// so that many CTAs per SM keep enough loads in flight for HBM.  The row sums
// are reduced per warp with shuffles, then over the row's W warps in a fixed
// order through shared memory.
// ---------------------------------------------------------------------------
struct RowSplit {
    int W, R;  // warps per row, rows per CTA pass
};

__device__ __forceinline__ float row_sum(float v, float (*red)[4], int slot, int wr, int W) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[slot][wr] = v;
    __syncthreads();
    float t = 0.f;
    for (int k = 0; k < W; ++k) t += red[slot][k];
    __syncthreads();  // red is reused by the next row pass
    return t;
}

// With `res`, the normalized row is h = bf16(x + res) (the decoder's residual
// add, as torch adds two bf16 tensors), which is also written to `hout`.
template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const uint4* __restrict__ x, const uint4* __restrict__ w,
                                                          int64_t rows, int nvec, float eps, uint4* __restrict__ y,
                                                          float* __restrict__ rstd, uint32_t* __restrict__ amax,
                                                          const uint4* __restrict__ res, uint4* __restrict__ hout,
                                                          RowSplit rsp) {
    __shared__ float red[8][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = warp / rsp.W, wr = warp - slot * rsp.W;
    uint32_t am = 0;  // max |y| as bf16 magnitude bits (the NVFP4 global amax of the output)
    // the next row's x and residual are loaded while this row is reduced
    const int64_t step = (int64_t)gridDim.x * rsp.R;
    uint4 nx[VPL], nres[VPL];
    auto load_row = [&](int64_t r) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int c = 32 * wr + lane + 32 * rsp.W * j;
            const bool in = r < rows && c < nvec;
            nx[j] = in ? x[r * nvec + c] : make_uint4(0u, 0u, 0u, 0u);
            nres[j] = in && res != nullptr ? res[r * nvec + c] : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    load_row((int64_t)blockIdx.x * rsp.R + slot);
    for (int64_t base = (int64_t)blockIdx.x * rsp.R; base < rows; base += step) {
        const int64_t r = base + slot;
        const bool live = r < rows;
        uint4 v[VPL], rv[VPL];
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            v[j] = nx[j];
            rv[j] = nres[j];
        }
        load_row(base + step + slot);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int c = 32 * wr + lane + 32 * rsp.W * j;
            const bool in = live && c < nvec;
            float f[8];
            unpack8(v[j], f);
            if (res != nullptr && in) {
                float b[8];
                unpack8(rv[j], b);
#pragma unroll
                for (int i = 0; i < 8; ++i) f[i] += b[i];
                v[j] = pack8(f);
                hout[r * nvec + c] = v[j];
                unpack8(v[j], f);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
        }
        ss = row_sum(ss, red, slot, wr, rsp.W);
        const float rs = rsqrtf(ss / (float)(8 * nvec) + eps);
        if (live && wr == 0 && lane == 0) rstd[r] = rs;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int c = 32 * wr + lane + 32 * rsp.W * j;
            if (!live || c >= nvec) continue;
            float f[8], g[8];
            unpack8(v[j], f);
            unpack8(w[c], g);
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = g[i] * rbf(f[i] * rs);
            const uint4 o = pack8(f);
            y[r * nvec + c] = o;
            am = mag8(am, o);
        }
    }
    if (amax) cta_amax(am, amax);
}

// dx = bf16(rs * g1 - x * rs^3 * sum(g1 * x) / d) with g1 = bf16(dy * w);
// dw partial sums (fp32, one row of `part` per CTA) of dy * bf16(x * rs).
// With `dres`, dx = bf16(dx + dres): the gradient the residual branch adds
// (autograd's sum of the two bf16 gradients of the residual input); `amax`
// (optional) receives the bf16 magnitude maximum of dx.
template <int VPL>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const uint4* __restrict__ dy, const uint4* __restrict__ x,
                                                          const uint4* __restrict__ w, const float* __restrict__ rstd,
                                                          int64_t rows, int nvec, uint4* __restrict__ dx,
                                                          float* __restrict__ part, const uint4* __restrict__ dres,
                                                          uint32_t* __restrict__ amax, RowSplit rsp) {
    extern __shared__ float dw_s[];  // [8 * nvec]
    __shared__ float red[8][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = warp / rsp.W, wr = warp - slot * rsp.W;
    for (int i = threadIdx.x; i < 8 * nvec; i += blockDim.x) dw_s[i] = 0.f;
    __syncthreads();
    float acc[VPL][8];
#pragma unroll
    for (int j = 0; j < VPL; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[j][i] = 0.f;
    const float inv_d = 1.0f / (float)(8 * nvec);
    uint32_t am = 0;
    for (int64_t base = (int64_t)blockIdx.x * rsp.R; base < rows; base += (int64_t)gridDim.x * rsp.R) {
        const int64_t r = base + slot;
        const bool live = r < rows;
        const float rs = live ? rstd[r] : 0.f;
        uint4 xv[VPL], dv[VPL];  // the row stays in registers as bf16; fp32 values are recomputed
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int c = 32 * wr + lane + 32 * rsp.W * j;
            const bool in = live && c < nvec;
            xv[j] = in ? x[r * nvec + c] : make_uint4(0u, 0u, 0u, 0u);
            dv[j] = in ? dy[r * nvec + c] : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int c = 32 * wr + lane + 32 * rsp.W * j;
            if (!live || c >= nvec) continue;
            float xf[8], d8[8], w8[8];
            unpack8(xv[j], xf);
            unpack8(dv[j], d8);
            unpack8(w[c], w8);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                dot = fmaf(rbf(d8[i] * w8[i]), xf[i], dot);
                acc[j][i] = fmaf(d8[i], rbf(xf[i] * rs), acc[j][i]);
            }
        }
        dot = row_sum(dot, red, slot, wr, rsp.W);
        const float k = rs * rs * rs * dot * inv_d;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const int c = 32 * wr + lane + 32 * rsp.W * j;
            if (!live || c >= nvec) continue;
            float xf[8], d8[8], w8[8], o[8];
            unpack8(xv[j], xf);
            unpack8(dv[j], d8);
            unpack8(w[c], w8);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = rs * rbf(d8[i] * w8[i]) - xf[i] * k;
            if (dres != nullptr) {
                float r8[8];
                unpack8(dres[r * nvec + c], r8);
#pragma unroll
                for (int i = 0; i < 8; ++i) o[i] = rbf(o[i]) + r8[i];
            }
            const uint4 ov = pack8(o);
            dx[r * nvec + c] = ov;
            am = mag8(am, ov);
        }
    }
    // the row slots fold their column sums in slot order (not with shared
    // atomics), so the fp32 partials, and dw, are the same on every run;
    // within a slot the warps own disjoint columns
    for (int s = 0; s < rsp.R; ++s) {
        if (slot == s) {
#pragma unroll
            for (int j = 0; j < VPL; ++j) {
                const int c = 32 * wr + lane + 32 * rsp.W * j;
                if (c >= nvec) continue;
#pragma unroll
                for (int i = 0; i < 8; ++i) dw_s[8 * c + i] += acc[j][i];
            }
        }
        __syncthreads();
    }
    for (int i = threadIdx.x; i < 8 * nvec; i += blockDim.x) part[(int64_t)blockIdx.x * 8 * nvec + i] = dw_s[i];
    if (amax) cta_amax(am, amax);
}

// dw[i] = bf16(sum over the CTA partials): a CTA per 32 columns, its 8 warps
// splitting the partials.
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ part, int nparts, int d,
                                                     uint16_t* __restrict__ dw) {
    __shared__ float red[8][33];
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int i = blockIdx.x * 32 + lane;
    float s = 0.f;
    if (i < d)
        for (int p = wp; p < nparts; p += 8) s += part[(int64_t)p * d + i];
    red[wp][lane] = s;
    __syncthreads();
    if (wp == 0) {
        float t = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) t += red[k][lane];
        if (i < d) dw[i] = (uint16_t)(pack_bf2(t, 0.f) & 0xffffu);
    }
}

// ---------------------------------------------------------------------------
// RoPE on x[tokens, heads, D] (D = 8 * 2 * halfv), cos/sin[cos_tokens, D],
// token t using row t % cos_tokens (a batch sharing one position table).  One
// thread per (token, head, 8-value vector of the first half) handles that
// vector and its partner in the second half.
// ---------------------------------------------------------------------------
// Index math: 32-bit multiply-shift divisions (FastDiv) when the item count
// is below 2^31 (FAST), else 64-bit divisions.
struct RopeDivs {
    FastDiv halfv, heads, cos_tokens;
};

template <bool FAST>
__global__ void __launch_bounds__(256) rope_kernel(const uint4* __restrict__ x, const uint4* __restrict__ cosv,
                                                   const uint4* __restrict__ sinv, int64_t tokens, int heads,
                                                   int halfv, int64_t cos_tokens, int backward,
                                                   uint4* __restrict__ out, uint32_t* __restrict__ amax,
                                                   RopeDivs dv) {
    const int64_t total = tokens * heads * halfv;
    uint32_t am = 0;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
        int v;
        int64_t th, tok;  // (token, head) row and the token's cos/sin row (repeating every cos_tokens)
        if constexpr (FAST) {
            const uint32_t t32 = (uint32_t)t, th32 = dv.halfv.div(t32), tk = dv.heads.div(th32);
            v = (int)(t32 - th32 * dv.halfv.d);
            th = th32;
            tok = tk - dv.cos_tokens.div(tk) * dv.cos_tokens.d;
        } else {
            v = (int)(t % halfv);
            th = t / halfv;
            tok = (th / heads) % cos_tokens;
        }
        const int64_t base = th * 2 * halfv;
        float a[8], b[8], c1[8], c2[8], s1[8], s2[8], o1[8], o2[8];
        unpack8(x[base + v], a);
        unpack8(x[base + halfv + v], b);
        unpack8(cosv[tok * 2 * halfv + v], c1);
        unpack8(cosv[tok * 2 * halfv + halfv + v], c2);
        unpack8(sinv[tok * 2 * halfv + v], s1);
        unpack8(sinv[tok * 2 * halfv + halfv + v], s2);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (!backward) {  // (x*cos) + (rot(x)*sin), rot(x) = (-b, a)
                o1[i] = rbf(a[i] * c1[i]) - rbf(b[i] * s1[i]);
                o2[i] = rbf(b[i] * c2[i]) + rbf(a[i] * s2[i]);
            } else {  // g*cos + rot^T(g*sin), rot^T(u) = (u2, -u1)
                o1[i] = rbf(a[i] * c1[i]) + rbf(b[i] * s2[i]);
                o2[i] = rbf(b[i] * c2[i]) - rbf(a[i] * s1[i]);
            }
        }
        const uint4 p1 = pack8(o1), p2 = pack8(o2);
        out[base + v] = p1;
        out[base + halfv + v] = p2;
        am = mag8(mag8(am, p1), p2);
    }
    if (amax) cta_amax(am, amax);
}

// ---------------------------------------------------------------------------
// SwiGLU: h = bf16(bf16(silu(g)) * u); backward with s = sigmoid(g):
//   dsilu = bf16(dh * u), du = bf16(dh * bf16(silu(g))),
//   dg = bf16(dsilu * s * (1 + g * (1 - s)))
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoid_f(float g) { return 1.0f / (1.0f + expf(-g)); }

__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const uint4* __restrict__ g, const uint4* __restrict__ u,
                                                         int64_t nvec, uint4* __restrict__ h, uint32_t* __restrict__ amax) {
    // two vectors per thread and iteration (t and t + stride), both loaded
    // before either is computed
    uint32_t am = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += 2 * stride) {
        const bool two = t + stride < nvec;
        uint4 gv[2], uv[2];
        gv[0] = g[t];
        uv[0] = u[t];
        if (two) {
            gv[1] = g[t + stride];
            uv[1] = u[t + stride];
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (k == 1 && !two) break;
            float a[8], b[8];
            unpack8(gv[k], a);
            unpack8(uv[k], b);
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = rbf(a[i] * sigmoid_f(a[i])) * b[i];
            const uint4 o = pack8(a);
            h[t + k * stride] = o;
            am = mag8(am, o);
        }
    }
    if (amax) cta_amax(am, amax);
}

__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const uint4* __restrict__ dh, const uint4* __restrict__ g,
                                                         const uint4* __restrict__ u, int64_t nvec,
                                                         uint4* __restrict__ dg, uint4* __restrict__ du,
                                                         uint32_t* __restrict__ amax_g, uint32_t* __restrict__ amax_u) {
    uint32_t ag = 0, au = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += 2 * stride) {
        const bool two = t + stride < nvec;
        uint4 dv[2], gv[2], uv[2];
        dv[0] = dh[t];
        gv[0] = g[t];
        uv[0] = u[t];
        if (two) {
            dv[1] = dh[t + stride];
            gv[1] = g[t + stride];
            uv[1] = u[t + stride];
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (k == 1 && !two) break;
            float d[8], a[8], b[8], og[8], ou[8];
            unpack8(dv[k], d);
            unpack8(gv[k], a);
            unpack8(uv[k], b);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float s = sigmoid_f(a[i]);
                const float ds = rbf(d[i] * b[i]);
                ou[i] = d[i] * rbf(a[i] * s);
                og[i] = ds * (s * (1.0f + a[i] * (1.0f - s)));
            }
            const uint4 pg = pack8(og), pu = pack8(ou);
            dg[t + k * stride] = pg;
            du[t + k * stride] = pu;
            ag = mag8(ag, pg);
            au = mag8(au, pu);
        }
    }
    if (amax_g || amax_u) cta_amax2(ag, amax_g, au, amax_u);
}

// ---------------------------------------------------------------------------
// Cross entropy over bf16 logits, one CTA per row, three passes over the row
// (the second and third come from L2):
//   m = max x,  lse = log(sum exp(x - m)) + m,  loss = lse - x[t],
//   x <- bf16((exp(x - lse) - [j == t]) * scale)  (in place; scale = 1/n gives
//                                                  d(sum loss / n)/dx, as torch's
//                                                  division by a scalar n does)
// A target outside [0, vocab) (an ignored position) gives loss 0 and a zero
// gradient row.
// ---------------------------------------------------------------------------
constexpr int kXentThreads = 512;

template <bool MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = MAX ? fmaxf(v, w) : v + w;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();  // red[] is reused by consecutive reductions
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = lane < kXentThreads / 32 ? red[lane] : (MAX ? -INFINITY : 0.0f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = MAX ? fmaxf(v, w) : v + w;
    }
    return v;
}

__global__ void __launch_bounds__(kXentThreads) xent_kernel(uint4* __restrict__ logits,
                                                            const int64_t* __restrict__ targets, int64_t vocab,
                                                            float scale, float* __restrict__ loss) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int nv = (int)(vocab / 8);
    uint4* x = logits + row * nv;
    const int64_t t = targets[row];
    const bool valid = t >= 0 && t < vocab;
    const float xt = valid ? bf_lo((uint32_t)reinterpret_cast<const uint16_t*>(x)[t]) : 0.0f;

    float m = -INFINITY;
    for (int i = threadIdx.x; i < nv; i += kXentThreads) {
        float f[8];
        unpack8(x[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, f[j]);
    }
    m = block_reduce<true>(m, red);
    const float mu = isinf(m) ? 0.0f : m;  // as torch.logsumexp: an infinite max is not subtracted
    float s = 0.0f;
    for (int i = threadIdx.x; i < nv; i += kXentThreads) {
        float f[8];
        unpack8(x[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) s += expf(f[j] - mu);
    }
    s = block_reduce<false>(s, red);
    const float lse = logf(s) + mu;
    if (threadIdx.x == 0) loss[row] = valid ? lse - xt : 0.0f;
    for (int i = threadIdx.x; i < nv; i += kXentThreads) {
        float f[8];
        unpack8(x[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p = valid ? expf(f[j] - lse) - (8 * (int64_t)i + j == t ? 1.0f : 0.0f) : 0.0f;
            f[j] = __fmul_rn(p, scale);
        }
        x[i] = pack8(f);
    }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int grid_for(int64_t items, int per_block) {
    const int64_t cap = (int64_t)num_sms() * 8;
    const int64_t g = (items + per_block - 1) / per_block;
    return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

// x *= s in place, as torch multiplies a bf16 tensor by a bf16 scalar (the
// fp32 product rounded to bf16); s is read on the device, and a launch whose
// s is 1 leaves x as it is without touching it (x * 1 == x for every value
// but a NaN's payload), so the multiply costs nothing in the common case.
__global__ void __launch_bounds__(256) scale_bf16_kernel(uint4* __restrict__ x, int64_t nvec,
                                                         const uint16_t* __restrict__ s) {
    const uint32_t sb = *s;
    if (sb == 0x3f80u) return;
    const float sc = __uint_as_float(sb << 16);
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < nvec; t += (int64_t)gridDim.x * blockDim.x) {
        float f[8];
        unpack8(x[t], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] *= sc;
        x[t] = pack8(f);
    }
}
}  // namespace
}  // namespace cdlb200

extern "C" int cdlb200_scale_bf16(void* x, int64_t n, const void* scale, void* stream) {
    using namespace cdlb200;
    if (n < 0 || (n % 8) != 0) return CDLB200_ERR_INVALID_ARG;
    if (n == 0) return CDLB200_OK;
    if (!x || !scale) return CDLB200_ERR_INVALID_ARG;
    if (!al16(x) || (reinterpret_cast<uintptr_t>(scale) & 1u) != 0) return CDLB200_ERR_ALIGNMENT;
    scale_bf16_kernel<<<grid_for(n / 8, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint4*>(x), n / 8, static_cast<const uint16_t*>(scale));
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

using namespace cdlb200;

namespace {
// W = the smallest power of two with 64 W >= nvec (at most 4), VPL = vectors per lane
RowSplit row_split(int nvec, int& vpl) {
    int W = 1;
    while (W < 4 && 64 * W < nvec) W *= 2;
    vpl = (nvec + 32 * W - 1) / (32 * W);
    return RowSplit{W, 8 / W};
}

int rmsnorm_fwd_launch(const void* x, const void* res, const void* w, int64_t rows, int64_t d, float eps, void* h,
                       void* y, float* rstd, uint32_t* amax, void* stream) {
    if (rows < 0 || d <= 0 || (d % 8) != 0 || d > 8 * 32 * 8) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0) return CDLB200_OK;
    if (!x || !w || !y || !rstd || (res != nullptr) != (h != nullptr)) return CDLB200_ERR_INVALID_ARG;
    if (!al16(x) || !al16(w) || !al16(y) || !al16(res) || !al16(h)) return CDLB200_ERR_ALIGNMENT;
    const int nvec = (int)(d / 8);
    int vpl = 1;
    const RowSplit rsp = row_split(nvec, vpl);
    const int grid = grid_for(rows, rsp.R);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto args = [&](auto kern) {
        kern<<<grid, 256, 0, st>>>(static_cast<const uint4*>(x), static_cast<const uint4*>(w), rows, nvec, eps,
                                   static_cast<uint4*>(y), rstd, amax, static_cast<const uint4*>(res),
                                   static_cast<uint4*>(h), rsp);
    };
    if (vpl <= 1) args(rmsnorm_fwd_kernel<1>);
    else args(rmsnorm_fwd_kernel<2>);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}
}  // namespace

extern "C" int cdlb200_rmsnorm_fwd(const void* x, const void* w, int64_t rows, int64_t d, float eps, void* y,
                                   float* rstd, uint32_t* amax, void* stream) {
    return rmsnorm_fwd_launch(x, nullptr, w, rows, d, eps, nullptr, y, rstd, amax, stream);
}

extern "C" int cdlb200_add_rmsnorm_fwd(const void* res, const void* x, const void* w, int64_t rows, int64_t d,
                                       float eps, void* h, void* y, float* rstd, uint32_t* amax, void* stream) {
    if (rows > 0 && (!res || !h)) return CDLB200_ERR_INVALID_ARG;
    return rmsnorm_fwd_launch(x, res, w, rows, d, eps, h, y, rstd, amax, stream);
}

// the backward runs one persistent CTA per SM (each accumulates its rows' dw
// in registers, then once into shared memory and one partial row)
// the backward keeps each CTA's dw in registers and writes one partial row per
// CTA: 4 CTAs per SM at most (for 2048 columns, 4.8 MB of partials)
static int bwd_grid(int64_t rows, int64_t d) {
    int vpl = 1;
    const RowSplit rsp = row_split((int)(d / 8), vpl);
    const int64_t g = (rows + rsp.R - 1) / rsp.R, cap = 4 * (int64_t)num_sms();
    return (int)(g < 1 ? 1 : (g < cap ? g : cap));
}

extern "C" int64_t cdlb200_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t d) {
    if (rows <= 0 || d <= 0) return 0;
    return (int64_t)bwd_grid(rows, d) * d * (int64_t)sizeof(float);
}

extern "C" int cdlb200_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, int64_t rows,
                                   int64_t d, void* dx, void* dw, void* workspace, int64_t workspace_bytes,
                                   void* stream) {
    return cdlb200_rmsnorm_bwd_add(dy, x, w, rstd, nullptr, rows, d, dx, dw, nullptr, workspace, workspace_bytes,
                                   stream);
}

extern "C" int cdlb200_rmsnorm_bwd_add(const void* dy, const void* x, const void* w, const float* rstd,
                                       const void* dres, int64_t rows, int64_t d, void* dx, void* dw, uint32_t* amax,
                                       void* workspace, int64_t workspace_bytes, void* stream) {
    if (rows < 0 || d <= 0 || (d % 8) != 0 || d > 8 * 32 * 8) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0) return CDLB200_OK;
    if (!dy || !x || !w || !rstd || !dx || !dw || !workspace) return CDLB200_ERR_INVALID_ARG;
    if (!al16(dy) || !al16(x) || !al16(w) || !al16(dx) || !al16(dres)) return CDLB200_ERR_ALIGNMENT;
    if (workspace_bytes < cdlb200_rmsnorm_bwd_workspace_bytes(rows, d)) return CDLB200_ERR_WORKSPACE;
    const int nvec = (int)(d / 8);
    int vpl = 1;
    const RowSplit rsp = row_split(nvec, vpl);
    const int grid = bwd_grid(rows, d);
    const size_t smem = (size_t)d * sizeof(float);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = static_cast<float*>(workspace);
    auto args = [&](auto kern) {
        kern<<<grid, 256, smem, st>>>(static_cast<const uint4*>(dy), static_cast<const uint4*>(x),
                                      static_cast<const uint4*>(w), rstd, rows, nvec, static_cast<uint4*>(dx), part,
                                      static_cast<const uint4*>(dres), amax, rsp);
    };
    if (vpl <= 1) args(rmsnorm_bwd_kernel<1>);
    else args(rmsnorm_bwd_kernel<2>);
    CDLB200_CHECK_LAUNCH();
    colsum_kernel<<<(unsigned)((d + 31) / 32), 256, 0, st>>>(part, grid, (int)d, static_cast<uint16_t*>(dw));
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int cdlb200_rope(const void* x, const void* cos, const void* sin, int64_t tokens, int64_t heads,
                            int64_t head_dim, int64_t cos_tokens, int backward, void* out, uint32_t* amax,
                            void* stream) {
    if (tokens < 0 || heads <= 0 || head_dim <= 0 || (head_dim % 16) != 0 || (backward != 0 && backward != 1) ||
        cos_tokens <= 0)
        return CDLB200_ERR_INVALID_ARG;
    if (tokens == 0) return CDLB200_OK;
    if (!x || !cos || !sin || !out) return CDLB200_ERR_INVALID_ARG;
    if (!al16(x) || !al16(cos) || !al16(sin) || !al16(out)) return CDLB200_ERR_ALIGNMENT;
    const int halfv = (int)(head_dim / 16);
    const int64_t items = tokens * heads * halfv;
    const RopeDivs dv{FastDiv((uint32_t)halfv), FastDiv((uint32_t)(heads < (1ll << 31) ? heads : 1)),
                      FastDiv((uint32_t)(cos_tokens < (1ll << 31) ? cos_tokens : 1))};
    auto launch = [&](auto kern) {
        kern<<<grid_for(items, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const uint4*>(x), static_cast<const uint4*>(cos), static_cast<const uint4*>(sin), tokens,
            (int)heads, halfv, cos_tokens, backward, static_cast<uint4*>(out), amax, dv);
    };
    if (items < (1ll << 31) && cos_tokens < (1ll << 31)) launch(rope_kernel<true>);
    else launch(rope_kernel<false>);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int cdlb200_swiglu_fwd(const void* g, const void* u, int64_t n, void* h, uint32_t* amax, void* stream) {
    if (n < 0 || (n % 8) != 0) return CDLB200_ERR_INVALID_ARG;
    if (n == 0) return CDLB200_OK;
    if (!g || !u || !h) return CDLB200_ERR_INVALID_ARG;
    if (!al16(g) || !al16(u) || !al16(h)) return CDLB200_ERR_ALIGNMENT;
    swiglu_fwd_kernel<<<grid_for(n / 8, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(g), static_cast<const uint4*>(u), n / 8, static_cast<uint4*>(h), amax);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int cdlb200_swiglu_bwd(const void* dh, const void* g, const void* u, int64_t n, void* dg, void* du,
                                  uint32_t* amax_dg, uint32_t* amax_du, void* stream) {
    if (n < 0 || (n % 8) != 0) return CDLB200_ERR_INVALID_ARG;
    if (n == 0) return CDLB200_OK;
    if (!dh || !g || !u || !dg || !du) return CDLB200_ERR_INVALID_ARG;
    if (!al16(dh) || !al16(g) || !al16(u) || !al16(dg) || !al16(du)) return CDLB200_ERR_ALIGNMENT;
    swiglu_bwd_kernel<<<grid_for(n / 8, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(dh), static_cast<const uint4*>(g), static_cast<const uint4*>(u), n / 8,
        static_cast<uint4*>(dg), static_cast<uint4*>(du), amax_dg, amax_du);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

extern "C" int cdlb200_cross_entropy(void* logits, const int64_t* targets, int64_t rows, int64_t vocab,
                                     float scale, float* loss, void* stream) {
    if (rows < 0 || vocab <= 0 || (vocab % 8) != 0) return CDLB200_ERR_INVALID_ARG;
    if (rows == 0) return CDLB200_OK;
    if (!logits || !targets || !loss) return CDLB200_ERR_INVALID_ARG;
    if (!al16(logits)) return CDLB200_ERR_ALIGNMENT;
    if (rows > 0x7fffffffLL) return CDLB200_ERR_INVALID_ARG;
    xent_kernel<<<(unsigned)rows, kXentThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint4*>(logits), targets, vocab, scale, loss);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}
