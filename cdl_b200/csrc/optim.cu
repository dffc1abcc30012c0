// optim.cu -- gradient-norm clipping and AdamW for the QAT step.
//
// The reference's step (cdl smollm2.py) calls torch.nn.utils.clip_grad_norm_
// and then torch.optim.AdamW: a per-tensor norm pass, a stack + norm, an
// in-place multiply of every gradient, then the optimizer pass.  Here the
// whole thing is three launches per group of up to kOptGroup tensors, and the
// gradients are read twice in total (norm, update) and never written:
//
//   sumsq     every work chunk (kOptChunk elements of one tensor) -> one fp32
//             sum of squares in the workspace (fixed order: deterministic)
//   finalize  one CTA: per-tensor norms (a warp per tensor, fixed-order
//             reduction), rounded to bf16 as torch's per-tensor norms are, the
//             total norm, the clip coefficient and the bias corrections of the
//             next step, all into a scalar block in the workspace
//   adamw     g = bf16(grad * coef), then torch's foreach AdamW sequence
//             per element (every step rounded to bf16 as the list
//             operations store it), p/m/v written back
//
// The tensor table (pointers, sizes, chunk offsets) travels in the kernel
// parameter block, so a launch needs no host-to-device copy and the sequence
// can be captured in a CUDA graph as is.
#include <vector>

#include "common.cuh"
#include "cdlb200_step.h"

namespace cdlb200 {
namespace {

constexpr int kOptChunk = 16384;  // elements of one work chunk (a tensor's last chunk may be shorter)
constexpr int kOptThreads = 256;  // each thread moves 8 bf16 (16 bytes) per access
constexpr int kOptGroup = 512;    // tensors per launch (the table is a kernel parameter, < 25 KB of the 32 KB)

struct OptGroup {
    int count;                       // tensors in this group
    int pad;
    int64_t chunk0[kOptGroup + 1];   // global index of each tensor's first chunk; chunk0[count] = end
    cdlb200_adamw_tensor t[kOptGroup];
};

// Scalars shared by the three kernels, at the start of the workspace.  The
// step counter persists between calls (the workspace starts zero-filled).
struct OptScalars {
    float step;       // completed steps
    float sumsq;      // running sum of the squared bf16 per-tensor norms
    float norm;       // bf16(total norm)
    float coef;       // clip coefficient
    float step_size;  // -lr / (1 - beta1^step), rounded to fp32
    float bc2s;       // sqrt(1 - beta2^step), rounded to fp32
    float pad[2];
};
constexpr int64_t kScalarBytes = 64;

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float bf_round(float v) { return u2f(pack2(v, 0.f) << 16); }

// tensor of global chunk c (the group's chunk0 is increasing; empty tensors
// are never in a group)
__device__ __forceinline__ int tensor_of(const OptGroup& g, int64_t c) {
    int lo = 0, hi = g.count - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (g.chunk0[mid] <= c) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__global__ void __launch_bounds__(kOptThreads) sumsq_kernel(const __grid_constant__ OptGroup g,
                                                            float* __restrict__ partial) {
    __shared__ float red[kOptThreads / 32];
    const int tid = threadIdx.x;
    for (int64_t c = g.chunk0[0] + blockIdx.x; c < g.chunk0[g.count]; c += gridDim.x) {
        const int ti = tensor_of(g, c);
        const int64_t base = (c - g.chunk0[ti]) * kOptChunk;
        const int64_t left = g.t[ti].numel - base;
        const int nv = (int)((left < kOptChunk ? left : kOptChunk) / 8);
        const uint4* src = static_cast<const uint4*>(g.t[ti].grad) + base / 8;
        uint4 v[kOptChunk / 8 / kOptThreads];
#pragma unroll
        for (int u = 0; u < kOptChunk / 8 / kOptThreads; ++u) {
            const int i = u * kOptThreads + tid;
            v[u] = i < nv ? ldg_stream(src + i) : make_uint4(0u, 0u, 0u, 0u);
        }
        float s = 0.f;
#pragma unroll
        for (int u = 0; u < kOptChunk / 8 / kOptThreads; ++u) {
            const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float lo = bf16lo(w[j]), hi = bf16hi(w[j]);
                s = __fmaf_rn(lo, lo, s);
                s = __fmaf_rn(hi, hi, s);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if ((tid & 31) == 0) red[tid >> 5] = s;
        __syncthreads();
        if (tid == 0) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kOptThreads / 32; ++w) t += red[w];
            partial[c] = t;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(1024) finalize_kernel(const __grid_constant__ OptGroup g,
                                                        const float* __restrict__ partial, OptScalars* sc,
                                                        int first, int last, float max_norm, double lr, double beta1,
                                                        double beta2, float* grad_norm) {
    __shared__ float nrm[kOptGroup];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // the update kernel folds each tensor's new max|param| into its amax word
    for (int ti = threadIdx.x; ti < g.count; ti += blockDim.x)
        if (g.t[ti].amax) *g.t[ti].amax = 0u;
    for (int ti = warp; ti < g.count; ti += 32) {
        float s = 0.f;
        for (int64_t c = g.chunk0[ti] + lane; c < g.chunk0[ti + 1]; c += 32) s += partial[c];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) nrm[ti] = bf_round(sqrtf(s));  // torch._foreach_norm of a bf16 tensor is bf16
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    float acc = first ? 0.f : sc->sumsq;
    for (int ti = 0; ti < g.count; ++ti) acc = __fmaf_rn(nrm[ti], nrm[ti], acc);
    sc->sumsq = acc;
    if (!last) return;
    const float norm = bf_round(sqrtf(acc));  // vector_norm of the stacked bf16 norms, bf16 result
    float coef = 1.0f;
    if (max_norm > 0.f && max_norm <= 3.4028234e38f) {
        // max_norm / (norm + 1e-6) on a bf16 tensor: torch evaluates the
        // reversed division as reciprocal(x) * max_norm, each rounded to bf16
        const float r = bf_round(__fdiv_rn(1.0f, bf_round(norm + 1e-6f)));
        const float cf = bf_round(__fmul_rn(r, max_norm));
        coef = cf > 1.0f ? 1.0f : cf;  // clamp(max=1): a NaN coefficient passes through, as in torch
    }
    const float step = sc->step + 1.0f;
    const double bc1 = 1.0 - pow(beta1, (double)step);
    const double bc2 = 1.0 - pow(beta2, (double)step);
    sc->step = step;
    sc->norm = norm;
    sc->coef = coef;
    sc->step_size = (float)(-(lr / bc1));
    sc->bc2s = (float)sqrt(bc2);
    if (grad_norm) *grad_norm = norm;
}

// The update follows, per element and in order, the foreach AdamW torch runs
// for bf16 parameters on CUDA (torch.optim.AdamW's default, which cdl's
// training script uses): every list operation computes in fp32 with its
// scalar in fp32 and stores bf16.
//   p = bf16(p * (1 - lr*wd))                     _foreach_mul_
//   m = bf16(m + w1 * (g - m))                    _foreach_lerp_ (w1 = 1 - b1 < 0.5)
//   v = bf16(v * b2);  v = bf16(v + c2 * (g*g))   _foreach_mul_, _foreach_addcmul_
//   s = bf16(sqrt(v)); s = bf16(s / bc2s); s = bf16(s + eps)
//   p = bf16(p + step * (m / s))                  _foreach_addcdiv_ (step < 0)
// with the fused multiply-adds the compiled list kernels use.
struct AdamConst {
    float w1, b2, c2, eps, wd_scale;
    int decay;
};

__device__ __forceinline__ void adamw8(uint4& p, const uint4& gr, uint4& m, uint4& v, float coef,
                                       const AdamConst& k, float step, float bc2s) {
    const uint32_t pw[4] = {p.x, p.y, p.z, p.w}, gw[4] = {gr.x, gr.y, gr.z, gr.w};
    const uint32_t mw[4] = {m.x, m.y, m.z, m.w}, vw[4] = {v.x, v.y, v.z, v.w};
    uint32_t po[4], mo[4], vo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float pf[2] = {bf16lo(pw[j]), bf16hi(pw[j])}, gf[2] = {bf16lo(gw[j]), bf16hi(gw[j])};
        float mf[2] = {bf16lo(mw[j]), bf16hi(mw[j])}, vf[2] = {bf16lo(vw[j]), bf16hi(vw[j])};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float g = bf_round(__fmul_rn(gf[h], coef));  // clip: _foreach_mul_(grads, coef)
            if (k.decay) pf[h] = bf_round(__fmul_rn(pf[h], k.wd_scale));
            mf[h] = bf_round(__fmaf_rn(k.w1, __fsub_rn(g, mf[h]), mf[h]));
            vf[h] = bf_round(__fmul_rn(vf[h], k.b2));
            vf[h] = bf_round(__fmaf_rn(k.c2, __fmul_rn(g, g), vf[h]));
            float sq = bf_round(__fsqrt_rn(vf[h]));
            sq = bf_round(__fdiv_rn(sq, bc2s));
            sq = bf_round(__fadd_rn(sq, k.eps));
            pf[h] = bf_round(__fmaf_rn(step, __fdiv_rn(mf[h], sq), pf[h]));
        }
        po[j] = pack2(pf[0], pf[1]);
        mo[j] = pack2(mf[0], mf[1]);
        vo[j] = pack2(vf[0], vf[1]);
    }
    p = make_uint4(po[0], po[1], po[2], po[3]);
    m = make_uint4(mo[0], mo[1], mo[2], mo[3]);
    v = make_uint4(vo[0], vo[1], vo[2], vo[3]);
}

__global__ void __launch_bounds__(kOptThreads) adamw_kernel(const __grid_constant__ OptGroup g,
                                                            const OptScalars* __restrict__ sc, AdamConst k) {
    const float coef = sc->coef, step_size = sc->step_size, bc2s = sc->bc2s;
    const int tid = threadIdx.x;
    constexpr int kU = 2;  // 8-element groups per thread in flight (4 loads each)
    for (int64_t c = g.chunk0[0] + blockIdx.x; c < g.chunk0[g.count]; c += gridDim.x) {
        const int ti = tensor_of(g, c);
        const cdlb200_adamw_tensor& t = g.t[ti];
        const int64_t base = (c - g.chunk0[ti]) * kOptChunk;
        const int64_t left = t.numel - base;
        const int nv = (int)((left < kOptChunk ? left : kOptChunk) / 8);
        uint4* pp = static_cast<uint4*>(t.param) + base / 8;
        const uint4* gp = static_cast<const uint4*>(t.grad) + base / 8;
        uint4* mp = static_cast<uint4*>(t.exp_avg) + base / 8;
        uint4* vp = static_cast<uint4*>(t.exp_avg_sq) + base / 8;
        uint32_t amax = 0;  // max |new param| over this thread's values, as bf16 magnitude bits
        for (int i0 = 0; i0 < nv; i0 += kU * kOptThreads) {
            uint4 p[kU], gr[kU], m[kU], v[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int i = i0 + u * kOptThreads + tid;
                if (i < nv) {
                    p[u] = pp[i];
                    gr[u] = ldg_stream(gp + i);
                    m[u] = mp[i];
                    v[u] = vp[i];
                }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int i = i0 + u * kOptThreads + tid;
                if (i < nv) {
                    adamw8(p[u], gr[u], m[u], v[u], coef, k, step_size, bc2s);
                    pp[i] = p[u];
                    mp[i] = m[u];
                    vp[i] = v[u];
                    if (t.amax) {
                        uint32_t a, b;
                        asm("max.u16x2 %0, %1, %2;" : "=r"(a) : "r"(p[u].x & 0x7fff7fffu), "r"(p[u].y & 0x7fff7fffu));
                        asm("max.u16x2 %0, %1, %2;" : "=r"(b) : "r"(p[u].z & 0x7fff7fffu), "r"(p[u].w & 0x7fff7fffu));
                        asm("max.u16x2 %0, %1, %2;" : "=r"(a) : "r"(a), "r"(b));
                        amax = max(amax, max(a & 0xffffu, a >> 16));
                    }
                }
            }
        }
        if (t.amax) {  // uniform per CTA: one reduction per warp
            amax = __reduce_max_sync(0xffffffffu, amax);
            if ((tid & 31) == 0) atomicMax(t.amax, amax);
        }
    }
}

int64_t chunks_of(int64_t numel) { return (numel + kOptChunk - 1) / kOptChunk; }

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace cdlb200

using namespace cdlb200;

extern "C" int64_t cdlb200_clip_adamw_workspace_bytes(const cdlb200_adamw_tensor* tensors, int count) {
    if (count < 0 || (count > 0 && !tensors)) return 0;
    int64_t chunks = 0;
    for (int i = 0; i < count; ++i)
        if (tensors[i].numel > 0) chunks += chunks_of(tensors[i].numel);
    return kScalarBytes + chunks * (int64_t)sizeof(float);
}

extern "C" int cdlb200_clip_adamw(const cdlb200_adamw_tensor* tensors, int count, double max_norm, double lr,
                                  double beta1, double beta2, double eps, double weight_decay, void* workspace,
                                  int64_t workspace_bytes, float* grad_norm, void* stream) {
    if (count < 0 || (count > 0 && !tensors) || !workspace) return CDLB200_ERR_INVALID_ARG;
    if (!(beta1 >= 0.0 && beta1 < 1.0) || !(beta2 >= 0.0 && beta2 < 1.0) || !(eps >= 0.0))
        return CDLB200_ERR_INVALID_ARG;
    for (int i = 0; i < count; ++i) {
        const cdlb200_adamw_tensor& t = tensors[i];
        if (t.numel < 0 || (t.numel % 8) != 0) return CDLB200_ERR_INVALID_ARG;
        if (t.numel == 0) continue;
        if (!t.param || !t.grad || !t.exp_avg || !t.exp_avg_sq) return CDLB200_ERR_INVALID_ARG;
        if (!al16(t.param) || !al16(t.grad) || !al16(t.exp_avg) || !al16(t.exp_avg_sq)) return CDLB200_ERR_ALIGNMENT;
    }
    if (workspace_bytes < cdlb200_clip_adamw_workspace_bytes(tensors, count)) return CDLB200_ERR_WORKSPACE;
    if (!al16(workspace)) return CDLB200_ERR_ALIGNMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    OptScalars* sc = static_cast<OptScalars*>(workspace);
    float* partial = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kScalarBytes);
    const int cap = num_sms() * 8;

    // groups of up to kOptGroup non-empty tensors, chunk indices global
    std::vector<OptGroup> groups;
    int64_t chunk = 0;
    for (int i = 0; i < count; ++i) {
        if (tensors[i].numel == 0) continue;
        if (groups.empty() || groups.back().count == kOptGroup) {
            groups.emplace_back();
            groups.back().count = 0;
            groups.back().pad = 0;
        }
        OptGroup& g = groups.back();
        g.t[g.count] = tensors[i];
        g.chunk0[g.count] = chunk;
        chunk += chunks_of(tensors[i].numel);
        g.chunk0[++g.count] = chunk;
    }
    const int ng = (int)groups.size();
    if (ng == 0) return CDLB200_OK;
    for (int k = 0; k < ng; ++k) {
        const int64_t n = groups[k].chunk0[groups[k].count] - groups[k].chunk0[0];
        sumsq_kernel<<<(int)(n < cap ? n : cap), kOptThreads, 0, st>>>(groups[k], partial);
        CDLB200_CHECK_LAUNCH();
        finalize_kernel<<<1, 1024, 0, st>>>(groups[k], partial, sc, k == 0, k == ng - 1, (float)max_norm, lr, beta1,
                                            beta2, grad_norm);
        CDLB200_CHECK_LAUNCH();
    }
    AdamConst kc;
    kc.w1 = (float)(1.0 - beta1);
    kc.b2 = (float)beta2;
    kc.c2 = (float)(1.0 - beta2);
    kc.eps = (float)eps;
    kc.wd_scale = (float)(1.0 - lr * weight_decay);
    kc.decay = weight_decay != 0.0;
    for (int k = 0; k < ng; ++k) {
        const int64_t n = groups[k].chunk0[groups[k].count] - groups[k].chunk0[0];
        adamw_kernel<<<(int)(n < cap ? n : cap), kOptThreads, 0, st>>>(groups[k], sc, kc);
        CDLB200_CHECK_LAUNCH();
    }
    return CDLB200_OK;
}
