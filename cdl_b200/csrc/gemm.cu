// gemm.cu -- block-scaled FP4 / FP8 GEMMs on the 5th-generation tensor cores.
//
// Replaces cdl's `cdl::mm_fp4` / `cdl::mm_mxfp8` custom ops
// (cdl/model/wrapper/flashinfer.py:5-62), which call FlashInfer's sm_120-only
// `b12x` kernels:
//     out[m, n] = alpha * sum_k deq(a)[m, k] * deq(b)[n, k]        (bf16 out)
// with a = packed codes [M, K/2] (FP4) or e4m3 [M, K] (FP8), b likewise
// [N, K] (cdl passes it as the [K, N] column-major view of the weight codes),
// and both scale matrices in the 128x4-tiled layout of
// cdl/core/mm/swizzle.py:5-14.
//
// One CTA computes a 128 x 128 output tile, accumulating in fp32 in tensor
// memory (TMEM).  Warp roles:
//   warp 0      TMA producer: per K tile, two 2-D tensor copies (A and B
//               tiles, 128 rows x 128 bytes, 128-byte swizzle) and two 1-D
//               bulk copies of the matching scale-factor atoms (512 bytes
//               each) into one of kStages shared-memory stages;
//   warp 1      allocates TMEM, then one thread copies each stage's scale
//               atoms into TMEM (tcgen05.cp 32x128b.warpx4) and issues the
//               block-scaled MMAs (tcgen05.mma ... block_scale), committing
//               each stage back to the producer;
//   warps 2-5   epilogue: tcgen05.ld the fp32 accumulator (each warp its 32
//               TMEM lanes), multiply by alpha, round to bf16, store.
// MMA kinds: NVFP4 = kind::mxf4nvf4 block16 with ue4m3 scales; MXFP4 =
// kind::mxf4 block32 with ue8m0; MXFP8 = kind::mxf8f6f4 (e4m3) with ue8m0.
// Every mbarrier wait is bounded; a timed-out wait sets a status word and
// the CTA stops issuing work, waits (bounded) for the MMAs it issued, frees
// TMEM and exits.  No TMA load uses multicast (the pair kernel's only
// multicast is the tcgen05.commit that signals both CTAs).
#include <cuda.h>

#include "common.cuh"

namespace cdlb200 {
namespace {

constexpr int kBM = 128, kBN = 128;
constexpr int kBKBytes = 128;  // K bytes per tile: 256 FP4 or 128 FP8 elements
constexpr int kStages = 5;
constexpr int kTileBytes = kBM * kBKBytes;      // 16 KiB (A and B alike)
constexpr int kSfAtomBytes = 512;               // 128 rows x 4 scale bytes
constexpr int kSfStageBytes = 4 * kSfAtomBytes;  // up to 4 atoms per K tile
constexpr int kStageBytes = 2 * kTileBytes + 2 * kSfStageBytes;
constexpr int kThreads = 192;
constexpr int kSfBufs = 4;  // scale-factor TMEM buffers, rotated per K tile
constexpr uint32_t kTmemCols = 256;  // 128 accumulator + 4 x 16 SFA + 4 x 16 SFB
// A bounded wait polls mbarrier.try_wait, each poll suspending the thread
// for at most kWaitHintNs unless the phase completes first (measured at
// 8192^3: 261 us against 277 us without the hint): at most about
// kSpinLimit * kWaitHintNs (~2.6 s) before a wait gives up.
constexpr uint32_t kSpinLimit = 1u << 18;
constexpr uint32_t kWaitHintNs = 10000;

enum Kind : int { kNv = 0, kMx4 = 1, kMx8 = 2 };

template <int KIND>
struct KindTraits;
template <>
struct KindTraits<kNv> {  // 16-element blocks, ue4m3
    static constexpr int kKmma = 64, kVec = 16, kFmt = 1, kSfFmt = 0;
};
template <>
struct KindTraits<kMx4> {  // 32-element blocks, ue8m0
    static constexpr int kKmma = 64, kVec = 32, kFmt = 1, kSfFmt = 1;
};
template <>
struct KindTraits<kMx8> {  // e4m3 elements, 32-element blocks, ue8m0
    static constexpr int kKmma = 32, kVec = 32, kFmt = 0, kSfFmt = 1;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Bounded wait for the phase of `bar` with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(a), "r"(parity), "n"(kWaitHintNs)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// UMMA shared-memory descriptor: K-major tile, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm100).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3fffu);
    d |= (uint64_t)1u << 16;                     // LBO (unused for swizzled K-major)
    d |= (uint64_t)((1024u >> 4) & 0x3fffu) << 32;  // SBO
    d |= (uint64_t)1u << 46;                     // version
    d |= (uint64_t)2u << 61;                     // SWIZZLE_128B
    return d;
}

// Descriptor of one 512-byte scale-factor atom (32 rows x 16 bytes, no
// swizzle; 8-row core matrices 128 bytes apart) for tcgen05.cp.
__device__ __forceinline__ uint64_t desc_sf_atom(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3fffu);
    d |= (uint64_t)1u << 16;                     // LBO
    d |= (uint64_t)((128u >> 4) & 0x3fffu) << 32;  // SBO
    d |= (uint64_t)1u << 46;                     // version
    return d;
}

template <int KIND>
__device__ __forceinline__ uint32_t instr_desc(uint32_t a_sf_id, uint32_t b_sf_id) {
    using T = KindTraits<KIND>;
    uint32_t d = 0;
    d |= (b_sf_id & 3u) << 4;
    d |= (uint32_t)T::kFmt << 7;   // a format
    d |= (uint32_t)T::kFmt << 10;  // b format
    // bits 15/16: K-major A and B (0)
    d |= (uint32_t)(kBN >> 3) << 17;
    d |= (uint32_t)T::kSfFmt << 23;
    d |= (uint32_t)(kBM >> 4) << 24;
    d |= (a_sf_id & 3u) << 29;
    return d;
}

template <int KIND>
__device__ __forceinline__ void mma_issue(uint32_t tmem_c, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
    if constexpr (KIND == kNv) {
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
                tmem_c),
            "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
    } else if constexpr (KIND == kMx4) {
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
                tmem_c),
            "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
    } else {
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
                tmem_c),
            "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
    }
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

struct GemmArgs;
__device__ __forceinline__ float epilogue_alpha(const GemmArgs& args);

struct GemmArgs {
    const uint8_t* sfa;  // swizzled scale atoms of A
    const uint8_t* sfb;  // swizzled scale atoms of B
    const float* alpha;    // device scalar, may be null (1.0)
    const float* alpha_b;  // second device scalar multiplied in (fp32, RN), may be null
    uint16_t* out;       // bf16 [M, ldo]
    int m, n, kbytes;    // kbytes = K in bytes per row (K/2 FP4, K FP8)
    int ldo;
    int c4a, c4b;        // scale atoms per 128-row block (ceil(nb/4))
    uint32_t* status;    // optional: non-zero after a timed-out wait
    const uint16_t* addend;  // optional bf16 [M, ld_add] added to the product (pair kernel: == out)
    int64_t ld_add;
};

// Two bf16 pairs added as torch adds two bf16 tensors: the fp32 sum of the
// widened values (one rounding), rounded to bf16.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
    const float lo = __fadd_rn(__uint_as_float(a << 16), __uint_as_float(b << 16));
    const float hi = __fadd_rn(__uint_as_float(a & 0xffff0000u), __uint_as_float(b & 0xffff0000u));
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// pk[j] (bf16 pairs of 8 * NV consecutive columns) += the addend's values at
// src (16-byte aligned), the loads issued together
template <int NV>
__device__ __forceinline__ void add_addend(uint32_t* pk, const uint16_t* src) {
    uint4 t[NV];
#pragma unroll
    for (int c = 0; c < NV; ++c) t[c] = reinterpret_cast<const uint4*>(src)[c];
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        pk[4 * c] = add_bf16x2(pk[4 * c], t[c].x);
        pk[4 * c + 1] = add_bf16x2(pk[4 * c + 1], t[c].y);
        pk[4 * c + 2] = add_bf16x2(pk[4 * c + 2], t[c].z);
        pk[4 * c + 3] = add_bf16x2(pk[4 * c + 3], t[c].w);
    }
}

// alpha * alpha_b as one fp32 product (what a torch multiply of the two
// scalars would give)
__device__ __forceinline__ float epilogue_alpha(const GemmArgs& args) {
    const float a = args.alpha ? *args.alpha : 1.0f;
    return args.alpha_b ? __fmul_rn(a, *args.alpha_b) : a;
}

template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    bs_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const GemmArgs args) {
    using T = KindTraits<KIND>;
    constexpr int kMmaPerTile = (kBKBytes * (KIND == kMx8 ? 1 : 2)) / T::kKmma;  // 4
    constexpr int kSfPerMma = T::kKmma / T::kVec;                               // scale bytes per row per MMA
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full_bar[kStages], empty_bar[kStages], acc_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
    const int nk = (args.kbytes + kBKBytes - 1) / kBKBytes;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&acc_bar, 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {  // whole warp allocates TMEM
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;
    // scale factors live in kSfBufs rotating 16-column buffers, so the copy for
    // a K tile never overwrites columns that the previous tile's MMAs read
    const uint32_t tmem_acc = tmem, tmem_sfa0 = tmem + 128, tmem_sfb0 = tmem + 128 + 16 * kSfBufs;

    // K tile kt holds kbytes_in_tile bytes of each row; the last may be partial
    auto tile_mmas = [&](int kt) {
        const int kb = args.kbytes - kt * kBKBytes < kBKBytes ? args.kbytes - kt * kBKBytes : kBKBytes;
        const int kel = kb * (KIND == kMx8 ? 1 : 2);
        return (kel + T::kKmma - 1) / T::kKmma;
    };
    auto tile_atoms = [&](int nmma) { return (nmma * kSfPerMma + 3) / 4; };

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            const int atoms_per_tile = (kMmaPerTile * kSfPerMma) / 4;
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % kStages;
                const uint32_t ph = (uint32_t)(kt / kStages) & 1u;
                if (!mbar_wait(&empty_bar[s], ph ^ 1u)) {
                    atomicExch(&abort_s, 1);
                    break;
                }
                if (*(volatile int*)&abort_s) break;
                const int natoms = tile_atoms(tile_mmas(kt));
                uint8_t* st = smem + (size_t)s * kStageBytes;
                mbar_expect_tx(&full_bar[s], 2u * kTileBytes + 2u * natoms * kSfAtomBytes);
                tma_load_2d(st, &map_a, kt * kBKBytes, m0, &full_bar[s]);
                tma_load_2d(st + kTileBytes, &map_b, kt * kBKBytes, n0, &full_bar[s]);
                const uint8_t* sa = args.sfa + ((size_t)(m0 / 128) * args.c4a + (size_t)kt * atoms_per_tile) * kSfAtomBytes;
                const uint8_t* sb = args.sfb + ((size_t)(n0 / 128) * args.c4b + (size_t)kt * atoms_per_tile) * kSfAtomBytes;
                bulk_load(st + 2 * kTileBytes, sa, natoms * kSfAtomBytes, &full_bar[s]);
                bulk_load(st + 2 * kTileBytes + kSfStageBytes, sb, natoms * kSfAtomBytes, &full_bar[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            int issued = 0;
            for (int kt = 0; kt < nk; ++kt) {
                const int s = kt % kStages;
                const uint32_t ph = (uint32_t)(kt / kStages) & 1u;
                if (!mbar_wait(&full_bar[s], ph)) {
                    atomicExch(&abort_s, 1);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const int nmma = tile_mmas(kt), natoms = tile_atoms(nmma);
                const uint32_t st = smem_addr(smem + (size_t)s * kStageBytes);
                const uint32_t tmem_sfa = tmem_sfa0 + 16u * (uint32_t)(kt % kSfBufs);
                const uint32_t tmem_sfb = tmem_sfb0 + 16u * (uint32_t)(kt % kSfBufs);
                for (int a = 0; a < natoms; ++a) {
                    const uint64_t dsa = desc_sf_atom(st + 2 * kTileBytes + a * kSfAtomBytes);
                    const uint64_t dsb = desc_sf_atom(st + 2 * kTileBytes + kSfStageBytes + a * kSfAtomBytes);
                    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_sfa + 4 * a), "l"(dsa)
                                 : "memory");
                    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(tmem_sfb + 4 * a), "l"(dsb)
                                 : "memory");
                }
                for (int kk = 0; kk < nmma; ++kk) {
                    const uint64_t da = desc_sw128(st + kk * 32);
                    const uint64_t db = desc_sw128(st + kTileBytes + kk * 32);
                    const uint32_t sfi = (uint32_t)(kk * kSfPerMma);  // scale byte index in the tile
                    const uint32_t col = 4u * (sfi >> 2), byte = sfi & 3u;
                    const uint32_t tsfa = (tmem_sfa + col) | (byte << 30);
                    const uint32_t tsfb = (tmem_sfb + col) | (byte << 30);
                    mma_issue<KIND>(tmem_acc, da, db, instr_desc<KIND>(byte, byte), tsfa, tsfb,
                                    (kt > 0 || kk > 0) ? 1u : 0u);
                }
                mma_commit(&empty_bar[s]);
                ++issued;
            }
            mma_commit(&acc_bar);  // also tracks the MMAs issued before an abort
            (void)issued;
        }
    } else {  // ---- epilogue warps 2..5
        const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
        bool ok = mbar_wait(&acc_bar, 0);
        if (!ok) atomicExch(&abort_s, 1);
        ok = __all_sync(0xffffffffu, ok && !*(volatile int*)&abort_s);  // tcgen05.ld is warp-collective
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const float alpha = epilogue_alpha(args);
        const int row = m0 + 32 * q + lane;
        if (ok) {
#pragma unroll 1
            for (int c0 = 0; c0 < kBN; c0 += 32) {
                uint32_t v[32];
                const uint32_t taddr = tmem_acc + ((uint32_t)(32 * q) << 16) + (uint32_t)c0;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                    "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                      "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                      "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
                      "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
                      "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (row < args.m) {
                    uint32_t packed[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float lo = __fmul_rn(u2f(v[2 * i]), alpha), hi = __fmul_rn(u2f(v[2 * i + 1]), alpha);
                        uint32_t r;
                        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
                        packed[i] = r;
                    }
                    uint16_t* dst = args.out + (size_t)row * args.ldo + n0 + c0;
                    const int ncol = args.n - (n0 + c0);
                    if (args.addend != nullptr && ncol > 0) {
                        const uint16_t* src = args.addend + (size_t)row * args.ld_add + n0 + c0;
                        if (ncol >= 32 && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
                            add_addend<4>(packed, src);
                        } else {
                            for (int i = 0; i < 32 && i < ncol; ++i) {
                                const uint32_t sh = 16u * (uint32_t)(i & 1);
                                const uint32_t sum = add_bf16x2(packed[i >> 1] >> sh, (uint32_t)src[i]) & 0xffffu;
                                packed[i >> 1] = (packed[i >> 1] & ~(0xffffu << sh)) | (sum << sh);
                            }
                        }
                    }
                    if (ncol >= 32 && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
                        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            d4[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2], packed[4 * i + 3]);
                    } else {
                        for (int i = 0; i < 32 && i < ncol; ++i)
                            dst[i] = (uint16_t)((packed[i >> 1] >> (16 * (i & 1))) & 0xffffu);
                    }
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && abort_s && args.status) atomicExch(args.status, 1u);
    if (warp == 1) {
        // every MMA this CTA issued has completed before TMEM is released
        (void)mbar_wait(&acc_bar, 0);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Pair kernel: two CTAs of a cluster (one per SM) compute a 256 x 256 tile
// with cta_group::2 MMAs (M = 256, N = 256).  CTA rank r holds rows
// [m0 + 128 r, +128) of A and rows [n0 + 128 r, +128) of B in its shared
// memory; the tensor cores of the pair read both halves of B, so every SM
// loads 32 KiB per K tile instead of the 48 KiB a single-SM 128 x 256 tile
// needs -- the TMA engine of one SM is what bounds this GEMM.
//
// Scale factors do not go through the tensor-memory copy engine (whose
// per-instruction cost would exceed the MMA time at N = 256): the four
// epilogue warps write them into TMEM with tcgen05.st while the MMAs of the
// previous stages run.  Layout the block-scaled MMA reads (M = 128 per SM):
//   A row r       -> TMEM lane r,              column tsfa + r/32
//   B column n    -> lane 32 (r/32) + n % 32,  column tsfb + n/32
// i.e. each lane quarter needs every column's B scales; one 4-byte cell holds
// the scales of four consecutive K blocks (the sf_id selects the byte for the
// MX kinds).  Warp q (lanes 32q..32q+31) therefore stores, per cell, its own
// A scales in all four columns of the cell and both 128-column B atoms' rows.
//
// Barriers: full[s] lives in the leader (rank 0) and collects the A/B TMA
// bytes of both CTAs; sfdata[s] is local (this CTA's scale bytes landed);
// sffull[s] (leader) collects one arrival per CTA once its scales are in
// TMEM; empty[s] and acc_full are signalled in both CTAs by a multicast
// tcgen05.commit of the leader.  No TMA load uses multicast.
// ---------------------------------------------------------------------------
constexpr int k2Stages = 5;
constexpr int k2TileBytes = 128 * kBKBytes;                     // 16 KiB
constexpr int k2SfaBytes = 4 * kSfAtomBytes;                    // 2 KiB
constexpr int k2SfbBytes = 8 * kSfAtomBytes;                    // 4 KiB: two 128-column blocks
constexpr int k2StageBytes = 2 * k2TileBytes + k2SfaBytes + k2SfbBytes;  // 38 KiB
constexpr int k2OutBytes = 128 * 128 * 2;  // bf16 staging of half of one CTA's 128 x 256 output tile
// TMEM columns: accumulator [0, 256); per stage s the B scales at 256 + 32 s
// (32 columns) and the A scales at 416 + 16 s (16 columns), so every
// tcgen05.st / MMA scale address is aligned to its width.
constexpr uint32_t k2TmemCols = 512;
constexpr uint32_t k2SfbCol0 = 256, k2SfaCol0 = 256 + 32 * k2Stages;

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared variable in CTA `rank`
__device__ __forceinline__ uint32_t map_rank(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}

__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_addr(bar)),
        "h"((uint16_t)3)
        : "memory");
}

template <int KIND>
__device__ __forceinline__ void mma_issue_pair(uint32_t tmem_c, uint64_t da, uint64_t db, uint32_t idesc, uint32_t tsfa,
                                               uint32_t tsfb, uint32_t accumulate) {
    if constexpr (KIND == kNv) {
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
                tmem_c),
            "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
    } else if constexpr (KIND == kMx4) {
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
                tmem_c),
            "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
    } else {
        asm volatile(
            "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
            "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(
                tmem_c),
            "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb));
    }
}

template <int KIND>
__device__ __forceinline__ uint32_t instr_desc_pair(uint32_t sf_id) {
    using T = KindTraits<KIND>;
    uint32_t d = 0;
    d |= (sf_id & 3u) << 4;
    d |= (uint32_t)T::kFmt << 7;
    d |= (uint32_t)T::kFmt << 10;
    d |= (uint32_t)(256 >> 3) << 17;  // N = 256
    d |= (uint32_t)T::kSfFmt << 23;
    d |= (uint32_t)(256 >> 4) << 24;  // M = 256 (128 per CTA)
    d |= (sf_id & 3u) << 29;
    return d;
}

// tcgen05.st.32x32b of N consecutive columns (one 32-bit value per lane and column).
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t addr, const uint32_t* r);
template <>
__device__ __forceinline__ void tmem_st<4>(uint32_t addr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r[0]), "r"(r[1]), "r"(r[2]),
                 "r"(r[3])
                 : "memory");
}
template <>
__device__ __forceinline__ void tmem_st<8>(uint32_t addr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
template <>
__device__ __forceinline__ void tmem_st<16>(uint32_t addr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            addr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
template <>
__device__ __forceinline__ void tmem_st<32>(uint32_t addr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(addr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Scales of one K tile (CELLS 4-byte cells) for this warp's 32 lanes: A cell g
// in columns ta + 4g .. +3 (the MMA reads column ta + 4g + quarter), B cell g
// of the two 128-column blocks in columns tb + 8g .. +7.
template <int CELLS>
__device__ __forceinline__ void store_scales(uint32_t ta, uint32_t tb, const uint32_t (&a)[4], const uint4 (&b)[8]) {
    uint32_t ra[4 * CELLS], rb[8 * CELLS];
#pragma unroll
    for (int g = 0; g < CELLS; ++g) {
        ra[4 * g] = ra[4 * g + 1] = ra[4 * g + 2] = ra[4 * g + 3] = a[g];
        rb[8 * g + 0] = b[2 * g].x;
        rb[8 * g + 1] = b[2 * g].y;
        rb[8 * g + 2] = b[2 * g].z;
        rb[8 * g + 3] = b[2 * g].w;
        rb[8 * g + 4] = b[2 * g + 1].x;
        rb[8 * g + 5] = b[2 * g + 1].y;
        rb[8 * g + 6] = b[2 * g + 1].z;
        rb[8 * g + 7] = b[2 * g + 1].w;
    }
    tmem_st<4 * CELLS>(ta, ra);
    tmem_st<8 * CELLS>(tb, rb);
}

// OR of `v` over the 128 threads of named barrier ID (one four-warp group).
template <int ID>
__device__ __forceinline__ bool group_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, %2, 128, p;\nselp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(ID)
        : "memory");
    return r != 0;
}

template <int ID>
__device__ __forceinline__ void group_sync() {
    asm volatile("bar.sync %0, 128;" ::"n"(ID) : "memory");
}

// OR of `v` over the 256 threads of the two epilogue groups (named barrier 6).
__device__ __forceinline__ bool epilogue_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n.reg .pred p, q;\nsetp.ne.u32 p, %1, 0;\nbar.red.or.pred q, 6, 256, p;\nselp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

// the four warps of epilogue group `hf` (named barriers 2 and 3)
__device__ __forceinline__ void epilogue_group_sync(int hf) {
    if (hf == 0) group_sync<2>();
    else group_sync<3>();
}

__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void arrive_remote(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// 2-D TMA store of a 64-column x 128-row bf16 box (128-byte swizzled in shared
// memory); the tensor map clips rows and columns outside the output.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
                 "r"(y), "r"(smem_addr(src))
                 : "memory");
}

// The same box added to the bf16 values already in global memory (the TMA
// unit's reduce-add: out = bf16(out + staged)), for the accumulating GEMM.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, int x, int y, const void* src) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map),
                 "r"(x), "r"(y), "r"(smem_addr(src))
                 : "memory");
}

// 64 fp32 accumulator columns of this warp's 32 TMEM lanes (one row per lane).
// The load completes asynchronously: the registers are valid after
// tmem_wait_ld.
__device__ __forceinline__ void tmem_ld64(uint32_t (&v)[64], uint32_t taddr) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,"
        "%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]), "=r"(v[32]),
          "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]),
          "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]),
          "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]), "=r"(v[56]),
          "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63])
        : "r"(taddr));
}

// Waits for this thread's outstanding tcgen05.ld and ties the buffer's
// registers to the wait, so that no use of them is scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&v)[64]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 64; ++j) asm volatile("" : "+r"(v[j]));
}

// 64 accumulator columns x alpha (packed fp32 multiplies, each lane an IEEE
// round-to-nearest product) -> 32 bf16 pairs, columns (2j, 2j + 1) in pk[j].
__device__ __forceinline__ void pack64(const uint32_t (&v)[64], float alpha, uint32_t (&pk)[32]) {
    uint64_t aa;
    asm("mov.b64 %0, {%1, %1};" : "=l"(aa) : "f"(alpha));
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        uint64_t pv, pr;
        asm("mov.b64 %0, {%1, %2};" : "=l"(pv) : "r"(v[2 * j]), "r"(v[2 * j + 1]));
        asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(pr) : "l"(pv), "l"(aa));
        asm("{\n.reg .f32 lo, hi;\nmov.b64 {lo, hi}, %1;\ncvt.rn.bf16x2.f32 %0, hi, lo;\n}" : "=r"(pk[j]) : "l"(pr));
    }
}

// 32 packed bf16 pairs of row r into the 128-byte-swizzled staging block `blk`.
__device__ __forceinline__ void stage_packed64(const uint32_t (&pk)[32], uint8_t* out_s, int r, int blk) {
    uint8_t* row = out_s + blk * (128 * 128) + r * 128;
#pragma unroll
    for (int chunk = 0; chunk < 8; ++chunk)
        *reinterpret_cast<uint4*>(row + ((chunk ^ (r & 7)) * 16)) =
            make_uint4(pk[4 * chunk], pk[4 * chunk + 1], pk[4 * chunk + 2], pk[4 * chunk + 3]);
}

// warp 0 TMA, 1 MMA (2, 3 idle), 4-7 scale factors, 8-15 epilogue (two groups of
// four warps, one per 128-column half of the tile)
constexpr int k2Threads = 512;

// Persistent: cluster c (of gridDim.x / 2) computes pair tiles c, c + C, c + 2C, ...
// (row-major over 256 x 256 tiles).  The shared-memory stage ring and the
// scale-factor TMEM buffers run on across tiles.  Eight epilogue warps drain
// the accumulator: each group of four loads its 128-column half into
// registers, so the accumulator is released (acc_empty) as soon as both
// halves are loaded, and the two groups then take turns with the one
// staging buffer (stg_free) while the MMAs of the next tile already run.
//
// Registers: 512 threads x 128.  An epilogue warp holds its 128 columns as
// 64 packed bf16 pairs: the first 64 columns are scaled and packed before
// the second 64 are loaded.
template <int KIND>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(k2Threads, 1)
    bs_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_out, const GemmArgs args, int tiles_n,
                        int tiles_total) {
    using T = KindTraits<KIND>;
    constexpr int kMmaPerTile = (kBKBytes * (KIND == kMx8 ? 1 : 2)) / T::kKmma;  // 4
    constexpr int kSfPerMma = T::kKmma / T::kVec;                               // scale bytes per row per MMA
    constexpr int kCells = kMmaPerTile * kSfPerMma / 4;                         // 4-byte cells per K tile
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full_bar[k2Stages], empty_bar[k2Stages], sfdata_bar[k2Stages], sffull_bar[k2Stages],
        acc_full, acc_empty, done_bar, stg_free[2];
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cluster = (int)(blockIdx.x >> 1), nclusters = (int)(gridDim.x >> 1);
    const int my_tiles = cluster < tiles_total ? (tiles_total - 1 - cluster) / nclusters + 1 : 0;
    const int nk = (args.kbytes + kBKBytes - 1) / kBKBytes;

    if (threadIdx.x == 0) {
        for (int s = 0; s < k2Stages; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
            mbar_init(&sfdata_bar[s], 1);
            mbar_init(&sffull_bar[s], 2);
        }
        mbar_init(&acc_full, 1);
        mbar_init(&acc_empty, 4);  // one arrival per epilogue group of each CTA
        mbar_init(&done_bar, 1);
        mbar_init(&stg_free[0], 1);
        mbar_init(&stg_free[1], 1);
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base_s)),
                     "r"(k2TmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_s;

    auto tile_origin = [&](int i, int& m0, int& n0) {
        const int t = cluster + i * nclusters;
        n0 = (t % tiles_n) * 256;
        m0 = (t / tiles_n) * 256;
    };
    auto tile_mmas = [&](int kt) {
        const int kb = args.kbytes - kt * kBKBytes < kBKBytes ? args.kbytes - kt * kBKBytes : kBKBytes;
        const int kel = kb * (KIND == kMx8 ? 1 : 2);
        return (kel + T::kKmma - 1) / T::kKmma;
    };
    auto tile_atoms = [&](int nmma) { return (nmma * kSfPerMma + 3) / 4; };
    auto aborted = [&]() { return *(volatile int*)&abort_s != 0; };

    if (warp < 4) {
        if (warp == 0) {
            if (lane == 0) {  // ---- TMA producer (both CTAs)
                const uint32_t full0 = map_rank(&full_bar[0], 0);
                int g = 0;
                for (int i = 0; i < my_tiles && !aborted(); ++i) {
                    int m0, n0;
                    tile_origin(i, m0, n0);
                    const int mblk = (m0 >> 7) + (int)rank, nblk = n0 >> 7;
                    const bool a_ok = mblk * 128 < args.m;
                    const bool b0_ok = nblk * 128 < args.n, b1_ok = (nblk + 1) * 128 < args.n;
                    for (int kt = 0; kt < nk; ++kt, ++g) {
                        const int s = g % k2Stages;
                        const uint32_t ph = (uint32_t)(g / k2Stages) & 1u;
                        if (!mbar_wait(&empty_bar[s], ph ^ 1u)) atomicExch(&abort_s, 1);
                        if (aborted()) break;
                        uint8_t* st = smem + (size_t)s * k2StageBytes;
                        // the scale atoms first: they land while the A / B
                        // tiles are still in flight, so the scale warps' TMEM
                        // stores overlap the operand copies
                        const int natoms = tile_atoms(tile_mmas(kt));
                        const uint32_t sfb = (uint32_t)(natoms * kSfAtomBytes);
                        mbar_expect_tx(&sfdata_bar[s], (a_ok ? sfb : 0u) + (b0_ok ? sfb : 0u) + (b1_ok ? sfb : 0u));
                        uint8_t* sf = st + 2 * k2TileBytes;
                        const size_t at = (size_t)kt * kCells;
                        if (a_ok)
                            bulk_load(sf, args.sfa + ((size_t)mblk * args.c4a + at) * kSfAtomBytes, sfb, &sfdata_bar[s]);
                        if (b0_ok)
                            bulk_load(sf + k2SfaBytes, args.sfb + ((size_t)nblk * args.c4b + at) * kSfAtomBytes, sfb,
                                      &sfdata_bar[s]);
                        if (b1_ok)
                            bulk_load(sf + k2SfaBytes + 4 * kSfAtomBytes,
                                      args.sfb + ((size_t)(nblk + 1) * args.c4b + at) * kSfAtomBytes, sfb, &sfdata_bar[s]);
                        if (rank == 0) mbar_expect_tx(&full_bar[s], 4u * k2TileBytes);
                        tma_load_2d_pair(st, &map_a, kt * kBKBytes, m0 + 128 * (int)rank, full0 + 8u * s);
                        tma_load_2d_pair(st + k2TileBytes, &map_b, kt * kBKBytes, n0 + 128 * (int)rank, full0 + 8u * s);
                    }
                }
            }
        } else if (warp == 1) {
            if (rank == 0 && lane == 0) {  // ---- MMA issuer (leader CTA only)
                int g = 0;
                for (int i = 0; i < my_tiles && !aborted(); ++i) {
                    // both CTAs' epilogues have drained the accumulator of tile i - 1
                    if (i > 0 && !mbar_wait(&acc_empty, (uint32_t)(i - 1) & 1u)) {
                        atomicExch(&abort_s, 1);
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    for (int kt = 0; kt < nk; ++kt, ++g) {
                        const int s = g % k2Stages;
                        const uint32_t ph = (uint32_t)(g / k2Stages) & 1u;
                        if (!mbar_wait(&full_bar[s], ph) || !mbar_wait(&sffull_bar[s], ph)) {
                            atomicExch(&abort_s, 1);
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const int nmma = tile_mmas(kt);
                        const uint32_t st = smem_addr(smem + (size_t)s * k2StageBytes);
                        const uint32_t tsfa0 = tmem + k2SfaCol0 + 16u * (uint32_t)s;
                        const uint32_t tsfb0 = tmem + k2SfbCol0 + 32u * (uint32_t)s;
                        for (int kk = 0; kk < nmma; ++kk) {
                            const uint64_t da = desc_sw128(st + kk * 32);
                            const uint64_t db = desc_sw128(st + k2TileBytes + kk * 32);
                            const uint32_t sfi = (uint32_t)(kk * kSfPerMma);
                            const uint32_t cell = sfi >> 2, byte = sfi & 3u;
                            mma_issue_pair<KIND>(tmem, da, db, instr_desc_pair<KIND>(byte),
                                                 (tsfa0 + 4u * cell) | (byte << 30), (tsfb0 + 8u * cell) | (byte << 30),
                                                 (kt > 0 || kk > 0) ? 1u : 0u);
                        }
                        mma_commit_pair(&empty_bar[s]);
                    }
                    if (aborted()) break;
                    mma_commit_pair(&acc_full);
                }
                mma_commit_pair(&done_bar);  // completes once every MMA issued above has
            }
        }
    } else if (warp < 8) {  // ---- warps 4..7: scale factors into TMEM
        const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
        const uint32_t lane_off = (uint32_t)(32 * q) << 16;
        const uint32_t sffull0 = map_rank(&sffull_bar[0], 0);
        const int total = my_tiles * nk;
        for (int g = 0; g < total; ++g) {
            const int s = g % k2Stages, kt = g % nk;
            const uint32_t ph = (uint32_t)(g / k2Stages) & 1u;
            bool ok = mbar_wait(&sfdata_bar[s], ph);
            // the MMAs that last read this stage's scale columns have completed
            if (ok && g >= k2Stages) ok = mbar_wait(&empty_bar[s], ph ^ 1u);
            if (!ok) atomicExch(&abort_s, 1);
            if (group_any<1>(!ok || aborted())) break;  // the four warps leave together
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            (void)kt;
            const uint8_t* sf = smem + (size_t)s * k2StageBytes + 2 * k2TileBytes;
            uint32_t a[4];
            uint4 b[8];
#pragma unroll
            for (int c = 0; c < kCells; ++c) {
                a[c] = *reinterpret_cast<const uint32_t*>(sf + c * kSfAtomBytes + 16 * lane + 4 * q);
                b[2 * c] = *reinterpret_cast<const uint4*>(sf + k2SfaBytes + c * kSfAtomBytes + 16 * lane);
                b[2 * c + 1] = *reinterpret_cast<const uint4*>(sf + k2SfaBytes + (4 + c) * kSfAtomBytes + 16 * lane);
            }
            store_scales<kCells>(tmem + lane_off + k2SfaCol0 + 16u * (uint32_t)s,
                                 tmem + lane_off + k2SfbCol0 + 32u * (uint32_t)s, a, b);
            // the stores are complete once wait::st returns; a relaxed arrive is
            // enough to publish them (a cluster-scope release would also wait
            // for this CTA's in-flight TMA loads, ~1 us per K tile)
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            group_sync<1>();
            if (threadIdx.x == 128) arrive_remote(sffull0 + 8u * s);
        }
    } else {  // ---- warps 8..15: epilogue, 128 rows x 256 columns of this CTA per tile
        const int q = warp & 3, hf = (warp >> 2) - 2;  // TMEM lane quarter, 128-column half of the tile
        const int r = 32 * q + lane;                   // row of the tile = TMEM lane
        const uint32_t lane_off = (uint32_t)(32 * q) << 16;
        const uint32_t acc_empty0 = map_rank(&acc_empty, 0);
        const bool leader = (threadIdx.x & 127) == 0;  // issues this group's stores
        const float alpha = epilogue_alpha(args);
        // staging: two 64-column blocks of 128 rows x 128 bytes (one group's
        // 128 columns), 16-byte chunk c of row r at chunk c ^ (r & 7) (the TMA
        // 128-byte swizzle); group 0 and group 1 use it in turn
        uint8_t* out_s = smem + (size_t)k2Stages * k2StageBytes;
        int i = 0;
        for (; i < my_tiles; ++i) {
            const bool ok = mbar_wait(&acc_full, (uint32_t)i & 1u);
            if (!ok) atomicExch(&abort_s, 1);
            if (epilogue_any(!ok || aborted())) break;  // all eight warps leave together
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t pa[32], pb[32];  // the half's 128 columns x alpha, as bf16 pairs
            {
                uint32_t v[64];
                tmem_ld64(v, tmem + lane_off + 128u * (uint32_t)hf);
                tmem_wait_ld(v);
                pack64(v, alpha, pa);
            }
            uint32_t vb[64];
            tmem_ld64(vb, tmem + lane_off + 128u * (uint32_t)hf + 64u);
            tmem_wait_ld(vb);
            // this group's half is in registers: once both groups of both CTAs
            // have arrived the next tile's MMAs may overwrite the accumulator
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            epilogue_group_sync(hf);
            if (leader) arrive_remote(acc_empty0);
            // the staging buffer is free: group 1 waits for group 0's stores of
            // this tile, group 0 for group 1's stores of the previous tile
            bool free_ok = true;
            if (hf == 1) free_ok = mbar_wait(&stg_free[1], (uint32_t)i & 1u);
            else if (i > 0) free_ok = mbar_wait(&stg_free[0], (uint32_t)(i - 1) & 1u);
            if (!free_ok) atomicExch(&abort_s, 1);
            pack64(vb, alpha, pb);
            if (free_ok) {
                stage_packed64(pa, out_s, r, 0);
                stage_packed64(pb, out_s, r, 1);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // staging visible to the TMA engine
            }
            epilogue_group_sync(hf);
            if (leader) {
                if (free_ok) {
                    int m0, n0;
                    tile_origin(i, m0, n0);
                    const int y = m0 + 128 * (int)rank;
                    if (y < args.m) {
                        for (int b = 0; b < 2; ++b) {
                            const int x = n0 + 128 * hf + 64 * b;
                            if (x >= args.n) continue;
                            // accumulating GEMM (addend == out): the TMA unit adds the
                            // bf16 tile to out in L2, no loads in the epilogue
                            if (args.addend != nullptr) tma_reduce_add_2d(&map_out, x, y, out_s + b * (128 * 128));
                            else tma_store_2d(&map_out, x, y, out_s + b * (128 * 128));
                        }
                    }
                }
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // staging read
                mbar_arrive_local(&stg_free[hf ^ 1]);
            }
        }
        if (leader) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // output written
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0 && abort_s && args.status) atomicExch(args.status, 1u);
    if (warp == 1) (void)mbar_wait(&done_bar, 0);  // every MMA of the pair has completed
    cluster_sync_all();  // neither CTA touches the other's barriers or TMEM any more
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(k2TmemCols) : "memory");
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D byte tensor [rows, row_bytes] with a 128 x 128-byte box, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)kBKBytes, 128u};
    cuuint32_t estr[2] = {1u, 1u};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 output [rows, cols] with row pitch ldo elements, 64-column x 128-row
// boxes, 128-byte swizzle (the layout the pair kernel stages its tile in).
bool make_out_map(CUtensorMap* map, void* base, int64_t rows, int64_t cols, int64_t ldo) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ldo * 2)};
    cuuint32_t box[2] = {64u, 128u};
    cuuint32_t estr[2] = {1u, 1u};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int KIND>
int launch_gemm(const void* a, const void* b, const void* sfa, const void* sfb, const float* alpha,
                const float* alpha_b, int64_t m, int64_t n, int64_t k, void* out, int64_t ldo, void* status,
                cudaStream_t st, bool accumulate = false) {
    using T = KindTraits<KIND>;
    const int64_t kbytes = KIND == kMx8 ? k : k / 2;
    CUtensorMap ma, mb;
    if (!make_map(&ma, a, m, kbytes) || !make_map(&mb, b, n, kbytes)) return CDLB200_ERR_CUDA;
    static bool attr_set[3] = {false, false, false};
    const int smem = kStages * kStageBytes + 1024;
    if (!attr_set[KIND]) {
        if (cudaFuncSetAttribute(bs_gemm_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
            return CDLB200_ERR_CUDA;
        attr_set[KIND] = true;
    }
    GemmArgs args;
    args.sfa = static_cast<const uint8_t*>(sfa);
    args.sfb = static_cast<const uint8_t*>(sfb);
    args.alpha = alpha;
    args.alpha_b = alpha_b;
    args.out = static_cast<uint16_t*>(out);
    args.m = (int)m;
    args.n = (int)n;
    args.kbytes = (int)kbytes;
    args.ldo = (int)ldo;
    const int64_t nb = (k + T::kVec - 1) / T::kVec;
    args.c4a = args.c4b = (int)((nb + 3) / 4);
    args.status = static_cast<uint32_t*>(status);
    // accumulate: out is read as the addend of the product (out += product)
    args.addend = accumulate ? static_cast<const uint16_t*>(out) : nullptr;
    args.ld_add = ldo;
    // pair kernel: 256 x 256 tiles on SM pairs (its TMA store needs a 16-byte
    // aligned output with a row pitch that is a multiple of 16 bytes; an
    // accumulating launch adds into out with the TMA reduce-add)
    CUtensorMap mo;
    if (n > kBN && ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) && (ldo % 8) == 0 &&
        make_out_map(&mo, out, m, n, ldo)) {
        static bool pair_attr_set[3] = {false, false, false};
        const int smem2 = k2Stages * k2StageBytes + k2OutBytes + 1024;
        if (!pair_attr_set[KIND]) {
            if (cudaFuncSetAttribute(bs_gemm_pair_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2) !=
                cudaSuccess)
                return CDLB200_ERR_CUDA;
            pair_attr_set[KIND] = true;
        }
        const int64_t tiles_n = (n + 255) / 256, tiles_m = (m + 255) / 256, tiles = tiles_n * tiles_m;
        if (tiles > (int64_t)INT32_MAX) return CDLB200_ERR_INVALID_ARG;
        const int64_t pairs = persistent_sms() / 2;  // SM pairs it may occupy
        const int64_t clusters = tiles < pairs ? tiles : pairs;
        bs_gemm_pair_kernel<KIND><<<(unsigned)(2 * clusters), k2Threads, smem2, st>>>(ma, mb, mo, args, (int)tiles_n,
                                                                                           (int)tiles);
        CDLB200_CHECK_LAUNCH();
        return CDLB200_OK;
    }
    dim3 grid((unsigned)((n + kBN - 1) / kBN), (unsigned)((m + kBM - 1) / kBM));
    bs_gemm_kernel<KIND><<<grid, kThreads, smem, st>>>(ma, mb, args);
    CDLB200_CHECK_LAUNCH();
    return CDLB200_OK;
}

bool al(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) & (uintptr_t)(a - 1)) == 0; }

int gemm_checks(const void* a, const void* b, const void* sfa, const void* sfb, int64_t m, int64_t n, int64_t k,
                int64_t kmul, const void* out, int64_t ldo) {
    if (m < 0 || n < 0 || k < 0) return CDLB200_ERR_INVALID_ARG;
    if (m == 0 || n == 0) return CDLB200_OK;
    if (!a || !b || !sfa || !sfb || !out || ldo < n || k == 0 || (k % kmul) != 0) return CDLB200_ERR_INVALID_ARG;
    if (m > (1ll << 31) - 1 || n > (1ll << 31) - 1 || k > (1ll << 31) - 1) return CDLB200_ERR_INVALID_ARG;
    if (!al(a, 16) || !al(b, 16) || !al(sfa, 16) || !al(sfb, 16) || !al(out, 2)) return CDLB200_ERR_ALIGNMENT;
    int dev = 0, major = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
        return CDLB200_ERR_CUDA;
    return major == 10 ? CDLB200_OK : CDLB200_ERR_UNSUPPORTED;
}

}  // namespace
}  // namespace cdlb200

using namespace cdlb200;

extern "C" int cdlb200_mm_fp4(const void* a, const void* b, const void* a_scale, const void* b_scale,
                              const float* alpha, int64_t m, int64_t n, int64_t k, int block_size, int use_nvfp4,
                              void* out, int64_t ldo, void* status, void* stream) {
    if ((use_nvfp4 && block_size != 16) || (!use_nvfp4 && block_size != 32)) return CDLB200_ERR_INVALID_ARG;
    int rc = gemm_checks(a, b, a_scale, b_scale, m, n, k, 32, out, ldo);
    if (rc != CDLB200_OK || m == 0 || n == 0) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return use_nvfp4 ? launch_gemm<kNv>(a, b, a_scale, b_scale, alpha, nullptr, m, n, k, out, ldo, status, st)
                     : launch_gemm<kMx4>(a, b, a_scale, b_scale, alpha, nullptr, m, n, k, out, ldo, status, st);
}

extern "C" int cdlb200_mm_fp4_alpha2(const void* a, const void* b, const void* a_scale, const void* b_scale,
                                     const float* alpha_a, const float* alpha_b, int64_t m, int64_t n, int64_t k,
                                     int block_size, int use_nvfp4, void* out, int64_t ldo, void* status,
                                     void* stream) {
    if ((use_nvfp4 && block_size != 16) || (!use_nvfp4 && block_size != 32)) return CDLB200_ERR_INVALID_ARG;
    int rc = gemm_checks(a, b, a_scale, b_scale, m, n, k, 32, out, ldo);
    if (rc != CDLB200_OK || m == 0 || n == 0) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return use_nvfp4 ? launch_gemm<kNv>(a, b, a_scale, b_scale, alpha_a, alpha_b, m, n, k, out, ldo, status, st)
                     : launch_gemm<kMx4>(a, b, a_scale, b_scale, alpha_a, alpha_b, m, n, k, out, ldo, status, st);
}

extern "C" int cdlb200_mm_fp4_alpha2_acc(const void* a, const void* b, const void* a_scale, const void* b_scale,
                                         const float* alpha_a, const float* alpha_b, int64_t m, int64_t n,
                                         int64_t k, int block_size, int use_nvfp4, void* out, int64_t ldo,
                                         void* status, void* stream) {
    if ((use_nvfp4 && block_size != 16) || (!use_nvfp4 && block_size != 32)) return CDLB200_ERR_INVALID_ARG;
    int rc = gemm_checks(a, b, a_scale, b_scale, m, n, k, 32, out, ldo);
    if (rc != CDLB200_OK || m == 0 || n == 0) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return use_nvfp4 ? launch_gemm<kNv>(a, b, a_scale, b_scale, alpha_a, alpha_b, m, n, k, out, ldo, status, st, true)
                     : launch_gemm<kMx4>(a, b, a_scale, b_scale, alpha_a, alpha_b, m, n, k, out, ldo, status, st,
                                         true);
}

extern "C" int cdlb200_mm_mxfp8(const void* a, const void* b, const void* a_scale, const void* b_scale,
                                const float* alpha, int64_t m, int64_t n, int64_t k, void* out, int64_t ldo,
                                void* status, void* stream) {
    int rc = gemm_checks(a, b, a_scale, b_scale, m, n, k, 16, out, ldo);
    if (rc != CDLB200_OK || m == 0 || n == 0) return rc;
    return launch_gemm<kMx8>(a, b, a_scale, b_scale, alpha, nullptr, m, n, k, out, ldo, status,
                             static_cast<cudaStream_t>(stream));
}
