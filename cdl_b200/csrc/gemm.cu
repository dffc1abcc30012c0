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
// TMEM and exits.  No multicast is used anywhere.
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
constexpr uint32_t kSpinLimit = 1u << 20;

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
            "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(a), "r"(parity)
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

struct GemmArgs {
    const uint8_t* sfa;  // swizzled scale atoms of A
    const uint8_t* sfb;  // swizzled scale atoms of B
    const float* alpha;  // device scalar, may be null (1.0)
    uint16_t* out;       // bf16 [M, ldo]
    int m, n, kbytes;    // kbytes = K in bytes per row (K/2 FP4, K FP8)
    int ldo;
    int c4a, c4b;        // scale atoms per 128-row block (ceil(nb/4))
    uint32_t* status;    // optional: non-zero after a timed-out wait
};

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
        const bool ok = mbar_wait(&acc_bar, 0);
        if (!ok) atomicExch(&abort_s, 1);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const float alpha = args.alpha ? *args.alpha : 1.0f;
        const int row = m0 + 32 * q + lane;
        if (ok && !*(volatile int*)&abort_s) {
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

template <int KIND>
int launch_gemm(const void* a, const void* b, const void* sfa, const void* sfb, const float* alpha, int64_t m,
                int64_t n, int64_t k, void* out, int64_t ldo, void* status, cudaStream_t st) {
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
    args.out = static_cast<uint16_t*>(out);
    args.m = (int)m;
    args.n = (int)n;
    args.kbytes = (int)kbytes;
    args.ldo = (int)ldo;
    const int64_t nb = (k + T::kVec - 1) / T::kVec;
    args.c4a = args.c4b = (int)((nb + 3) / 4);
    args.status = static_cast<uint32_t*>(status);
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
    return use_nvfp4 ? launch_gemm<kNv>(a, b, a_scale, b_scale, alpha, m, n, k, out, ldo, status, st)
                     : launch_gemm<kMx4>(a, b, a_scale, b_scale, alpha, m, n, k, out, ldo, status, st);
}

extern "C" int cdlb200_mm_mxfp8(const void* a, const void* b, const void* a_scale, const void* b_scale,
                                const float* alpha, int64_t m, int64_t n, int64_t k, void* out, int64_t ldo,
                                void* status, void* stream) {
    int rc = gemm_checks(a, b, a_scale, b_scale, m, n, k, 16, out, ldo);
    if (rc != CDLB200_OK || m == 0 || n == 0) return rc;
    return launch_gemm<kMx8>(a, b, a_scale, b_scale, alpha, m, n, k, out, ldo, status,
                             static_cast<cudaStream_t>(stream));
}
