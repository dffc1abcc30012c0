/*
 * cdlb200.h -- C ABI of the B200-native (sm_100a) cdl low-precision hot path.
 *
 * Every entry point takes device pointers owned by the caller, sizes in
 * elements, and a CUDA stream (as `void*`, a cudaStream_t; NULL = legacy
 * default stream).  Calls are asynchronous: they enqueue kernels on `stream`,
 * never synchronize the host and never allocate device memory (scratch space
 * is passed in as `workspace`).  They return CDLB200_OK (0) or a negative
 * CDLB200_ERR_* code; argument errors are detected on the host before any
 * launch.
 *
 * Formats follow cdl (FelysNeko/cdl):
 *   NVFP4 : e2m1 elements, blocks of 16 along the last dim, e4m3 (UE4M3, zero
 *           excluded) block scales, per-tensor fp32 alpha = amax / (6 * 448).
 *   MXFP4 : e2m1 elements, blocks of 32, e8m0 scales (alpha = 1).
 *   MXFP8 : e4m3 elements, blocks of 32, e8m0 scales (no alpha).
 * Packed FP4 stores element 2j in the low nibble of byte j.  Block scales are
 * written either linear row-major [rows, nb] (what cdl's quantizers return) or
 * in the 128x4-tiled layout consumed by the block-scaled GEMM (cdl's
 * swizzle_scale_factors, zero-padded to [ceil(rows/128)*128, ceil(nb/4)*4]).
 * A K that is not a multiple of the block is zero-padded to whole blocks, so
 * packed rows hold nb*B/2 (FP4) or nb*B (FP8) bytes, as in cdl.
 *
 * Numerics: codes and scales are bit-identical to cdl's torch nearest-round
 * path with fp32 format tables for finite inputs.  NaN/Inf are outside that
 * contract (cdl itself gives platform-dependent results for them), except
 * +-Inf in the MX formats, which follows cdl's torch path.
 */
#ifndef CDLB200_H_
#define CDLB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CDLB200_OK 0
#define CDLB200_ERR_INVALID_ARG (-1)  /* bad shape, null pointer, bad flag */
#define CDLB200_ERR_ALIGNMENT (-2)    /* pointer / leading dimension alignment */
#define CDLB200_ERR_UNSUPPORTED (-3)  /* device is not sm_100 */
#define CDLB200_ERR_LAUNCH (-4)       /* CUDA launch error (cudaGetLastError) */
#define CDLB200_ERR_TIMEOUT (-5)      /* a bounded device-side wait gave up */
#define CDLB200_ERR_WORKSPACE (-6)    /* workspace too small */
#define CDLB200_ERR_CUDA (-7)         /* other CUDA runtime error */

/* scale_layout values */
#define CDLB200_SCALE_LINEAR 0    /* [rows, nb] row-major */
#define CDLB200_SCALE_SWIZZLED 1  /* 128x4 tiles, zero-padded */

/* element types of cdlb200_quant_wide's input */
#define CDLB200_DTYPE_F32 1
#define CDLB200_DTYPE_F16 2

/* Human-readable name of a status code. */
const char* cdlb200_status_string(int status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int cdlb200_version(void);

/*
 * Poll limit of the bounded grid-wide wait in the one-launch NVFP4 quantizer
 * (default 2^20 polls, about a second); returns the previous limit.  A wait
 * that reaches the limit does not hang: the kernel records the timeout in the
 * status word of its workspace (see cdlb200_nvfp4_quant) and finishes with
 * the partial amax.  A diagnostic knob with no counterpart in the reference:
 * tests set a limit of 0 to make the wait give up and check that the timeout
 * reaches the host.
 */
uint32_t cdlb200_set_wait_limit(uint32_t polls);

/*
 * Caps the SMs that the persistent kernels fill from later launches on: the
 * pair GEMM behind cdlb200_mm_* (one CTA pair per two SMs) and the dual
 * encoder cdlb200_nvfp4_dual_multi (four CTAs per SM); 0 (the default), or
 * any value of at least the device's SM count, means all SMs.  Results do not
 * depend on it.  The data-parallel training step sets it for its backward
 * pass, where the gradient all-reduces run beside the GEMMs: the SMs left
 * free keep NCCL's kernels running instead of queued behind a kernel that
 * holds every SM.  A launch captured in a CUDA graph keeps the limit that was
 * set when it was captured.  Process-wide; no counterpart in the reference
 * (whose step runs on one GPU).  Returns CDLB200_ERR_INVALID_ARG for sms < 0.
 */
int cdlb200_set_persistent_sm_limit(int sms);

/*
 * NVFP4 quantize of a bf16 matrix.
 * Replaces cdl/core/kernel/quant.py:126-131 `nvfp4_quant` (its `_quant` host
 * code at quant.py:71-123 with group 16, e4m3 scales, and the torch global
 * amax at quant.py:96-101) and the Triton `_quant_kernel` (quant.py:13-68).
 *
 *   x        bf16 [rows, k], row stride `ldx` elements (ldx >= k)
 *   transpose 0: quantize x along its last dim (blocks of 16 along k);
 *            1: quantize x^T, i.e. blocks of 16 along `rows`; outputs are then
 *               laid out for the [k, rows] matrix (the wgrad requantize).
 *   packed   uint8 [R, nb*8]   (R, C = rows, k or k, rows; nb = ceil(C/16))
 *   scale    uint8 [R, nb] or swizzled (scale_layout)
 *   gmax     optional fp32 [1] output: max|x| clamped to FLT_MIN (may be NULL)
 *   alpha    fp32 [1] output: gmax / 2688
 *   workspace device scratch of cdlb200_nvfp4_quant_workspace_bytes() bytes,
 *            zero-filled before its first use; the call leaves it re-usable
 *            (calls sharing one workspace must be stream-ordered).  The
 *            32-bit word at byte offset 8 is the status word: the call sets
 *            it non-zero if its bounded grid-wide wait timed out (the codes
 *            of that call are then unreliable).  It stays set until the
 *            caller reads and clears it, which needs no ordering beyond the
 *            stream's.
 */
size_t cdlb200_nvfp4_quant_workspace_bytes(int64_t rows, int64_t k);
int cdlb200_nvfp4_quant(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                        void* packed, void* scale, int scale_layout, float* gmax, float* alpha,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Block-scaled quantize of an fp32 or fp16 matrix (dtype CDLB200_DTYPE_F32 /
 * CDLB200_DTYPE_F16), format 0 = NVFP4, 1 = MXFP4, 2 = MXFP8.  cdl's `_quant`
 * (cdl/core/kernel/quant.py:71-123) accepts any floating input: its Triton
 * kernel casts each block to fp32 and divides, and the NVFP4 global amax is
 * taken in the input's dtype.  This entry performs those fp32 operations
 * literally (the bf16 entry points above use bf16-exact shortcuts) and gives
 * the same codes, scale bytes and alpha.  Arguments as cdlb200_nvfp4_quant /
 * cdlb200_mx*_quant; alpha (fp32 [1]) and workspace are needed for NVFP4 only
 * (the global amax is kept in the workspace).  Not tuned: cdl's training step
 * quantizes bf16 tensors.
 */
int cdlb200_quant_wide(const void* x, int dtype, int format, int64_t rows, int64_t k, int64_t ldx, int transpose,
                       void* packed, void* scale, int scale_layout, float* alpha, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * The global-amax pass of cdlb200_nvfp4_quant on its own: gmax = max|x|
 * clamped to FLT_MIN (NaN if x holds one), alpha = gmax / 2688, as cdl's
 * `_quant` forms them before its Triton kernel (cdl/core/kernel/quant.py:96-101).
 * gmax and alpha are fp32 [1] device outputs; workspace as for
 * cdlb200_nvfp4_quant.  Feeds cdlb200_nvfp4_dual_multi (cdlb200_step.h).
 */
int cdlb200_nvfp4_amax(const void* x, int64_t rows, int64_t k, int64_t ldx, float* gmax, float* alpha,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * NVFP4 quantize that allocates nothing and takes no workspace.  It has no
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory (a host binding this C ABI from another runtime without a
 * CUDA allocator, or a runtime that owns all device memory in a fixed arena).
 * Same arguments and results as cdlb200_nvfp4_quant minus the workspace; the
 * scratch is a fixed 8 KiB array in the library's device memory, held on
 * every GPU that loads the library until it is unloaded.  Returns
 * CDLB200_ERR_WORKSPACE if a call would need more scratch than that.  The
 * first call on a device looks up that array's address, so make it before
 * any stream capture.  All calls on a device share the array: calls that
 * overlap on the GPU race.
 */
int cdlb200_nvfp4_quant_noalloc(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                                void* packed, void* scale, int scale_layout, float* gmax,
                                float* alpha, void* stream);

/*
 * MXFP4 / MXFP8 quantize of a bf16 matrix (blocks of 32, e8m0 scales).
 * Replaces cdl/core/kernel/quant.py:134-139 `mxfp4_quant` and :142-146
 * `mxfp8_quant` (their `_quant_kernel` e8m0 branch, quant.py:39-46, 56-68).
 * MXFP4 packed: uint8 [R, nb*16]; MXFP8 packed: e4m3 bytes [R, nb*32].
 * cdl's MXFP4 alpha (a constant 1.0) and MXFP8 alpha (None) are host-side.
 */
int cdlb200_mxfp4_quant(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                        void* packed, void* scale, int scale_layout, void* stream);
int cdlb200_mxfp8_quant(const void* x, int64_t rows, int64_t k, int64_t ldx, int transpose,
                        void* packed, void* scale, int scale_layout, void* stream);

/*
 * FP4 dequantize: out[r, c] = bf16((e2m1 * scale) * alpha).
 * Replaces cdl/core/kernel/dequant.py:103-109 `nvfp4_dequant` (block 16, e4m3
 * scale) and :112-118 `mxfp4_dequant` (block 32, e8m0 scale), i.e. the Triton
 * `_fp4_dequant_kernel` (dequant.py:25-47).  k must be a multiple of `block`.
 *   packed uint8 [rows, k/2], scale uint8 [rows, k/block] linear,
 *   alpha fp32 [1] (device), out bf16 [rows, k].
 */
int cdlb200_fp4_dequant(const void* packed, const void* scale, const float* alpha, int64_t rows,
                        int64_t k, int block, int scale_is_e8m0, void* out, void* stream);

/*
 * FP4 dequantize with the scales in the 128x4 tiled layout the block-scaled
 * GEMM reads ([ceil(rows/128)*128, ceil(k/block/4)*4], as written by the
 * quantizers with CDLB200_SCALE_SWIZZLED), so that a linear layer can keep one
 * scale copy for its forward GEMM and its backward dequantize.  Same result
 * as cdlb200_fp4_dequant on the linear scales.  k % 32 == 0, packed and out
 * 16-byte aligned (else CDLB200_ERR_ALIGNMENT).
 */
int cdlb200_fp4_dequant_swizzled(const void* packed, const void* scale, const float* alpha, int64_t rows,
                                 int64_t k, int block, int scale_is_e8m0, void* out, void* stream);

/*
 * MXFP8 dequantize: out = bf16(e4m3 * e8m0 [* alpha]).
 * Replaces cdl/core/kernel/dequant.py:121-143 `mxfp8_dequant` / the Triton
 * `_mxfp8_dequant_kernel` (dequant.py:50-72).  alpha may be NULL (None).
 */
int cdlb200_mxfp8_dequant(const void* packed, const void* scale, const float* alpha, int64_t rows,
                          int64_t k, void* out, void* stream);

/*
 * Scale-factor swizzle of a linear uint8 [m, b] scale matrix into the 128x4
 * tiled layout, zero-padded to [ceil(m/128)*128, ceil(b/4)*4].
 * Replaces cdl/core/mm/swizzle.py:5-14 `swizzle_scale_factors`.
 */
int cdlb200_swizzle_scales(const void* sf, int64_t m, int64_t b, void* out, void* stream);

/*
 * Block-scaled FP4 GEMM on the tcgen05 tensor cores:
 *   out[m, n] = bf16(alpha * sum_k deq(a)[m, k] * deq(b)[n, k])
 * Replaces cdl/model/wrapper/flashinfer.py:5-25 `cdl::mm_fp4` (FlashInfer
 * mm_fp4, backend "b12x", sm_120 only) as called by cdl/core/mm/nvfp4.py:36-44
 * and mxfp4.py:36-44.
 *   a        packed e2m1 [m, k/2] row-major (16-byte aligned)
 *   b        packed e2m1 [n, k/2] row-major, i.e. the storage of cdl's
 *            [k/2, n] column-major `w_theta.T`
 *   a_scale, b_scale  128x4-tiled scales of a and b (swizzle_scale_factors)
 *   alpha    fp32 [1] device scalar (x_alpha * w_alpha), NULL = 1
 *   block_size 16 with use_nvfp4 = 1 (e4m3 scales) or 32 with use_nvfp4 = 0
 *            (e8m0 scales); k must be a multiple of 32
 *   out      bf16 [m, ldo], ldo >= n
 *   status   optional device uint32: set non-zero if a bounded wait timed out
 */
int cdlb200_mm_fp4(const void* a, const void* b, const void* a_scale, const void* b_scale,
                   const float* alpha, int64_t m, int64_t n, int64_t k, int block_size, int use_nvfp4,
                   void* out, int64_t ldo, void* status, void* stream);

/*
 * cdlb200_mm_fp4 with the alpha of each operand passed separately: the
 * epilogue multiplies by RN(alpha_a * alpha_b), the product cdl forms on the
 * host side of the call (cdl/core/mm/nvfp4.py:36-44 passes x_alpha * w_alpha),
 * so the same GEMM needs no separate multiply launch.  Either may be NULL (1).
 */
int cdlb200_mm_fp4_alpha2(const void* a, const void* b, const void* a_scale, const void* b_scale,
                          const float* alpha_a, const float* alpha_b, int64_t m, int64_t n, int64_t k,
                          int block_size, int use_nvfp4, void* out, int64_t ldo, void* status, void* stream);

/*
 * cdlb200_mm_fp4_alpha2 that adds its product to the bf16 values already in
 * `out`: out = bf16(bf16(alpha_a * alpha_b * acc) + out), the fp32 sum of the
 * two bf16 values rounded once, i.e. what a torch add of the product to
 * `out` gives.  Replaces the sum autograd forms when several of cdl's
 * quantized linears read one input (q / k / v, gate / up: the input gradient
 * of each is cdl/core/mm/nvfp4.py:55-61's dgrad, and autograd adds them):
 * the dgrad GEMMs after the first accumulate into the first one's output
 * instead of writing their own and a separate add reading both.
 */
int cdlb200_mm_fp4_alpha2_acc(const void* a, const void* b, const void* a_scale, const void* b_scale,
                              const float* alpha_a, const float* alpha_b, int64_t m, int64_t n, int64_t k,
                              int block_size, int use_nvfp4, void* out, int64_t ldo, void* status, void* stream);

/*
 * Block-scaled MXFP8 GEMM (e4m3 elements, e8m0 scales, blocks of 32):
 * replaces cdl/model/wrapper/flashinfer.py:41-52 `cdl::mm_mxfp8` as called by
 * cdl/core/mm/mxfp8.py:36-51.  a: e4m3 [m, k], b: e4m3 [n, k] (storage of the
 * [k, n] column-major view), scales 128x4-tiled, k a multiple of 16; alpha
 * as above (cdl's op takes none: pass NULL).
 */
int cdlb200_mm_mxfp8(const void* a, const void* b, const void* a_scale, const void* b_scale,
                     const float* alpha, int64_t m, int64_t n, int64_t k, void* out, int64_t ldo,
                     void* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CDLB200_H_ */
