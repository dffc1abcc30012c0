/*
 * cdlb200_step.h -- fused elementwise operations of the SmolLM2 (Llama) QAT
 * step (the rest of the step around the quantized linears).  They replace the
 * eager modules the reference's training script runs through Hugging Face
 * transformers (cdl's smollm2.py builds a LlamaForCausalLM): LlamaRMSNorm,
 * apply_rotary_pos_emb and the SwiGLU product of LlamaMLP.  Same conventions
 * as cdlb200.h: bf16 tensors, row-major, 16-byte aligned rows, caller-owned
 * buffers, the stream passed as a cudaStream_t cast to void*, status codes
 * from cdlb200.h.
 */
#ifndef CDLB200_STEP_H_
#define CDLB200_STEP_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) per row of x[rows, d]
 * (d % 8 == 0, d <= 2048); rstd[rows] (fp32) receives rsqrt(mean(x^2) + eps).
 * amax (optional): CDLB200_AMAX_WORDS words, zero on entry, whose maximum
 * becomes the bf16 magnitude bits of max|y| -- the global amax the NVFP4
 * quantize of y needs, formed in the epilogue so that the quantize skips its
 * own amax pass (cdlb200_nvfp4_encode_multi).  The CTAs spread their atomics
 * over the words. */
#define CDLB200_AMAX_WORDS 32
int cdlb200_rmsnorm_fwd(const void* x, const void* w, int64_t rows, int64_t d, float eps, void* y, float* rstd,
                        uint32_t* amax, void* stream);

/* The decoder's residual add fused with the RMSNorm that follows it
 * (transformers' LlamaDecoderLayer: hidden = residual + branch, then the next
 * norm of hidden): h = bf16(res + x) is written to h and normalized into y as
 * above.  Same outputs as a bf16 add followed by cdlb200_rmsnorm_fwd(h). */
int cdlb200_add_rmsnorm_fwd(const void* res, const void* x, const void* w, int64_t rows, int64_t d, float eps,
                            void* h, void* y, float* rstd, uint32_t* amax, void* stream);

/* Device scratch (bytes) cdlb200_rmsnorm_bwd needs for rows x d. */
int64_t cdlb200_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t d);

/* dx[rows, d] and dw[d] (bf16) of the RMSNorm above, given dy and the rstd
 * of the forward pass. */
int cdlb200_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, int64_t rows, int64_t d,
                        void* dx, void* dw, void* workspace, int64_t workspace_bytes, void* stream);

/* cdlb200_rmsnorm_bwd for cdlb200_add_rmsnorm_fwd: dx = bf16(norm's dx +
 * dres), the gradient of both inputs of the residual add (dres = the
 * gradient of h from its other consumer; NULL: none), with amax (optional,
 * CDLB200_AMAX_WORDS words, zero on entry) receiving the bf16 magnitude
 * maximum of dx -- the o / down projections' gradient the quantized backward
 * encodes.  x is the forward's h. */
int cdlb200_rmsnorm_bwd_add(const void* dy, const void* x, const void* w, const float* rstd, const void* dres,
                            int64_t rows, int64_t d, void* dx, void* dw, uint32_t* amax, void* workspace,
                            int64_t workspace_bytes, void* stream);

/* Rotary embedding of x[tokens, heads, head_dim] with cos/sin[cos_tokens,
 * head_dim] (token t uses row t % cos_tokens; head_dim % 16 == 0):
 * forward = x*cos + rotate_half(x)*sin, each product and the sum rounded to
 * bf16; backward = the gradient of that (g*cos + rotate_half^T(g*sin)).
 * amax (optional, CDLB200_AMAX_WORDS words, zero on entry) receives the bf16
 * magnitude maximum of out, as for the RMSNorm above (the backward's output
 * is the q / k projections' gradient, which the quantized backward encodes). */
int cdlb200_rope(const void* x, const void* cos, const void* sin, int64_t tokens, int64_t heads, int64_t head_dim,
                 int64_t cos_tokens, int backward, void* out, uint32_t* amax, void* stream);

/* h = bf16(bf16(silu(g)) * u) over n values (n % 8 == 0); amax (optional,
 * CDLB200_AMAX_WORDS words, zero on entry) as for the RMSNorm above. */
int cdlb200_swiglu_fwd(const void* g, const void* u, int64_t n, void* h, uint32_t* amax, void* stream);

/* dg, du of the SwiGLU product above, given dh; amax_dg / amax_du (optional,
 * CDLB200_AMAX_WORDS words each, zero on entry) receive the bf16 magnitude
 * maxima of dg and du, so that their NVFP4 encodings in the quantized
 * backward skip a separate amax pass. */
int cdlb200_swiglu_bwd(const void* dh, const void* g, const void* u, int64_t n, void* dg, void* du,
                       uint32_t* amax_dg, uint32_t* amax_du, void* stream);

/* Cross entropy of bf16 logits[rows, vocab] (contiguous, vocab % 8 == 0)
 * against int64 targets[rows], the per-chunk step of the reference's fused
 * linear cross entropy (Liger, used by cdl smollm2.py for the LM head):
 *   lse = log(sum exp(x - max x)) + max x (fp32),  loss[r] = lse - x[r, t_r],
 *   logits <- bf16((exp(x - lse) - onehot(t_r)) * scale)   (in place),
 * with scale = 1/n the gradient of sum(loss) / n (torch divides a tensor by a
 * scalar n as a multiply by the fp32 reciprocal).  A target outside
 * [0, vocab) gives loss 0 and a zero gradient row. */
int cdlb200_cross_entropy(void* logits, const int64_t* targets, int64_t rows, int64_t vocab, float scale,
                          float* loss, void* stream);

/* x[0..n) *= *scale in place: bf16 x (16-byte aligned, n % 8 == 0) times a
 * bf16 scalar held in device memory, each product rounded to bf16 as torch
 * multiplies two bf16 tensors.  The backward of the fused linear cross
 * entropy above (Liger's, as cdl smollm2.py:667-677 uses it) multiplies the
 * gradients it stored in the forward by grad_output; this does it in place,
 * reading the scale on the device, and leaves x untouched when the scale is
 * 1 (the loss's own backward), which gives the same bits for every value but
 * a NaN's payload. */
int cdlb200_scale_bf16(void* x, int64_t n, const void* scale, void* stream);

/* One parameter tensor of the optimizer below: param, its gradient and the
 * two AdamW moments, all bf16, contiguous, 16-byte aligned, numel % 8 == 0. */
typedef struct {
    void* param;
    const void* grad;
    void* exp_avg;
    void* exp_avg_sq;
    int64_t numel;
    /* optional (NULL: none): receives the bf16 magnitude bits of max|param|
     * after the update, the global amax an NVFP4 encode of the new weights
     * needs (cdlb200_nvfp4_encode_multi) */
    uint32_t* amax;
} cdlb200_adamw_tensor;

/* Device workspace (bytes) cdlb200_clip_adamw needs for these tensors. */
int64_t cdlb200_clip_adamw_workspace_bytes(const cdlb200_adamw_tensor* tensors, int count);

/* Gradient clipping and one AdamW step over all tensors, as the reference's
 * training step runs them (cdl smollm2.py: torch.nn.utils.clip_grad_norm_
 * then torch.optim.AdamW with its default foreach implementation):
 *   norm_i = bf16(||grad_i||_2), norm = bf16(sqrt(sum norm_i^2)),
 *   coef   = min(bf16(bf16(1 / bf16(norm + 1e-6)) * max_norm), 1),  g = bf16(grad * coef),
 *   step  += 1,  p = bf16(p * (1 - lr*wd)),  m = bf16(lerp(m, g, 1 - b1)),
 *   v = bf16(bf16(v * b2) + (1 - b2) * g*g),
 *   s = bf16(bf16(bf16(sqrt(v)) / sqrt(1 - b2^step)) + eps),
 *   p = bf16(p - lr/(1 - b1^step) * (m / s)),
 * each operation in fp32 with fp32 scalars, as torch's list kernels compute
 * it; max_norm <= 0 disables the clip (coef = 1).  The step counter lives in
 * the workspace, which must be zero-filled before the first step and kept
 * between steps.  grad_norm (device fp32, optional) receives norm.  Three
 * kernel launches per 512 tensors, no host synchronization. */
int cdlb200_clip_adamw(const cdlb200_adamw_tensor* tensors, int count, double max_norm, double lr,
                       double beta1, double beta2, double eps, double weight_decay, void* workspace,
                       int64_t workspace_bytes, float* grad_norm, void* stream);

/* One tensor of the multi-tensor NVFP4 encoder below. */
typedef struct {
    const void* x;         /* bf16 [rows, k], contiguous, 16-byte aligned */
    int64_t rows, k;       /* k % 16 == 0; rows % 128 == 0 and (k/16) % 4 == 0 (swizzled scales need no padding) */
    const uint32_t* amax;  /* bf16 magnitude bits of max|x|: the maximum of amax_words words */
    int32_t amax_words;    /* 1 (cdlb200_clip_adamw's word) or CDLB200_AMAX_WORDS (the RMSNorm / SwiGLU epilogues) */
    int32_t pad;
    void* packed;          /* uint8 [rows, k/2]: e2m1 codes, element 2j in the low nibble */
    void* scale;           /* uint8 [rows, k/16] in the 128x4 GEMM layout */
    float* alpha;          /* fp32 [1]: gmax / 2688 */
    void* deq;             /* optional bf16 [rows, k]: bf16((e2m1 * scale) * alpha), the backward operand */
} cdlb200_nvfp4_encode_tensor;

/* NVFP4 quantize of many tensors whose global amax is already known (the
 * weights of a QAT step, right after the optimizer wrote them and their
 * amax): the same codes, scale bytes and alpha as cdlb200_nvfp4_quant with
 * CDLB200_SCALE_SWIZZLED, plus the dequantized copy the bf16 backward GEMMs
 * read, for all tensors in one pass (one launch per 256 tensors).  Replaces,
 * per QLinear, the weight quantize of the forward (cdl core/mm/nvfp4.py) and
 * the weight dequantize of the backward (dequant.py:103-109). */
int cdlb200_nvfp4_encode_multi(const cdlb200_nvfp4_encode_tensor* tensors, int count, void* stream);

/* One tensor of the dual NVFP4 encoder below. */
#define CDLB200_DUAL_ROW_LINEAR 1
#define CDLB200_DUAL_COL_LINEAR 2
typedef struct {
    const void* x;          /* bf16 [rows, cols], contiguous, 16-byte aligned; rows % 64 == 0, cols % 64 == 0 */
    int64_t rows, cols;
    const uint32_t* amax;   /* bf16 magnitude bits of max|x| (the maximum of amax_words words), or NULL and ... */
    const float* gmax;      /* ... max|x| as fp32 (cdlb200_nvfp4_quant's gmax output, e.g. of its amax pass) */
    int32_t amax_words;     /* 1..64 with amax */
    int32_t flags;          /* CDLB200_DUAL_ROW_LINEAR / CDLB200_DUAL_COL_LINEAR: that encoding's scales
                               linear [rows, cols/16] / [cols, rows/16] instead of the 128x4 layout */
    float* alpha;           /* fp32 [1] output: gmax / 2688, the alpha of both encodings */
    void* row_packed;       /* optional (NULL: skipped): uint8 [rows, cols/2], x in blocks of 16 along cols, 8-byte aligned */
    void* row_scale;        /* uint8, the 128x4 GEMM layout of [rows, cols/16] (rows padded to 128), or linear */
    void* col_packed;       /* optional: uint8 [cols, rows/2], x^T in blocks of 16 along rows, 16-byte aligned */
    void* col_scale;        /* uint8, the 128x4 GEMM layout of [cols, rows/16] (cols padded to 128), or linear */
} cdlb200_nvfp4_dual_tensor;

/* NVFP4 encodings of x and of x^T from one read of x, for many tensors in one
 * launch (per 128 tensors): the codes, scale bytes and alpha that
 * cdlb200_nvfp4_quant (CDLB200_SCALE_SWIZZLED) writes for x (transpose 0) and
 * for x^T (transpose 1), with the global amax given.  They are the operands of
 * the quantized backward GEMMs of a linear layer out = x w^T with gradient g:
 * dgrad = Q(g) Q(w^T)^T, wgrad = Q(g^T) Q(x^T)^T, where cdl's backward
 * (cdl/core/mm/nvfp4.py:46-63) multiplies bf16 g by dequantized operands
 * instead; each encoding is cdl's quantize (cdl/core/kernel/quant.py:71-131)
 * of that matrix.  Padding rows of a scale matrix (rows or cols not a
 * multiple of 128) are zeroed. */
int cdlb200_nvfp4_dual_multi(const cdlb200_nvfp4_dual_tensor* tensors, int count, void* stream);

/* ECDL stochastic quantizer (cdl/core/kernel/ecdl: launch.py launch_ecdl_fwd /
 * launch_ecdl_bwd, kernel.py _ecdl_fwd / _ecdl_bwd).  theta is bf16 (theta_f32
 * = 0) or fp32, [rows, nb * block] with block 16 (NVFP4) or 32 (MXFP4 /
 * MXFP8).  Forward: per block a scale (nvidia mode: UE4M3 index from
 * block amax * 448 / global amax, alpha = global amax / 2688; OCP mode: E8M0
 * from the block exponent, alpha = 1), then for every element a level index
 * sampled from the top-k window around x / s with weights
 * exp(-kappa (c - t)^2) and the uniform number of Triton's
 * tl.rand(seed, flat index) (Philox4x32-10).  packed: FP4 codes (two per
 * byte, element 2j low) or e4m3 bytes; scale: [rows, nb] bytes (index + 1
 * for UE4M3).  kappa (fp32) and seed (int64, low 32 bits used) are device
 * scalars; workspace >= 4 bytes.  Backward: dtheta = g * dE[level]/dx of the
 * CDL proxy with kappa (forward's or a fixed backward kappa), and, when
 * scalars is given, scalars = {d kappa, d alpha}. */
#define CDLB200_ECDL_NVFP4 0
#define CDLB200_ECDL_MXFP4 1
#define CDLB200_ECDL_MXFP8 2
#define CDLB200_ECDL_NVIDIA 0
#define CDLB200_ECDL_OCP 1
int cdlb200_ecdl_fwd(const void* theta, int theta_f32, int64_t rows, int64_t nb, int format, int scale_mode,
                     const float* kappa, const int64_t* seed, int topk, void* packed, void* scale, float* alpha,
                     void* workspace, void* stream);
int64_t cdlb200_ecdl_bwd_workspace_bytes(int64_t rows, int64_t nb, int format);
int cdlb200_ecdl_bwd(const void* grad, const void* theta, int theta_f32, int64_t rows, int64_t nb, int format,
                     const void* scale, const float* kappa, const float* alpha, int topk, void* dtheta,
                     float* scalars, void* workspace, int64_t workspace_bytes, void* stream);

/* CCDL stochastic quantizer (cdl/core/kernel/ccdl: launch.py launch_ccdl_fwd /
 * launch_ccdl_bwd, kernel.py _ccdl_fwd / _ccdl_bwd).  As ECDL, except that
 * each block's scale is a learnable value q (fp32 [rows, nb], or one shared
 * row when q_stride is 0) sampled on the scale grid (UE4M3 without zero for
 * NVFP4, E8M0 for MX) with the truncated window of q_topk levels and kappa_q,
 * from tl.rand(seed, rows * nb * block + r * q_stride + b); s = q_level *
 * alpha (alpha a learnable fp32 scalar).  scale: [rows, nb] bytes.
 * Backward: dtheta; dq[rows, nb] (per theta row; optional) = alpha *
 * sum_block(g * ds) * dE[q level]/dq; scalars (optional) = {d kappa_t,
 * d kappa_q, d alpha}.  scale_stride 0 reads one shared scale row. */
int cdlb200_ccdl_fwd(const void* theta, int theta_f32, int64_t rows, int64_t nb, int format, const float* q,
                     int64_t q_stride, const float* kappa_t, const float* kappa_q, const float* alpha,
                     const int64_t* seed, int theta_topk, int q_topk, void* packed, void* scale, void* stream);
int64_t cdlb200_ccdl_bwd_workspace_bytes(int64_t rows, int64_t nb, int format);
int cdlb200_ccdl_bwd(const void* grad, const void* theta, int theta_f32, int64_t rows, int64_t nb, int format,
                     const float* q, int64_t q_stride, const void* scale, int64_t scale_stride, const float* kappa_t,
                     const float* kappa_q, const float* alpha, int theta_topk, int q_topk, void* dtheta, float* dq,
                     float* scalars, void* workspace, int64_t workspace_bytes, void* stream);

/* CCDL deterministic (eval-mode) quantize, replacing the torch
 * cascaded_nearest_round of cdl/core/ccdl.py:78-89 that
 * CascadedCdlQuant.eval_forward (cdl/model/components/quant/ccdl/ccdl.py:146-162)
 * calls: q to its nearest scale level, s = level * alpha in the level dtype
 * (levels_bf16: rounded to bf16), theta to the nearest level of theta / s
 * (rounded to bf16 when theta and the levels are both bf16).  Same layouts
 * as cdlb200_ccdl_fwd; scale is written for every row. */
int cdlb200_ccdl_round(const void* theta, int theta_f32, int64_t rows, int64_t nb, int format, const float* q,
                       int64_t q_stride, const float* alpha, int levels_bf16, void* packed, void* scale,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CDLB200_STEP_H_ */
