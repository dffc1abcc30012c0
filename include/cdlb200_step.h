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
 * (d % 8 == 0, d <= 2048); rstd[rows] (fp32) receives rsqrt(mean(x^2) + eps). */
int cdlb200_rmsnorm_fwd(const void* x, const void* w, int64_t rows, int64_t d, float eps, void* y, float* rstd,
                        void* stream);

/* Device scratch (bytes) cdlb200_rmsnorm_bwd needs for rows x d. */
int64_t cdlb200_rmsnorm_bwd_workspace_bytes(int64_t rows, int64_t d);

/* dx[rows, d] and dw[d] (bf16) of the RMSNorm above, given dy and the rstd
 * of the forward pass. */
int cdlb200_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, int64_t rows, int64_t d,
                        void* dx, void* dw, void* workspace, int64_t workspace_bytes, void* stream);

/* Rotary embedding of x[tokens, heads, head_dim] with cos/sin[cos_tokens,
 * head_dim] (token t uses row t % cos_tokens; head_dim % 16 == 0):
 * forward = x*cos + rotate_half(x)*sin, each product and the sum rounded to
 * bf16; backward = the gradient of that (g*cos + rotate_half^T(g*sin)). */
int cdlb200_rope(const void* x, const void* cos, const void* sin, int64_t tokens, int64_t heads, int64_t head_dim,
                 int64_t cos_tokens, int backward, void* out, void* stream);

/* h = bf16(bf16(silu(g)) * u) over n values (n % 8 == 0). */
int cdlb200_swiglu_fwd(const void* g, const void* u, int64_t n, void* h, void* stream);

/* dg, du of the SwiGLU product above, given dh. */
int cdlb200_swiglu_bwd(const void* dh, const void* g, const void* u, int64_t n, void* dg, void* du, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CDLB200_STEP_H_ */
