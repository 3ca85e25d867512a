/*
 * stratum_layers.h -- C ABI of the fused decoder-layer kernels in libstratum_nf4.so.
 *
 * The reference's decoder layers are HF Llama / Qwen3 layers
 * (stratum/model/llama.py:252-331, stratum/model/qwen3.py) whose RMSNorm, rotary
 * embedding and SwiGLU activation run as chains of torch kernels around the
 * frozen linears this library replaces.  These entry points do each in one
 * pass over HBM, with the same bf16 / fp16 roundings as the HF forward, plus
 * the exact backward.  Conventions of stratum_nf4.h (device pointers, the
 * caller's stream, no allocation, status codes).  16-bit tensors are bf16 or
 * fp16 (dtype), 16-byte aligned.
 */
#ifndef STRATUM_LAYERS_H
#define STRATUM_LAYERS_H

#include "stratum_nf4.h"

#ifdef __cplusplus
extern "C" {
#endif

/* LlamaRMSNorm.forward over rows of n (n % 8 == 0):
 *   y = round(weight * round(x * rsqrt(mean(x^2) + eps))); rstd[row] (float32) saved
 *   for the backward (may be NULL). */
int stratum_rmsnorm_fwd(const void *x, const void *weight, int dtype, int64_t rows, int64_t n, float eps, void *y,
                        float *rstd, void *stream);

/* Input gradient of stratum_rmsnorm_fwd (the weight is frozen: no weight gradient). */
int stratum_rmsnorm_bwd(const void *x, const void *weight, const void *dy, const float *rstd, int dtype,
                        int64_t rows, int64_t n, void *dx, void *stream);

/* x [S, H, D] token-major -> y [H, S, D] head-major (D % 16 == 0); with cos / sin
 * ([S, D], the rotary table in dtype) applies apply_rotary_pos_emb:
 *   y = round(round(x * cos) + round(rotate_half(x) * sin)); with NULL tables, a copy. */
int stratum_rope_to_heads(const void *x, const void *cos_t, const void *sin_t, int dtype, int S, int H, int D,
                          void *y, void *stream);

/* Adjoint of stratum_rope_to_heads: dy [H, S, D] -> dx [S, H, D] (NULL tables: a copy,
 * which is also the head-major -> token-major move of the attention output). */
int stratum_rope_from_heads(const void *dy, const void *cos_t, const void *sin_t, int dtype, int S, int H, int D,
                            void *dx, void *stream);

/* LlamaMLP's act_fn(gate) * up with SiLU: h = round(round(silu(gate)) * up), n % 8 == 0. */
int stratum_swiglu_fwd(const void *gate, const void *up, int dtype, int64_t n, void *h, void *stream);

/* Its backward: dup = dh * round(silu(gate)); dgate = round(dh * up) * s * (1 + gate * (1 - s)),
 * s = sigmoid(gate). */
int stratum_swiglu_bwd(const void *gate, const void *up, const void *dh, int dtype, int64_t n, void *dgate, void *dup,
                       void *stream);

/* The same backward with the two gradients written side by side as rows of
 * dgate_up[rows, 2I] = [dgate | dup] (gate, up, dh: [rows, I], I % 8 == 0): the dY
 * of the stacked gate/up input gradient, stratum_nf4_gemm_dx_pair. */
int stratum_swiglu_bwd_cat(const void *gate, const void *up, const void *dh, int dtype, int64_t rows, int64_t I,
                           void *dgate_up, void *stream);

/* Next-token cross entropy of one row of logits per token, forward and gradient
 * in one pass (replaces the log_softmax / nll / autograd chain of the reference's
 * chunked_linear_cross_entropy, stratum/model/chunked_loss.py):
 *   loss[row]  = logsumexp(logits[row]) - logits[row][labels[row]]   (0 where
 *                labels[row] == ignore_index), computed in fp32
 *   logits[row] is overwritten with (softmax(logits[row]) - onehot) * scale
 *                (zeros for ignored rows), in dtype
 * logits: rows x vocab, vocab % 8 == 0; labels int64[rows] in [0, vocab) or
 * ignore_index (any other value is treated as ignored); loss float32[rows]. */
int stratum_ce_fwd_grad(void *logits, int dtype, const int64_t *labels, int64_t rows, int64_t vocab,
                        int64_t ignore_index, float scale, float *loss, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* STRATUM_LAYERS_H */
