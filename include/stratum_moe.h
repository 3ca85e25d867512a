/*
 * stratum_moe.h -- C ABI of the routed-expert (MoE) part of libstratum_nf4.so.
 *
 * Replaces the per-expert loop of HF Qwen3MoeExperts.forward that the reference
 * runs over NF4-staged 3-D expert weights (stratum/model/qwen3_moe.py builds the
 * layers; stratum/upload.py:361-366 flattens gate_up_proj [E, 2I, H] to
 * [E*2I, H] and down_proj [E, H, I] to [E*H, I] before quantize_4bit; the loop
 * itself is transformers' modeling_qwen3_moe.py Qwen3MoeExperts.forward):
 *
 *   for each expert e hit by the router:
 *       gate, up = chunk(x[tokens_e] . gate_up_proj[e]^T, 2)
 *       h        = silu(gate) * up
 *       y        = (h . down_proj[e]^T) * top_k_weights[tokens_e, slot]
 *       out.index_add_(0, tokens_e, y)
 *
 * The same work here: stratum_moe_route sorts the T*k (token, slot) pairs by
 * expert; stratum_moe_gather_rows builds x_sorted; two grouped NF4 GEMMs
 * (gate_up with the SwiGLU epilogue, then down) run over every expert in one
 * launch each; stratum_moe_combine sums each token's k rows with their routing
 * weights.  The backward uses stratum_moe_combine_grad, stratum_nf4_grouped_dx
 * (down, then gate_up) and stratum_swiglu_grad.
 *
 * Conventions are those of stratum_nf4.h (device pointers, caller's stream,
 * no allocation, status codes, stratum_last_error).  Expert weights are NF4 with
 * blocksize 64 along their last dimension, flattened as above: packed
 * uint8[E*N_e*K/2], absmax float32[E*N_e*K/64] or the double-quant set.
 * Routing indices are int32 except the router's int64 expert ids.
 */
#ifndef STRATUM_MOE_H
#define STRATUM_MOE_H

#include "stratum_nf4.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Workspace bytes stratum_moe_route needs for n_pairs = T*k pairs. */
size_t stratum_moe_route_workspace_bytes(int64_t n_pairs, int n_experts);

/* Stable counting sort of the routing pairs by expert (replaces the one_hot /
 * torch.where bookkeeping of Qwen3MoeExperts.forward).
 *   experts  : int64[T*k], the router's top-k expert ids (row-major [T, k]); an
 *              id outside [0, E) -- HF's "expert_idx == num_experts" skip value
 *              included -- drops that pair: it is sorted after every routed
 *              pair and contributes nothing
 *   order    : int32[T*k] out, order[p] = flat pair index j = t*k + slot of sorted row p
 *   inv      : int32[T*k] out, inv[j] = sorted row of pair j
 *   token_of : int32[T*k] out, token_of[p] = order[p] / k
 *   offsets  : int32[E+1] out, expert e owns sorted rows [offsets[e], offsets[e+1]);
 *              offsets[E] = number of routed (not dropped) pairs
 * E <= 1023. */
int stratum_moe_route(const int64_t *experts, int64_t T, int k, int E, int *order, int *inv, int *token_of,
                      int *offsets, void *workspace, size_t workspace_bytes, void *stream);

/* dst[p, :] = src[idx[p], :] for p < rows (row_bytes % 16 == 0, 16-byte aligned):
 * the hidden_states[token_idx] gather of Qwen3MoeExperts.forward for all experts. */
int stratum_moe_gather_rows(const void *src, int64_t row_bytes, const int *idx, int64_t rows, void *dst,
                            void *stream);

/* Bytes of the tile table the grouped GEMMs build on the device from the expert
 * offsets, for total_tokens sorted rows, E experts and weight_dim = the larger of
 * N_e and K of the call (one table serves both directions).  The table buffer
 * must be 16-byte aligned. */
size_t stratum_nf4_grouped_table_bytes(int64_t total_tokens, int n_experts, int64_t weight_dim);

/* Grouped NF4 forward over all experts in one launch:
 *   y[p, :] = x_sorted[p, :] . W[e(p)]^T     for offsets[0] <= p < offsets[E]
 *   x_sorted : Ttot x K, dtype BF16 or F16, 16-byte aligned, K % 64 == 0
 *   W        : expert e's rows are e*N_e .. e*N_e + N_e - 1 of the flattened
 *              [E*N_e, K] NF4 weight; N_e % 128 == 0; absmax == NULL selects the
 *              double-quant set (absmax_q, absmax2, code2, offset)
 *   swiglu=0 : y is Ttot x N_e; rw (float32[Ttot], per sorted row, or NULL)
 *              scales each row (Qwen3MoeExperts' "* top_k_weights")
 *   swiglu=1 : W is gate_up_proj (rows [0, N_e/2) gate, [N_e/2, N_e) up); y is
 *              Ttot x N_e/2 holding h = silu(gate) * up, computed from gate and
 *              up rounded to dtype (as HF's forward in that dtype computes it);
 *              gate_up (Ttot x N_e, optional) receives gate|up themselves for
 *              the backward
 * Rows of y outside [offsets[0], offsets[E]) are not written.  Offsets that are
 * decreasing or outside [0, Ttot] write nothing and set the status word read
 * by stratum_device_status. */
int stratum_nf4_grouped_fwd(const void *x_sorted, int dtype, int64_t Ttot, int K, const int *offsets, int E,
                            const uint8_t *packed, const float *absmax, const uint8_t *absmax_q,
                            const float *absmax2, const float *code2, const float *offset, const float *code16,
                            int N_e, int swiglu, const float *rw, void *y, void *gate_up, void *table,
                            size_t table_bytes, void *stream);

/* Grouped NF4 input gradient (the autograd backward of the per-expert F.linear):
 *   dx[p, :] = dy_sorted[p, :] . W[e(p)]     dy_sorted Ttot x N_e (N_e % 64 == 0),
 *                                            dx Ttot x K (K % 64 == 0) */
int stratum_nf4_grouped_dx(const void *dy_sorted, int dtype, int64_t Ttot, int N_e, const int *offsets, int E,
                           const uint8_t *packed, const float *absmax, const uint8_t *absmax_q,
                           const float *absmax2, const float *code2, const float *offset, const float *code16,
                           int K, void *dx, void *table, size_t table_bytes, void *stream);

/* out[t, :] = sum_{s<k} w[t*k+s] * rows[inv[t*k+s], :] in fp32, stored in dtype
 * (the routing-weight product and index_add_ of Qwen3MoeExperts.forward);
 * weights NULL means 1; dropped pairs (inv >= offsets[E]) are skipped.
 * width % 8 == 0, rows and out 16-byte aligned. */
int stratum_moe_combine(const void *rows, int dtype, const int *inv, const float *weights, const int *offsets,
                        int E, int64_t T, int k, int64_t width, void *out, void *stream);

/* Backward of stratum_moe_combine, per sorted row p (pair j = order[p]):
 *   dy_sorted[p, :] = w[j] * dout[token_of[p], :]            (weights NULL means 1)
 *   dweights[j]     = <dout[token_of[p], :], rows[p, :]>    (fp32; skipped when dweights is NULL)
 * Dropped pairs get zero rows and zero weight gradients. */
int stratum_moe_combine_grad(const void *dout, int dtype, const int *order, const int *token_of,
                             const float *weights, const int *offsets, int E, const void *rows, int64_t n_rows,
                             int64_t width, void *dy_sorted, float *dweights, void *stream);

/* d(gate|up) of h = silu(gate) * up (the autograd backward of
 * "self.act_fn(gate) * up" in Qwen3MoeExperts.forward):
 *   gate_up, dgate_up : rows x 2*inter ([gate | up]);  dh : rows x inter;  inter % 8 == 0 */
int stratum_swiglu_grad(const void *gate_up, const void *dh, int dtype, int64_t rows, int64_t inter, void *dgate_up,
                        void *stream);

#ifdef __cplusplus
}
#endif

#endif /* STRATUM_MOE_H */
