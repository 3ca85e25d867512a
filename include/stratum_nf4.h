/*
 * stratum_nf4.h -- C ABI of libstratum_nf4.so, the B200 (sm_100a) kernels behind
 * Stratum's NF4 frozen-weight path.
 *
 * Every entry point:
 *   - takes plain device pointers, element counts and a cudaStream_t (passed
 *     as void*) and runs on that stream's device; NULL means the legacy default
 *     stream of the device chosen with stratum_set_device() (default 0); while
 *     the stream is being captured into a CUDA graph its device cannot be
 *     queried, so the device chosen with stratum_set_device() (or by the last
 *     call) is used;
 *   - enqueues work on that stream and returns without synchronising;
 *   - allocates no device memory (callers pass outputs and workspaces);
 *   - returns STRATUM_OK (0) or a nonzero status; stratum_last_error() then
 *     holds a message for the calling thread.
 *
 * Layouts follow bitsandbytes' NF4 format, which the reference stores in its
 * NF4Payload (stratum/upload.py:70-95):
 *   packed  : uint8[ceil(n/2)], element 2i in the high nibble of byte i;
 *   absmax  : float32[ceil(n/blocksize)], one per block of the flattened tensor;
 *   code16  : float32[16], the NF4 levels (NF4Payload.code).
 * Double quantization (compress_statistics=True) replaces absmax by
 *   absmax_q: uint8[nb], absmax2: float32[ceil(nb/blocksize2)],
 *   code2: float32[256] (signed dynamic code), offset: float32[1] (device),
 * with absmax[b] = fp32(fp32(code2[absmax_q[b]] * absmax2[b/blocksize2]) + offset).
 */
#ifndef STRATUM_NF4_H
#define STRATUM_NF4_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum stratum_status {
    STRATUM_OK = 0,
    STRATUM_ERR_INVALID = 1,     /* bad argument: null pointer, size, alignment */
    STRATUM_ERR_UNSUPPORTED = 2, /* valid but not implemented (dtype, blocksize, shape) */
    STRATUM_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed */
    STRATUM_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up */
    STRATUM_ERR_NCCL = 5         /* an NCCL call failed */
};

enum stratum_dtype { STRATUM_F32 = 0, STRATUM_F16 = 1, STRATUM_BF16 = 2 };

/* ABI version; bumped on any signature change. */
int stratum_abi_version(void);

/* Message for the last nonzero status returned on the calling thread. */
const char *stratum_last_error(void);

/* Select the device used for calls made with a NULL (legacy default) stream. */
int stratum_set_device(int device);

/* Number of this library's kernel launches issued so far by this process
 * (all threads).  Used by benchmarks to count launches in a timed region. */
uint64_t stratum_launch_count(void);

/* ---------------------------------------------------------------- codec -- */

/* K1: blockwise NF4 quantization.
 * Replaces bitsandbytes.functional.quantize_4bit(A, blocksize=64,
 * compress_statistics=False, quant_type="nf4") called at
 * stratum/upload.py:367-369 and :725-727.
 *   src        : n elements of src_dtype (F32/F16/BF16), contiguous
 *   thresholds : device float32[15], sorted decision thresholds between the 16
 *                levels (q = number of thresholds strictly below x * (1/absmax))
 *   blocksize  : 32, 64, 128 or 256
 *   packed     : out uint8[ceil(n/2)]      absmax : out float32[ceil(n/blocksize)] */
int stratum_nf4_quantize(const void *src, int src_dtype, int64_t n, int blocksize,
                         const float *thresholds, uint8_t *packed, float *absmax,
                         void *stream);

/* Workspace bytes stratum_nf4_quantize_absmax_dq needs for nb blocks. */
size_t stratum_nf4_dq_workspace_bytes(int64_t nb);

/* Double quantization of a float32 absmax vector (the compress_statistics=True
 * branch of bitsandbytes' quantize_4bit; the reference always passes False at
 * stratum/upload.py:368, so this is an extension it can opt into).
 *   thresholds2 : device float32[255], midpoints of the sorted 256-entry code2
 *   blocksize2  : 256
 *   absmax_q : out uint8[nb]   absmax2 : out float32[ceil(nb/256)]
 *   offset   : out float32[1] (device) = deterministic mean of absmax
 *   workspace: >= stratum_nf4_dq_workspace_bytes(nb) bytes of device memory */
int stratum_nf4_quantize_absmax_dq(const float *absmax, int64_t nb, int blocksize2,
                                   const float *thresholds2, uint8_t *absmax_q,
                                   float *absmax2, float *offset, void *workspace,
                                   size_t workspace_bytes, void *stream);

/* NF4 quantization with double quantization in one call, for callers that
 * cannot allocate device memory for a workspace (an FFI host that only owns
 * the buffers it passes in, or code running where allocation is not
 * allowed).  This entry point has no counterpart in the reference.
 * Blocksize 64 (blocksize2 256); outputs as stratum_nf4_quantize followed by
 * stratum_nf4_quantize_absmax_dq.  Its scratch (the float32 absmax and the
 * mean's chunk sums) is one fixed array inside the library: at most 2^20
 * blocks (67,108,864 elements) per call, larger sizes return
 * STRATUM_ERR_INVALID; n == 0 returns STRATUM_OK and writes nothing (as
 * stratum_nf4_quantize); the array takes 4 MiB + 8 KiB on every GPU that loads
 * the library until the process exits.  A device's first call looks the array
 * up, so make it before any stream capture.  All calls share the array:
 * calls that overlap on the GPU (other streams, other threads) race. */
int stratum_nf4_quantize_dq_noalloc(const void *src, int src_dtype, int64_t n,
                                    const float *thresholds, const float *thresholds2,
                                    uint8_t *packed, uint8_t *absmax_q, float *absmax2,
                                    float *offset, void *stream);

/* K2: blockwise NF4 dequantization to F16/BF16/F32.
 * Replaces bitsandbytes.functional.dequantize_4bit(q, QuantState(...)) called at
 * stratum/upload.py:221, :946, :1038 and stratum/nf4_linear.py:44-46.
 *   out[i] = out_dtype(fp32(code16[q_i] * absmax[i / blocksize]))
 *   blocksize: power of two, 32..4096 */
int stratum_nf4_dequantize(const uint8_t *packed, const float *absmax, const float *code16,
                           int64_t n, int blocksize, void *out, int out_dtype, void *stream);

/* K2 with a double-quantized absmax (see the layout note at the top). */
int stratum_nf4_dequantize_dq(const uint8_t *packed, const uint8_t *absmax_q,
                              const float *absmax2, const float *code2, const float *offset,
                              int blocksize2, const float *code16, int64_t n, int blocksize,
                              void *out, int out_dtype, void *stream);

/* One NF4 tensor of a stratum_nf4_dequantize_many call: packed bytes, either
 * absmax (plain) or, with absmax == NULL, the double-quant set, its element
 * count and its output buffer. */
typedef struct stratum_nf4_tensor {
    const uint8_t *packed;
    const float *absmax;
    const uint8_t *absmax_q;
    const float *absmax2;
    const float *code2;
    const float *offset;
    int64_t n;
    void *out;
} stratum_nf4_tensor;

/* Dequantize `count` tensors (host array of descriptors) with one kernel launch
 * per 32 tensors of the same kind (plain / double quant), e.g. every frozen
 * weight of a layer.  Replaces the per-parameter dequantize_4bit loop of
 * ensure_weights (stratum/upload.py:1021-1040).  Same blocksize and out_dtype
 * for all; tensors whose n is not a multiple of 64 or whose buffers are not
 * 16-byte aligned fall back to one launch each.  Results are those of
 * stratum_nf4_dequantize / stratum_nf4_dequantize_dq. */
int stratum_nf4_dequantize_many(const stratum_nf4_tensor *tensors, int count, const float *code16,
                                int blocksize, int blocksize2, int out_dtype, void *stream);

/* -------------------------------------------------------------- GEMMs -- */

/* Status word written by the GEMM kernels when a bounded device-side wait gives
 * up (0 = ok).  Copies it to *out (host), synchronising `stream`; clears it
 * when `reset` is nonzero. */
int stratum_device_status(int *out, int reset, void *stream);

/* Diagnostic record beside the status word (8 ints, host): [0] the status, and
 * for a wait that gave up [1] block, [2] thread, [3] the parity it waited for,
 * [4] the barrier's shared-memory offset, [5..6] the barrier's 64-bit state.
 * Read it before stratum_device_status with reset, which clears it.  No
 * counterpart in the reference. */
int stratum_device_status_detail(int *out8, void *stream);

/* The whole diagnostic record (up to 72 ints; words beyond it are returned as 0):
 * the 8 of stratum_device_status_detail, then [7] the SM, [8..9] nanoseconds
 * (low word first) and [10] SM clock cycles the wait lasted, and from [12] 27
 * 64-bit shared-memory words around the barrier waited on (17 below, the
 * barrier, 9 above): the CTA's other stage barriers and, in the grouped
 * kernels, the progress words of each role.  No counterpart in the reference. */
int stratum_device_status_record(int *out, int n, void *stream);

/* Limit of every bounded device-side wait of the GEMM kernels on the stream's
 * device, in nanoseconds: 0 restores the default (2 s), otherwise 1 ms .. 60 s.
 * Synchronises `stream`.  No counterpart in the reference. */
int stratum_set_wait_limit_ns(uint64_t ns, void *stream);

/* Launches one warp that waits, through the GEMMs' bounded wait, on a barrier
 * nothing completes: after the limit in force the wait gives up and writes
 * status 0x1f0 with its record (read with stratum_device_status_record /
 * stratum_device_status), and the kernel returns -- a check of the failure path
 * that faults nothing.  No counterpart in the reference. */
int stratum_wait_selftest(void *stream);

/* GEMM kernel used by stratum_nf4_gemm_fwd and the input-gradient entry points
 * (stratum_nf4_gemm_dx, stratum_nf4_gemm_dx_pair): STRATUM_GEMM_AUTO picks by
 * estimated makespan; PAIR forces the CTA-pair kernels (512-token x 256-column
 * tiles shared by two SMs), SINGLE the one-SM kernels.  Process-wide; initially
 * from STRATUM_NF4_GEMM=pair|single, else AUTO.  Both give the same results up
 * to fp32 summation order.  No counterpart in the reference (a tuning control
 * of this library's kernels). */
enum stratum_gemm_kernel { STRATUM_GEMM_AUTO = 0, STRATUM_GEMM_PAIR = 1, STRATUM_GEMM_SINGLE = 2 };
int stratum_nf4_gemm_set_kernel(int which);

/* K3+K4: fused NF4 linear forward with the LoRA update in the same accumulator.
 * Replaces NF4Linear.forward (dequantize_4bit then F.linear,
 * stratum/nf4_linear.py:43-47) and PEFT lora.Linear's
 * y += scaling * lora_B(lora_A(x)) (scripts/train.py:568-573):
 *   y[T,N] = x[T,K] . W[N,K]^T + bias[N] + lora_xa[T,r] . lora_b[N,r]^T
 *   x        : T x K, x_dtype BF16 or F16, row-major, 16-byte aligned
 *   W        : NF4, blocksize 64 along K (K % 64 == 0): packed uint8[N*K/2] and
 *              either absmax float32[N*K/64] (absmax != NULL) or the
 *              double-quant set (absmax == NULL; absmax_q, absmax2, code2, offset)
 *   bias     : N values of bias_dtype, or NULL
 *   lora_xa  : T x ceil(r/64)*64 in x_dtype = scaling * x . lora_A^T, zero-padded
 *              columns (NULL when r == 0)
 *   lora_b   : N x r in x_dtype (r even), NULL when r == 0
 *   y        : T x N in x_dtype */
int stratum_nf4_gemm_fwd(const void *x, int x_dtype, int64_t T, int64_t K,
                         const uint8_t *packed, const float *absmax,
                         const uint8_t *absmax_q, const float *absmax2,
                         const float *code2, const float *offset, const float *code16,
                         int64_t N, const void *bias, int bias_dtype,
                         const void *lora_xa, const void *lora_b, int r,
                         void *y, void *stream);

/* K3+K4 backward: fused NF4 input gradient with the LoRA term.
 * Replaces the autograd backward of NF4Linear.forward's F.linear
 * (stratum/nf4_linear.py:47) and of PEFT lora.Linear (scripts/train.py:568-573):
 *   dx[T,K] = dy[T,N] . W[N,K] + lora_dyb[T,r] . lora_a[r,K]
 *   dy       : T x N (N % 8 == 0), dtype BF16 or F16, 16-byte aligned
 *   W        : as in stratum_nf4_gemm_fwd, K % 64 == 0
 *   lora_dyb : T x ceil(r/64)*64 = scaling * dy . lora_B, zero-padded (NULL when r == 0)
 *   lora_a   : r x K, 16-byte aligned (NULL when r == 0)
 *   dx       : T x K */
int stratum_nf4_gemm_dx(const void *dy, int dtype, int64_t T, int64_t N,
                        const uint8_t *packed, const float *absmax,
                        const uint8_t *absmax_q, const float *absmax2,
                        const float *code2, const float *offset, const float *code16,
                        int64_t K, const void *lora_dyb, const void *lora_a, int r,
                        void *dx, void *stream);

/* One NF4 weight for the fused MLP entry points below: packed bytes and either
 * absmax (plain) or, with absmax == NULL, the double-quant set. */
typedef struct stratum_nf4_weight {
    const uint8_t *packed;
    const float *absmax;
    const uint8_t *absmax_q;
    const float *absmax2;
    const float *code2;
    const float *offset;
} stratum_nf4_weight;

/* Fused SwiGLU up-projection of a dense MLP (LlamaMLP / Qwen3MLP with two
 * NF4Linear + PEFT LoRA projections and SiLU): one GEMM pass over x computes
 *   gate = x . Wg^T + lora_xa[:, 0:r] . lora_b_gate^T
 *   up   = x . Wu^T + lora_xa[:, rp:rp+r] . lora_b_up^T     (rp = ceil(r/64)*64)
 *   h    = r16(r16(silu(r16(gate))) * r16(up))              (HF's bf16 forward)
 * Replaces act_fn(gate_proj(x)) * up_proj(x) of the reference's MLP, whose
 * fused-memory variant is stratum/model/mlp_opt.py:154-245 (MemoryFlatFrozenMLP).
 *   x          : T x K (K % 64 == 0), BF16 or F16, 16-byte aligned
 *   gate, up   : NF4 weights I x K (I % 64 == 0), both plain or both double quant
 *   lora_xa    : T x 2*rp in x's dtype = [scaling_g * x . A_g^T | 0 | scaling_u * x . A_u^T | 0]
 *                (NULL when r == 0)
 *   lora_b_*   : I x r (r even, <= 256), NULL when r == 0
 *   h          : T x I;  gate_out / up_out: T x I (the 16-bit gate and up, for the
 *                backward), or NULL */
int stratum_nf4_gemm_swiglu_fwd(const void *x, int x_dtype, int64_t T, int64_t K,
                                const stratum_nf4_weight *gate, const stratum_nf4_weight *up,
                                const float *code16, int64_t I, const void *lora_xa,
                                const void *lora_b_gate, const void *lora_b_up, int r,
                                void *h, void *gate_out, void *up_out, void *stream);

/* Input gradient through two NF4 weights stacked along N (the gate and up
 * projections of a SwiGLU MLP), one pass:
 *   dx[T,K] = dy[T, N0+N1] . [W0; W1] + lora_dyb[T, r] . lora_a[r, K]
 * Replaces the two F.linear backwards (and PEFT LoRA's) of gate_proj and
 * up_proj, summed by autograd.  N0, N1 multiples of 64; both weights plain or
 * both double quantized; lora_dyb / lora_a as in stratum_nf4_gemm_dx, e.g. the
 * two adapters' terms side by side. */
int stratum_nf4_gemm_dx_pair(const void *dy, int dtype, int64_t T,
                             const stratum_nf4_weight *w0, int64_t N0,
                             const stratum_nf4_weight *w1, int64_t N1,
                             const float *code16, int64_t K, const void *lora_dyb,
                             const void *lora_a, int r, void *dx, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* STRATUM_NF4_H */
