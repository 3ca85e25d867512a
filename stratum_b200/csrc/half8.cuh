// 16-bit element helpers and the SwiGLU element arithmetic, shared by the
// standalone SwiGLU kernels (fused_ops.cu) and the NF4 GEMM epilogues that
// fuse SwiGLU (nf4_gemm.cu), so both round exactly alike:
//   forward   h  = r16(r16(silu(g)) * u)                         (HF LlamaMLP in bf16/fp16)
//   backward  du = r16(dh * r16(silu(g)))
//             dg = r16(r16(dh * u) * s * (1 + g * (1 - s))),  s = sigmoid(g)
// where r16 rounds to the 16-bit type (torch's silu_backward order).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace stratum {
namespace h16 {

template <bool BF16>
__device__ __forceinline__ float ld1(const uint16_t v) {
    if constexpr (BF16) return __uint_as_float(uint32_t(v) << 16);
    else return __half2float(__ushort_as_half(v));
}

template <bool BF16>
__device__ __forceinline__ uint16_t st1(float f) {
    if constexpr (BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(f));
    else return __half_as_ushort(__float2half_rn(f));
}

template <bool BF16>
__device__ __forceinline__ float rnd(float f) {  // round to the 16-bit type and back
    return ld1<BF16>(st1<BF16>(f));
}

template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4 v, float f[8]) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = ld1<BF16>(h[i]);
}

template <bool BF16>
__device__ __forceinline__ uint4 pack8(const float f[8]) {
    uint4 v;
    uint16_t *h = reinterpret_cast<uint16_t *>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = st1<BF16>(f[i]);
    return v;
}

__device__ __forceinline__ float sigmoid_f(float g) { return 1.f / (1.f + expf(-g)); }

// h for one element from the 16-bit gate and up values (as floats).
template <bool BF16>
__device__ __forceinline__ float swiglu_fwd1(float g, float u) {
    return rnd<BF16>(g / (1.f + expf(-g))) * u;
}

// True when fp32 v lies within `margin` fp32 ulps of a round-to-nearest-even
// boundary of bf16 (the dropped 16 bits near 0x8000), i.e. where an error of
// fewer than `margin` ulps in v could change its bf16 rounding.
__device__ __forceinline__ bool near_bf16_tie(float v, int margin) {
    const int low = int(__float_as_uint(v) & 0xFFFFu) - 0x8000;
    return low < margin && low > -margin;
}

// h for 8 elements, the same values as swiglu_fwd1 at a third of its cost: silu
// from the approximate exp and divide (relative error below 2^-20 for |g| <= 16:
// ex2.approx, the rounding of g * log2(e), a rounding of 1 + e and the
// approximate reciprocal), which rounds to the same bf16 as the exact silu
// unless it lies within 64 ulps of a rounding boundary; those elements, and
// |g| > 16, are recomputed exactly.  FP16 output always takes the exact path.
template <bool BF16>
__device__ __forceinline__ void swiglu_fwd8(const float g[8], const float u[8], float h[8]) {
    if constexpr (!BF16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = swiglu_fwd1<BF16>(g[i], u[i]);
    } else {
        uint32_t redo = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float s = __fdividef(g[i], 1.f + __expf(-g[i]));
            if (!(fabsf(g[i]) <= 16.f) || near_bf16_tie(s, 64)) redo |= 1u << i;
            h[i] = rnd<BF16>(s) * u[i];
        }
        if (redo) {  // rare; unrolled so the arrays stay in registers
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (redo & (1u << i)) h[i] = swiglu_fwd1<BF16>(g[i], u[i]);
        }
    }
}

// (dg, du) for one element from the 16-bit gate, up and dh values (as floats).
template <bool BF16>
__device__ __forceinline__ void swiglu_bwd1(float g, float u, float dh, float &dg, float &du) {
    const float s = sigmoid_f(g);
    du = dh * rnd<BF16>(g / (1.f + expf(-g)));
    const float dact = rnd<BF16>(dh * u);
    dg = dact * s * (1.f + g * (1.f - s));
}

}  // namespace h16
}  // namespace stratum
