// Fused elementwise kernels of the decoder layers around the NF4 GEMMs (B200).
//
// The reference runs HF Llama / Qwen3 decoder layers (stratum/model/llama.py,
// stratum/model/qwen3.py), whose RMSNorm, rotary embedding and SwiGLU are
// chains of separate torch kernels with fp32 round trips through HBM.  Each
// kernel here does one of them in a single pass, reproducing HF's arithmetic
// (the fp32 / bf16 roundings it performs between steps):
//   RMSNorm  (LlamaRMSNorm.forward): y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))
//   rotary   (apply_rotary_pos_emb): y = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)),
//            written head-major [H, S, D] (the attention kernel's layout), so the
//            transpose HF does with a strided copy is free
//   SwiGLU   (LlamaMLP): h = bf16(bf16(silu(g)) * u)
// and the matching backward passes.  All are HBM-bound: 16-byte vector
// accesses, one warp per row for the reductions, grids sized to the SM count.
#include "common.cuh"
#include "half8.cuh"

namespace stratum {
namespace fused {

using h16::ld1;
using h16::st1;
using h16::rnd;
using h16::unpack8;
using h16::pack8;
using h16::sigmoid_f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}

// ------------------------------------------------------------------ RMSNorm --

// One warp per row of `n` elements (n % 8 == 0); rstd[row] saved for the backward.
template <bool BF16>
__global__ void k_rmsnorm_fwd(const uint4 *__restrict__ x, const uint4 *__restrict__ w, int64_t rows, int vpr,
                              float eps, uint4 *__restrict__ y, float *__restrict__ rstd_out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
    const float inv_n = 1.f / float(vpr * 8);
    for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint4 *xr = x + r * vpr;
        float ss = 0.f;
        for (int c = lane; c < vpr; c += 32) {
            float f[8];
            unpack8<BF16>(xr[c], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) ss = fmaf(f[i], f[i], ss);
        }
        ss = warp_sum(ss);
        const float rs = rsqrtf(ss * inv_n + eps);
        if (lane == 0 && rstd_out) rstd_out[r] = rs;
        uint4 *yr = y + r * vpr;
        for (int c = lane; c < vpr; c += 32) {
            float f[8], g[8];
            unpack8<BF16>(xr[c], f);
            unpack8<BF16>(w[c], g);
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = g[i] * rnd<BF16>(f[i] * rs);
            yr[c] = pack8<BF16>(f);
        }
    }
}

// dx = rstd * (dy*w - xhat * mean(dy*w * xhat)), xhat = x * rstd (weight frozen: no dw).
template <bool BF16>
__global__ void k_rmsnorm_bwd(const uint4 *__restrict__ x, const uint4 *__restrict__ w, const uint4 *__restrict__ dy,
                              const float *__restrict__ rstd, int64_t rows, int vpr, uint4 *__restrict__ dx) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
    const float inv_n = 1.f / float(vpr * 8);
    for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint4 *xr = x + r * vpr, *dyr = dy + r * vpr;
        const float rs = rstd[r];
        float dot = 0.f;
        for (int c = lane; c < vpr; c += 32) {
            float f[8], g[8], d[8];
            unpack8<BF16>(xr[c], f);
            unpack8<BF16>(w[c], g);
            unpack8<BF16>(dyr[c], d);
#pragma unroll
            for (int i = 0; i < 8; ++i) dot = fmaf(d[i] * g[i], f[i] * rs, dot);
        }
        dot = warp_sum(dot) * inv_n;
        uint4 *dxr = dx + r * vpr;
        for (int c = lane; c < vpr; c += 32) {
            float f[8], g[8], d[8];
            unpack8<BF16>(xr[c], f);
            unpack8<BF16>(w[c], g);
            unpack8<BF16>(dyr[c], d);
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = rs * (d[i] * g[i] - f[i] * rs * dot);
            dxr[c] = pack8<BF16>(f);
        }
    }
}

// ------------------------------------------------------------------- rotary --

// x: [S, H, D] (row-major rows of H*D) -> y: [H, S, D], rotated when cos/sin are
// given (rotate_half pairs element i with i + D/2), copied otherwise.  One
// 16-byte vector per thread; D % 16 == 0.
template <bool BF16, bool ROT>
__global__ void k_rope_to_heads(const uint4 *__restrict__ x, const uint4 *__restrict__ cos_t,
                                const uint4 *__restrict__ sin_t, int S, int H, int D, uint4 *__restrict__ y) {
    const int vd = D / 8, half = vd / 2;
    const int64_t n = int64_t(S) * H * vd;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % vd);
        const int64_t sh = i / vd;
        const int h = int(sh % H), s = int(sh / H);
        const uint4 *xr = x + (int64_t(s) * H + h) * vd;
        uint4 out;
        if constexpr (ROT) {
            float a[8], b[8], cs[8], sn[8];
            unpack8<BF16>(xr[c], a);
            const int cp = c < half ? c + half : c - half;  // the partner half
            unpack8<BF16>(xr[cp], b);
            unpack8<BF16>(cos_t[int64_t(s) * vd + c], cs);
            unpack8<BF16>(sin_t[int64_t(s) * vd + c], sn);
            const float sgn = c < half ? -1.f : 1.f;  // rotate_half = cat(-x2, x1)
#pragma unroll
            for (int k = 0; k < 8; ++k) a[k] = rnd<BF16>(a[k] * cs[k]) + rnd<BF16>(sgn * b[k] * sn[k]);
            out = pack8<BF16>(a);
        } else {
            out = xr[c];
        }
        y[(int64_t(h) * S + s) * vd + c] = out;
    }
}

// Backward of k_rope_to_heads: dy [H, S, D] -> dx [S, H, D];
// dx = dy * cos + rotate_half^T(dy * sin), rotate_half^T(z) = cat(z2, -z1).
template <bool BF16, bool ROT>
__global__ void k_rope_from_heads(const uint4 *__restrict__ dy, const uint4 *__restrict__ cos_t,
                                  const uint4 *__restrict__ sin_t, int S, int H, int D, uint4 *__restrict__ dx) {
    const int vd = D / 8, half = vd / 2;
    const int64_t n = int64_t(S) * H * vd;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int c = int(i % vd);
        const int64_t sh = i / vd;
        const int h = int(sh % H), s = int(sh / H);
        const uint4 *dr = dy + (int64_t(h) * S + s) * vd;
        uint4 out;
        if constexpr (ROT) {
            float a[8], b[8], cs[8], sn[8];
            unpack8<BF16>(dr[c], a);
            const int cp = c < half ? c + half : c - half;
            unpack8<BF16>(dr[cp], b);
            unpack8<BF16>(cos_t[int64_t(s) * vd + c], cs);
            unpack8<BF16>(sin_t[int64_t(s) * vd + cp], sn);
            const float sgn = c < half ? 1.f : -1.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) a[k] = a[k] * cs[k] + sgn * b[k] * sn[k];
            out = pack8<BF16>(a);
        } else {
            out = dr[c];
        }
        dx[(int64_t(s) * H + h) * vd + c] = out;
    }
}

// ------------------------------------------------------------------- SwiGLU --

template <bool BF16>
__global__ void k_swiglu_fwd(const uint4 *__restrict__ g, const uint4 *__restrict__ u, int64_t n,
                             uint4 *__restrict__ h) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float a[8], b[8];
        unpack8<BF16>(g[i], a);
        unpack8<BF16>(u[i], b);
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = h16::swiglu_fwd1<BF16>(a[k], b[k]);
        h[i] = pack8<BF16>(a);
    }
}

// du = dh * silu(g)  (silu rounded as in the forward),  dg = (dh * u) * s * (1 + g * (1 - s))
template <bool BF16>
__global__ void k_swiglu_bwd(const uint4 *__restrict__ g, const uint4 *__restrict__ u, const uint4 *__restrict__ dh,
                             int64_t n, uint4 *__restrict__ dg, uint4 *__restrict__ du) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        float a[8], b[8], d[8], oa[8], ob[8];
        unpack8<BF16>(g[i], a);
        unpack8<BF16>(u[i], b);
        unpack8<BF16>(dh[i], d);
#pragma unroll
        for (int k = 0; k < 8; ++k) h16::swiglu_bwd1<BF16>(a[k], b[k], d[k], oa[k], ob[k]);
        dg[i] = pack8<BF16>(oa);
        du[i] = pack8<BF16>(ob);
    }
}

// The same backward for an MLP whose gate and up gradients feed one stacked
// input-gradient GEMM: rows of [dgate | dup] (width 2I) from gate, up, dh [rows, I].
template <bool BF16>
__global__ void k_swiglu_bwd_cat(const uint4 *__restrict__ g, const uint4 *__restrict__ u,
                                 const uint4 *__restrict__ dh, int64_t rows, int64_t iv, uint4 *__restrict__ dgu) {
    const int64_t n = rows * iv;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / iv, c = i - r * iv;
        float a[8], b[8], d[8], oa[8], ob[8];
        unpack8<BF16>(g[i], a);
        unpack8<BF16>(u[i], b);
        unpack8<BF16>(dh[i], d);
#pragma unroll
        for (int k = 0; k < 8; ++k) h16::swiglu_bwd1<BF16>(a[k], b[k], d[k], oa[k], ob[k]);
        dgu[r * 2 * iv + c] = pack8<BF16>(oa);
        dgu[r * 2 * iv + iv + c] = pack8<BF16>(ob);
    }
}

// ------------------------------------------------------------ cross entropy --

// Next-token cross entropy over bf16/fp16 logits, forward and gradient in one
// pass per row (the reference's chunked_linear_cross_entropy,
// stratum/model/chunked_loss.py, computes log_softmax in fp32 from the 16-bit
// logits and lets autograd form the gradient).  One block per row: an online
// max / sum-exp over the row, then the row is overwritten with
//     dlogits = (softmax - onehot(label)) * scale      (16-bit)
// and loss[row] = logsumexp - logit[label] (0 for ignored rows).
constexpr int kCeThreads = 512;

template <bool BF16>
__global__ void __launch_bounds__(kCeThreads)
k_ce_fwd_grad(uint4 *__restrict__ logits, const int64_t *__restrict__ labels, int64_t rows, int vpr,
              int64_t ignore_index, float scale, float *__restrict__ loss) {
    __shared__ float red_m[kCeThreads / 32], red_s[kCeThreads / 32];
    __shared__ float row_stats[2];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        uint4 *row = logits + r * vpr;
        const int64_t lab = labels[r];
        float m = -INFINITY, sum = 0.f;
        for (int c = threadIdx.x; c < vpr; c += kCeThreads) {
            float f[8];
            unpack8<BF16>(row[c], f);
            float lm = f[0];
#pragma unroll
            for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
            if (lm > m) {
                sum *= expf(m - lm);
                m = lm;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) sum += expf(f[i] - m);
        }
        // combine (m, sum) across the warp, then across warps
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const float om = __shfl_xor_sync(0xffffffffu, m, d), os = __shfl_xor_sync(0xffffffffu, sum, d);
            const float nm = fmaxf(m, om);
            sum = (m == -INFINITY ? 0.f : sum * expf(m - nm)) + (om == -INFINITY ? 0.f : os * expf(om - nm));
            m = nm;
        }
        if (lane == 0) {
            red_m[wid] = m;
            red_s[wid] = sum;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float M = red_m[0], Ssum = red_s[0];
            for (int w = 1; w < kCeThreads / 32; ++w) {
                if (red_m[w] == -INFINITY) continue;  // a warp that saw no element of the row
                const float nm = fmaxf(M, red_m[w]);
                Ssum = (M == -INFINITY ? 0.f : Ssum * expf(M - nm)) + red_s[w] * expf(red_m[w] - nm);
                M = nm;
            }
            row_stats[0] = M;
            row_stats[1] = logf(Ssum);
        }
        __syncthreads();
        const float M = row_stats[0], lse_off = row_stats[1];  // logsumexp = M + lse_off
        // labels outside [0, vocab) other than ignore_index are treated as ignored
        const bool live = lab != ignore_index && lab >= 0 && lab < int64_t(vpr) * 8;
        if (threadIdx.x == 0) {
            float l = 0.f;
            if (live) {
                const uint16_t *h = reinterpret_cast<const uint16_t *>(row);
                l = (M + lse_off) - ld1<BF16>(h[lab]);
            }
            loss[r] = l;
        }
        __syncthreads();  // the label's logit is read before the row is overwritten
        const float sc = live ? scale : 0.f;
        for (int c = threadIdx.x; c < vpr; c += kCeThreads) {
            float f[8];
            unpack8<BF16>(row[c], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float p = expf(f[i] - M - lse_off);
                if (int64_t(c) * 8 + i == lab) p -= 1.f;
                f[i] = p * sc;
            }
            row[c] = pack8<BF16>(f);
        }
        __syncthreads();  // row_stats reused by the next row
    }
}

inline int grid_for(int64_t work, int threads) {
    const int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = int64_t(sm_count()) * 8;
    return int(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

inline bool a16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace fused
}  // namespace stratum

using namespace stratum;
using namespace stratum::fused;

#define FUSED_DTYPE_CHECK(dt, what)                                                                    \
    if ((dt) != STRATUM_BF16 && (dt) != STRATUM_F16)                                                   \
        return fail(STRATUM_ERR_UNSUPPORTED, "%s: bf16 or fp16 only", what);

extern "C" {

int stratum_rmsnorm_fwd(const void *x, const void *weight, int dtype, int64_t rows, int64_t n, float eps, void *y,
                        float *rstd, void *stream) {
    STRATUM_REQUIRE(rows >= 0 && n > 0, "rmsnorm_fwd: bad sizes");
    if (rows == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "rmsnorm_fwd");
    STRATUM_REQUIRE(x && weight && y, "rmsnorm_fwd: null pointer");
    STRATUM_REQUIRE(n % 8 == 0 && a16(x) && a16(weight) && a16(y), "rmsnorm_fwd: n % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(rows * 32, 256);
    const int vpr = int(n / 8);
    if (dtype == STRATUM_BF16)
        k_rmsnorm_fwd<true><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(x), static_cast<const uint4 *>(weight), rows,
                                                  vpr, eps, static_cast<uint4 *>(y), rstd);
    else
        k_rmsnorm_fwd<false><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(x), static_cast<const uint4 *>(weight),
                                                   rows, vpr, eps, static_cast<uint4 *>(y), rstd);
    return check_launch("rmsnorm_fwd");
}

int stratum_rmsnorm_bwd(const void *x, const void *weight, const void *dy, const float *rstd, int dtype, int64_t rows,
                        int64_t n, void *dx, void *stream) {
    STRATUM_REQUIRE(rows >= 0 && n > 0, "rmsnorm_bwd: bad sizes");
    if (rows == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "rmsnorm_bwd");
    STRATUM_REQUIRE(x && weight && dy && rstd && dx, "rmsnorm_bwd: null pointer");
    STRATUM_REQUIRE(n % 8 == 0 && a16(x) && a16(weight) && a16(dy) && a16(dx),
                    "rmsnorm_bwd: n % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(rows * 32, 256);
    const int vpr = int(n / 8);
    if (dtype == STRATUM_BF16)
        k_rmsnorm_bwd<true><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(x), static_cast<const uint4 *>(weight),
                                                  static_cast<const uint4 *>(dy), rstd, rows, vpr,
                                                  static_cast<uint4 *>(dx));
    else
        k_rmsnorm_bwd<false><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(x), static_cast<const uint4 *>(weight),
                                                   static_cast<const uint4 *>(dy), rstd, rows, vpr,
                                                   static_cast<uint4 *>(dx));
    return check_launch("rmsnorm_bwd");
}

int stratum_rope_to_heads(const void *x, const void *cos_t, const void *sin_t, int dtype, int S, int H, int D, void *y,
                          void *stream) {
    STRATUM_REQUIRE(S >= 0 && H > 0 && D > 0, "rope_to_heads: bad sizes");
    if (S == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "rope_to_heads");
    STRATUM_REQUIRE(x && y && (cos_t == nullptr) == (sin_t == nullptr), "rope_to_heads: null pointer");
    STRATUM_REQUIRE(D % 16 == 0 && a16(x) && a16(y) && (!cos_t || (a16(cos_t) && a16(sin_t))),
                    "rope_to_heads: D % 16 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(int64_t(S) * H * (D / 8), 256);
    auto X = static_cast<const uint4 *>(x);
    auto C = static_cast<const uint4 *>(cos_t);
    auto Sn = static_cast<const uint4 *>(sin_t);
    auto Y = static_cast<uint4 *>(y);
    if (dtype == STRATUM_BF16) {
        if (cos_t) k_rope_to_heads<true, true><<<grid, 256, 0, st>>>(X, C, Sn, S, H, D, Y);
        else k_rope_to_heads<true, false><<<grid, 256, 0, st>>>(X, C, Sn, S, H, D, Y);
    } else {
        if (cos_t) k_rope_to_heads<false, true><<<grid, 256, 0, st>>>(X, C, Sn, S, H, D, Y);
        else k_rope_to_heads<false, false><<<grid, 256, 0, st>>>(X, C, Sn, S, H, D, Y);
    }
    return check_launch("rope_to_heads");
}

int stratum_rope_from_heads(const void *dy, const void *cos_t, const void *sin_t, int dtype, int S, int H, int D,
                            void *dx, void *stream) {
    STRATUM_REQUIRE(S >= 0 && H > 0 && D > 0, "rope_from_heads: bad sizes");
    if (S == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "rope_from_heads");
    STRATUM_REQUIRE(dy && dx && (cos_t == nullptr) == (sin_t == nullptr), "rope_from_heads: null pointer");
    STRATUM_REQUIRE(D % 16 == 0 && a16(dy) && a16(dx) && (!cos_t || (a16(cos_t) && a16(sin_t))),
                    "rope_from_heads: D % 16 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = grid_for(int64_t(S) * H * (D / 8), 256);
    auto Dy = static_cast<const uint4 *>(dy);
    auto C = static_cast<const uint4 *>(cos_t);
    auto Sn = static_cast<const uint4 *>(sin_t);
    auto Dx = static_cast<uint4 *>(dx);
    if (dtype == STRATUM_BF16) {
        if (cos_t) k_rope_from_heads<true, true><<<grid, 256, 0, st>>>(Dy, C, Sn, S, H, D, Dx);
        else k_rope_from_heads<true, false><<<grid, 256, 0, st>>>(Dy, C, Sn, S, H, D, Dx);
    } else {
        if (cos_t) k_rope_from_heads<false, true><<<grid, 256, 0, st>>>(Dy, C, Sn, S, H, D, Dx);
        else k_rope_from_heads<false, false><<<grid, 256, 0, st>>>(Dy, C, Sn, S, H, D, Dx);
    }
    return check_launch("rope_from_heads");
}

int stratum_swiglu_fwd(const void *gate, const void *up, int dtype, int64_t n, void *h, void *stream) {
    STRATUM_REQUIRE(n >= 0, "swiglu_fwd: bad size");
    if (n == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "swiglu_fwd");
    STRATUM_REQUIRE(gate && up && h, "swiglu_fwd: null pointer");
    STRATUM_REQUIRE(n % 8 == 0 && a16(gate) && a16(up) && a16(h), "swiglu_fwd: n % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t nv = n / 8;
    const int grid = grid_for(nv, 256);
    if (dtype == STRATUM_BF16)
        k_swiglu_fwd<true><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(gate), static_cast<const uint4 *>(up), nv,
                                                 static_cast<uint4 *>(h));
    else
        k_swiglu_fwd<false><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(gate), static_cast<const uint4 *>(up), nv,
                                                  static_cast<uint4 *>(h));
    return check_launch("swiglu_fwd");
}

int stratum_swiglu_bwd_cat(const void *gate, const void *up, const void *dh, int dtype, int64_t rows, int64_t I,
                           void *dgate_up, void *stream) {
    STRATUM_REQUIRE(rows >= 0 && I >= 0, "swiglu_bwd_cat: bad size");
    if (rows == 0 || I == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "swiglu_bwd_cat");
    STRATUM_REQUIRE(gate && up && dh && dgate_up, "swiglu_bwd_cat: null pointer");
    STRATUM_REQUIRE(I % 8 == 0 && a16(gate) && a16(up) && a16(dh) && a16(dgate_up),
                    "swiglu_bwd_cat: I % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t iv = I / 8;
    const int grid = grid_for(rows * iv, 256);
    auto G = static_cast<const uint4 *>(gate), U = static_cast<const uint4 *>(up), D = static_cast<const uint4 *>(dh);
    if (dtype == STRATUM_BF16)
        k_swiglu_bwd_cat<true><<<grid, 256, 0, st>>>(G, U, D, rows, iv, static_cast<uint4 *>(dgate_up));
    else
        k_swiglu_bwd_cat<false><<<grid, 256, 0, st>>>(G, U, D, rows, iv, static_cast<uint4 *>(dgate_up));
    return check_launch("swiglu_bwd_cat");
}

int stratum_swiglu_bwd(const void *gate, const void *up, const void *dh, int dtype, int64_t n, void *dgate, void *dup,
                       void *stream) {
    STRATUM_REQUIRE(n >= 0, "swiglu_bwd: bad size");
    if (n == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "swiglu_bwd");
    STRATUM_REQUIRE(gate && up && dh && dgate && dup, "swiglu_bwd: null pointer");
    STRATUM_REQUIRE(n % 8 == 0 && a16(gate) && a16(up) && a16(dh) && a16(dgate) && a16(dup),
                    "swiglu_bwd: n % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t nv = n / 8;
    const int grid = grid_for(nv, 256);
    if (dtype == STRATUM_BF16)
        k_swiglu_bwd<true><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(gate), static_cast<const uint4 *>(up),
                                                 static_cast<const uint4 *>(dh), nv, static_cast<uint4 *>(dgate),
                                                 static_cast<uint4 *>(dup));
    else
        k_swiglu_bwd<false><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(gate), static_cast<const uint4 *>(up),
                                                  static_cast<const uint4 *>(dh), nv, static_cast<uint4 *>(dgate),
                                                  static_cast<uint4 *>(dup));
    return check_launch("swiglu_bwd");
}

int stratum_ce_fwd_grad(void *logits, int dtype, const int64_t *labels, int64_t rows, int64_t vocab,
                        int64_t ignore_index, float scale, float *loss, void *stream) {
    STRATUM_REQUIRE(rows >= 0 && vocab > 0, "ce_fwd_grad: bad sizes");
    if (rows == 0) return STRATUM_OK;
    FUSED_DTYPE_CHECK(dtype, "ce_fwd_grad");
    STRATUM_REQUIRE(logits && labels && loss, "ce_fwd_grad: null pointer");
    STRATUM_REQUIRE(vocab % 8 == 0 && a16(logits), "ce_fwd_grad: vocab % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t cap = int64_t(sm_count()) * 4;
    const int grid = int(rows < cap ? rows : cap);
    if (dtype == STRATUM_BF16)
        k_ce_fwd_grad<true><<<grid, kCeThreads, 0, st>>>(static_cast<uint4 *>(logits), labels, rows, int(vocab / 8),
                                                         ignore_index, scale, loss);
    else
        k_ce_fwd_grad<false><<<grid, kCeThreads, 0, st>>>(static_cast<uint4 *>(logits), labels, rows, int(vocab / 8),
                                                          ignore_index, scale, loss);
    return check_launch("ce_fwd_grad");
}

}  // extern "C"
