// NF4 codec kernels for B200 (sm_100a): blockwise quantize (K1), double-quant
// of the absmax, and blockwise dequantize (K2).
//
// Both directions are HBM-bound byte work (2.5625 algorithmic bytes per
// element at blocksize 64), so the kernels are laid out for coalescing rather
// than arithmetic: every warp instruction touches whole 128-byte lines, the
// 16 levels / 15 thresholds sit in shared memory (16 distinct words in 16
// distinct banks: any lookup pattern is conflict-free), and grids are a
// multiple of the SM count with a grid-stride loop.
//
// Arithmetic follows bitsandbytes' blockwise NF4 codec (the reference calls it
// at stratum/upload.py:367-369 and :1038): q = #thresholds strictly below
// x * rcp_rn(absmax); dequant = round(fp32(level[q] * absmax)).  Every float
// op that the CPU restatement performs is written with an explicit _rn
// intrinsic so that the compiler cannot contract it into an FMA.
#include "common.cuh"
#include "nf4_decode.cuh"

#include <type_traits>

namespace stratum {

thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};

namespace {

constexpr int kThreads = 256;

// ------------------------------------------------------------ dequantize --

template <typename OutT> struct Out8;
template <> struct Out8<__half> {
    static __device__ __forceinline__ void store(__half *out, int64_t e0, const float v[8]) {
        __half2 h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
        *reinterpret_cast<uint4 *>(out + e0) = *reinterpret_cast<uint4 *>(h);
    }
    static __device__ __forceinline__ void store1(__half *out, int64_t e, float v) { out[e] = __float2half_rn(v); }
};
template <> struct Out8<__nv_bfloat16> {
    static __device__ __forceinline__ void store(__nv_bfloat16 *out, int64_t e0, const float v[8]) {
        __nv_bfloat162 h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
        *reinterpret_cast<uint4 *>(out + e0) = *reinterpret_cast<uint4 *>(h);
    }
    static __device__ __forceinline__ void store1(__nv_bfloat16 *out, int64_t e, float v) { out[e] = __float2bfloat16_rn(v); }
};
template <> struct Out8<float> {
    static __device__ __forceinline__ void store(float *out, int64_t e0, const float v[8]) {
        reinterpret_cast<float4 *>(out + e0)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4 *>(out + e0)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    static __device__ __forceinline__ void store1(float *out, int64_t e, float v) { out[e] = v; }
};

struct DequantArgs {
    const uint8_t *packed;
    const float *absmax;     // plain absmax (DQ == false)
    const uint8_t *absmax_q; // DQ == true
    const float *absmax2;
    const float *code2;
    const float *offset;
    int log2bs2;
    const float *code16;
    int64_t n;
    int log2bs;
};

template <bool DQ>
__device__ __forceinline__ float block_absmax(const DequantArgs &a, const float *c2, float offset, int64_t b) {
    if constexpr (DQ) {
        float s = __fmul_rn(c2[a.absmax_q[b]], __ldg(a.absmax2 + (b >> a.log2bs2)));
        return __fadd_rn(s, offset);
    } else {
        return __ldg(a.absmax + b);
    }
}

// Each warp owns 256 consecutive packed words (2048 elements) per step: lane l
// handles words base + l + 32*j, j = 0..7, so every 32-bit load covers one
// 128-byte line and every 16-byte fp16/bf16 store covers 512 contiguous bytes.
template <typename OutT, bool DQ>
__global__ void __launch_bounds__(kThreads) k_dequant(DequantArgs a, OutT *__restrict__ out) {
    __shared__ float lv[16];
    __shared__ float c2[DQ ? 256 : 1];
    if (threadIdx.x < 16) lv[threadIdx.x] = a.code16[threadIdx.x];
    if constexpr (DQ) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) c2[i] = a.code2[i];
    }
    const float offset = DQ ? *a.offset : 0.f;
    __syncthreads();

    const uint32_t *pw = reinterpret_cast<const uint32_t *>(a.packed);
    const int64_t nwords = a.n >> 3;  // words whose 8 elements are all valid
    const int lane = threadIdx.x & 31;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    const int64_t ntiles = (nwords + 255) >> 8;

    for (int64_t t = warp; t < ntiles; t += nwarps) {
        const int64_t base = t << 8;
        uint32_t p[8];
        float am[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t w = base + lane + 32 * j;
            p[j] = (w < nwords) ? __ldcs(pw + w) : 0u;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t w = base + lane + 32 * j;
            am[j] = (w < nwords) ? block_absmax<DQ>(a, c2, offset, (w << 3) >> a.log2bs) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t w = base + lane + 32 * j;
            if (w < nwords) {
                float v[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t byte = (p[j] >> (8 * k)) & 0xFFu;
                    v[2 * k] = __fmul_rn(lv[byte >> 4], am[j]);
                    v[2 * k + 1] = __fmul_rn(lv[byte & 0xFu], am[j]);
                }
                Out8<OutT>::store(out, w << 3, v);
            }
        }
    }
    // ragged tail: the last n % 8 elements
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        for (int64_t e = nwords << 3; e < a.n; ++e) {
            const uint8_t byte = a.packed[e >> 1];
            const uint32_t q = (e & 1) ? (byte & 0xFu) : (byte >> 4);
            Out8<OutT>::store1(out, e, __fmul_rn(lv[q], block_absmax<DQ>(a, c2, offset, e >> a.log2bs)));
        }
    }
}

// 16-bit outputs, blocksize >= 64: one thread per 64-element segment (32
// packed bytes, one absmax), decoded in registers with the scaled 16-entry
// table (nf4_decode.cuh).  Each warp owns 32 consecutive segments (4 KiB of
// output): lanes write their decoded 128-byte rows into shared memory with a
// 16-byte-chunk XOR swizzle (conflict-free), then the warp stores the 4 KiB as
// eight fully coalesced 512-byte rows.
template <bool BF16, bool DQ>
__global__ void __launch_bounds__(kThreads, 4) k_dequant_seg(DequantArgs a, uint4 *__restrict__ out) {
    __shared__ float lv_s[16];
    __shared__ float c2[DQ ? 256 : 1];
    __shared__ uint4 stage[kThreads / 32][32 * 8];  // per warp: 32 rows x 8 chunks of 16 B
    if (threadIdx.x < 16) lv_s[threadIdx.x] = a.code16[threadIdx.x];
    if constexpr (DQ) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) c2[i] = a.code2[i];
    }
    const float offset = DQ ? *a.offset : 0.f;
    __syncthreads();
    float lv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) lv[i] = lv_s[i];

    const int lane = threadIdx.x & 31;
    uint4 *buf = stage[threadIdx.x >> 5];
    const uint4 *pk = reinterpret_cast<const uint4 *>(a.packed);
    const int64_t nseg = a.n >> 6;
    const int64_t nwarp_tiles = (nseg + 31) >> 5;
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    for (int64_t wt = warp; wt < nwarp_tiles; wt += nwarps) {
        const int64_t g = (wt << 5) + lane;
        const bool valid = g < nseg;
        uint4 p0 = make_uint4(0, 0, 0, 0), p1 = p0;
        float am = 0.f;
        if (valid) {
            p0 = __ldcs(pk + 2 * g);
            p1 = __ldcs(pk + 2 * g + 1);
            am = block_absmax<DQ>(a, c2, offset, (g << 6) >> a.log2bs);
        }
        const Nf4Tables t = nf4_build_tables<BF16>(lv, am);
        const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t r[4];
            nf4_decode_word(t, w[i], r);
            buf[lane * 8 + (i ^ (lane & 7))] = make_uint4(r[0], r[1], r[2], r[3]);
        }
        __syncwarp();
        // chunk c of the warp's 4 KiB = chunk (c & 7) of row (c >> 3)
        const int64_t rows_valid = nseg - (wt << 5);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = k * 32 + lane;
            const int row = c >> 3;
            if (row < rows_valid) out[(wt << 8) + c] = buf[row * 8 + ((c & 7) ^ (row & 7))];
        }
        __syncwarp();
    }
    // ragged tail: the last n % 64 elements
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        using OutT = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        OutT *o = reinterpret_cast<OutT *>(out);
        for (int64_t e = nseg << 6; e < a.n; ++e) {
            const uint8_t byte = a.packed[e >> 1];
            const uint32_t q = (e & 1) ? (byte & 0xFu) : (byte >> 4);
            Out8<OutT>::store1(o, e, __fmul_rn(lv_s[q], block_absmax<DQ>(a, c2, offset, e >> a.log2bs)));
        }
    }
}

// Several tensors in one launch (one layer's weights, or any list): the same
// per-warp 4 KiB output tiles as k_dequant_seg, numbered across the tensors;
// a warp finds its tensor in the prefix table of tile counts.  Every tensor has
// n % 64 == 0 and 16-byte aligned packed / out; the double-quant tables are read
// per tensor through the read-only cache.
constexpr int kMaxMany = 32;

struct DequantMany {
    int count;
    int log2bs, log2bs2;
    const float *code16;
    int64_t tile0[kMaxMany + 1];  // first warp tile of each tensor; tile0[count] = total
    int64_t nseg[kMaxMany];       // 64-element segments of each tensor
    const uint8_t *packed[kMaxMany];
    const float *absmax[kMaxMany];
    const uint8_t *absmax_q[kMaxMany];
    const float *absmax2[kMaxMany];
    const float *code2[kMaxMany];
    const float *offset[kMaxMany];
    uint4 *out[kMaxMany];
};

template <bool BF16, bool DQ>
__global__ void __launch_bounds__(kThreads, 3) k_dequant_many(const __grid_constant__ DequantMany m) {
    __shared__ float lv_s[16];
    __shared__ uint4 stage[kThreads / 32][32 * 8];
    if (threadIdx.x < 16) lv_s[threadIdx.x] = m.code16[threadIdx.x];
    __syncthreads();
    float lv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) lv[i] = lv_s[i];
    const int lane = threadIdx.x & 31;
    uint4 *buf = stage[threadIdx.x >> 5];
    const int64_t total = m.tile0[m.count];
    const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
    // the tensor of warp tile gt: the last one whose first tile is <= gt
    auto tensor_of = [&](int64_t gt) {
        int lo = 0, hi = m.count - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (m.tile0[mid] <= gt) lo = mid;
            else hi = mid - 1;
        }
        return lo;
    };
    // loads of warp tile gt for this lane (zeros past the tensor's end); issued one tile
    // ahead, so each warp has the next tile's packed bytes in flight while it decodes
    auto load = [&](int64_t gt, uint4 &p0, uint4 &p1) {
        p0 = make_uint4(0, 0, 0, 0);
        p1 = p0;
        if (gt >= total) return;
        const int t = tensor_of(gt);
        const int64_t g = ((gt - m.tile0[t]) << 5) + lane;
        if (g < m.nseg[t]) {
            const uint4 *pk = reinterpret_cast<const uint4 *>(m.packed[t]);
            p0 = __ldcs(pk + 2 * g);
            p1 = __ldcs(pk + 2 * g + 1);
        }
    };
    uint4 n0, n1;
    load(warp, n0, n1);
    for (int64_t gt = warp; gt < total; gt += nwarps) {
        const int t = tensor_of(gt);
        const int64_t wt = gt - m.tile0[t];
        const int64_t nseg = m.nseg[t];
        const int64_t g = (wt << 5) + lane;
        const uint4 p0 = n0, p1 = n1;
        float am = 0.f;
        if (g < nseg) {
            const int64_t blk = (g << 6) >> m.log2bs;
            if constexpr (DQ) {
                am = __fadd_rn(__fmul_rn(__ldg(m.code2[t] + m.absmax_q[t][blk]),
                                         __ldg(m.absmax2[t] + (blk >> m.log2bs2))),
                               __ldg(m.offset[t]));
            } else {
                am = __ldg(m.absmax[t] + blk);
            }
        }
        load(gt + nwarps, n0, n1);
        const Nf4Tables tb = nf4_build_tables<BF16>(lv, am);
        const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            uint32_t r[4];
            nf4_decode_word(tb, w[i], r);
            buf[lane * 8 + (i ^ (lane & 7))] = make_uint4(r[0], r[1], r[2], r[3]);
        }
        __syncwarp();
        const int64_t rows_valid = nseg - (wt << 5);
        uint4 *out = m.out[t];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int c = k * 32 + lane;
            const int row = c >> 3;
            if (row < rows_valid) out[(wt << 8) + c] = buf[row * 8 + ((c & 7) ^ (row & 7))];
        }
        __syncwarp();
    }
}

// Fallback for buffers that are not 16-byte aligned: one element per thread.
template <typename OutT, bool DQ>
__global__ void __launch_bounds__(kThreads) k_dequant_unaligned(DequantArgs a, OutT *__restrict__ out) {
    __shared__ float lv[16];
    __shared__ float c2[DQ ? 256 : 1];
    if (threadIdx.x < 16) lv[threadIdx.x] = a.code16[threadIdx.x];
    if constexpr (DQ) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) c2[i] = a.code2[i];
    }
    const float offset = DQ ? *a.offset : 0.f;
    __syncthreads();
    for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < a.n; e += int64_t(gridDim.x) * blockDim.x) {
        const uint8_t byte = a.packed[e >> 1];
        const uint32_t q = (e & 1) ? (byte & 0xFu) : (byte >> 4);
        Out8<OutT>::store1(out, e, __fmul_rn(lv[q], block_absmax<DQ>(a, c2, offset, e >> a.log2bs)));
    }
}

template <bool DQ>
int launch_dequant(const DequantArgs &a, void *out, int out_dtype, cudaStream_t st) {
    const bool aligned = (reinterpret_cast<uintptr_t>(a.packed) % 4 == 0) &&
                         (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    const bool seg_path = (reinterpret_cast<uintptr_t>(a.packed) % 16 == 0) &&
                          (reinterpret_cast<uintptr_t>(out) % 16 == 0) && a.log2bs >= 6 &&
                          (out_dtype == STRATUM_F16 || out_dtype == STRATUM_BF16);
    if (seg_path) {
        const int64_t nseg = a.n >> 6;
        int64_t want = (nseg + kThreads - 1) / kThreads;
        if (out_dtype == STRATUM_BF16) {
            const int64_t cap = resident_grid<k_dequant_seg<true, DQ>>(kThreads);
            const int grid = int(want < 1 ? 1 : (want > cap ? cap : want));
            k_dequant_seg<true, DQ><<<grid, kThreads, 0, st>>>(a, reinterpret_cast<uint4 *>(out));
        } else {
            const int64_t cap = resident_grid<k_dequant_seg<false, DQ>>(kThreads);
            const int grid = int(want < 1 ? 1 : (want > cap ? cap : want));
            k_dequant_seg<false, DQ><<<grid, kThreads, 0, st>>>(a, reinterpret_cast<uint4 *>(out));
        }
        return check_launch(DQ ? "nf4_dequantize_dq" : "nf4_dequantize");
    }
    const int64_t nwords = a.n >> 3;
    const int64_t ntiles = (nwords + 255) >> 8;
    const int warps_per_cta = kThreads / 32;
    int64_t want = (ntiles + warps_per_cta - 1) / warps_per_cta;
    const int64_t cap = int64_t(sm_count()) * 8;  // 8 CTAs x 256 threads = full SM
    int grid = int(want < 1 ? 1 : (want > cap ? cap : want));
    if (!aligned) {
        int64_t g = (a.n + kThreads - 1) / kThreads;
        grid = int(g < 1 ? 1 : (g > cap ? cap : g));
    }
#define STRATUM_DQ_LAUNCH(T)                                                                   \
    do {                                                                                       \
        if (aligned) k_dequant<T, DQ><<<grid, kThreads, 0, st>>>(a, reinterpret_cast<T *>(out)); \
        else k_dequant_unaligned<T, DQ><<<grid, kThreads, 0, st>>>(a, reinterpret_cast<T *>(out)); \
    } while (0)
    switch (out_dtype) {
        case STRATUM_F16: STRATUM_DQ_LAUNCH(__half); break;
        case STRATUM_BF16: STRATUM_DQ_LAUNCH(__nv_bfloat16); break;
        case STRATUM_F32: STRATUM_DQ_LAUNCH(float); break;
        default: return fail(STRATUM_ERR_UNSUPPORTED, "dequantize: unsupported out_dtype %d", out_dtype);
    }
#undef STRATUM_DQ_LAUNCH
    return check_launch(DQ ? "nf4_dequantize_dq" : "nf4_dequantize");
}

// -------------------------------------------------------------- quantize --

template <typename InT> struct In8;
template <> struct In8<__half> {
    static __device__ __forceinline__ void load(const __half *src, int64_t e0, float v[8]) {
        uint4 r = __ldcs(reinterpret_cast<const uint4 *>(src + e0));
        const __half2 *h = reinterpret_cast<const __half2 *>(&r);
#pragma unroll
        for (int k = 0; k < 4; ++k) { float2 f = __half22float2(h[k]); v[2 * k] = f.x; v[2 * k + 1] = f.y; }
    }
};
template <> struct In8<__nv_bfloat16> {
    static __device__ __forceinline__ void load(const __nv_bfloat16 *src, int64_t e0, float v[8]) {
        uint4 r = __ldcs(reinterpret_cast<const uint4 *>(src + e0));
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&r);
#pragma unroll
        for (int k = 0; k < 4; ++k) { float2 f = __bfloat1622float2(h[k]); v[2 * k] = f.x; v[2 * k + 1] = f.y; }
    }
};
template <> struct In8<float> {
    static __device__ __forceinline__ void load(const float *src, int64_t e0, float v[8]) {
        float4 a = __ldcs(reinterpret_cast<const float4 *>(src + e0));
        float4 b = __ldcs(reinterpret_cast<const float4 *>(src + e0) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
};

__device__ __forceinline__ void load_thresholds(const float *thresholds, float *thr) {
    if (threadIdx.x < 16) thr[threadIdx.x] = threadIdx.x < 15 ? thresholds[threadIdx.x] : __int_as_float(0x7f800000);
}

// 16 consecutive elements (two packed words) per thread; the BS/16 lanes of a
// block reduce its absmax with xor-shuffles.  Only whole blocks here.
template <typename InT, int BS>
__global__ void __launch_bounds__(kThreads) k_quantize(const InT *__restrict__ src, int64_t nfull_words,
                                                        const float *__restrict__ thresholds,
                                                        uint32_t *__restrict__ packed, float *__restrict__ absmax) {
    constexpr int L = BS / 16;  // lanes per block
    __shared__ float thr[16];
    load_thresholds(thresholds, thr);
    __syncthreads();
    const float t7 = thr[7];
    const int64_t npairs = nfull_words >> 1;
    const int64_t stride = int64_t(gridDim.x) * blockDim.x;
    for (int64_t w = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; w - threadIdx.x % 32 < npairs; w += stride) {
        // whole warps iterate together (shuffles below); out-of-range lanes idle
        const bool valid = w < npairs;
        float v[16];
        if (valid) {
            In8<InT>::load(src, w << 4, v);
            In8<InT>::load(src, (w << 4) + 8, v + 8);
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = 0.f;
        }
        float am = 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k) am = fmaxf(am, fabsf(v[k]));
#pragma unroll
        for (int off = L / 2; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
        const float inv = __frcp_rn(am);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            uint32_t word = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t hi = nf4_code(__fmul_rn(v[8 * j + 2 * k], inv), thr, t7);
                const uint32_t lo = nf4_code(__fmul_rn(v[8 * j + 2 * k + 1], inv), thr, t7);
                word |= ((hi << 4) | lo) << (8 * k);
            }
            if (valid) __stcs(packed + 2 * w + j, word);
        }
        if (valid && (threadIdx.x % L) == 0) absmax[(w << 4) / BS] = am;
    }
}

// The ragged last block (n % blocksize != 0): one thread, elementwise.  Padding
// elements of an odd tail are quantized as 0.0 (like the bitsandbytes kernel).
template <typename InT>
__global__ void k_quantize_tail(const InT *__restrict__ src, int64_t start, int64_t n, const float *thresholds,
                                uint8_t *packed, float *absmax, int blocksize) {
    __shared__ float thr[16];
    load_thresholds(thresholds, thr);
    __syncthreads();
    if (threadIdx.x != 0) return;
    float am = 0.f;
    for (int64_t e = start; e < n; ++e) am = fmaxf(am, fabsf(load_as_f32(src, e)));
    absmax[start / blocksize] = am;
    const float inv = __frcp_rn(am);
    for (int64_t e = start; e < n; e += 2) {
        const uint32_t hi = nf4_code(__fmul_rn(load_as_f32(src, e), inv), thr, thr[7]);
        const float x1 = (e + 1 < n) ? load_as_f32(src, e + 1) : 0.f;
        const uint32_t lo = nf4_code(__fmul_rn(x1, inv), thr, thr[7]);
        packed[e >> 1] = uint8_t((hi << 4) | lo);
    }
}

template <typename InT, int BS>
int launch_quantize_bs(const InT *src, int64_t n, const float *thr, uint8_t *packed, float *absmax, cudaStream_t st) {
    const int64_t nfull_blocks = n / BS;
    const int64_t nfull_words = nfull_blocks * (BS / 8);
    if (nfull_words > 0) {
        const int64_t want = (nfull_words / 2 + kThreads - 1) / kThreads;
        const int64_t cap = int64_t(sm_count()) * 16;
        const int grid = int(want < 1 ? 1 : (want > cap ? cap : want));
        k_quantize<InT, BS><<<grid, kThreads, 0, st>>>(src, nfull_words, thr, reinterpret_cast<uint32_t *>(packed), absmax);
        int rc = check_launch("nf4_quantize");
        if (rc) return rc;
    }
    if (nfull_blocks * BS < n) {
        k_quantize_tail<InT><<<1, 32, 0, st>>>(src, nfull_blocks * BS, n, thr, packed, absmax, BS);
        return check_launch("nf4_quantize_tail");
    }
    return STRATUM_OK;
}

template <typename InT>
int launch_quantize(const InT *src, int64_t n, int bs, const float *thr, uint8_t *packed, float *absmax, cudaStream_t st) {
    switch (bs) {
        case 32: return launch_quantize_bs<InT, 32>(src, n, thr, packed, absmax, st);
        case 64: return launch_quantize_bs<InT, 64>(src, n, thr, packed, absmax, st);
        case 128: return launch_quantize_bs<InT, 128>(src, n, thr, packed, absmax, st);
        case 256: return launch_quantize_bs<InT, 256>(src, n, thr, packed, absmax, st);
        default: return fail(STRATUM_ERR_UNSUPPORTED, "quantize: blocksize %d not in {32,64,128,256}", bs);
    }
}

// ---------------------------------------------------------- double quant --

constexpr int kMeanChunk = 1024;

// partial[c] = sequential fp64 sum of absmax[c*1024 .. c*1024+1023]
__global__ void k_dq_partial(const float *__restrict__ absmax, int64_t nb, double *__restrict__ partial) {
    const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t c0 = c * kMeanChunk;
    if (c0 >= nb) return;
    const int64_t c1 = c0 + kMeanChunk < nb ? c0 + kMeanChunk : nb;
    double s = 0.0;
#pragma unroll 8
    for (int64_t i = c0; i < c1; ++i) s = __dadd_rn(s, double(__ldg(absmax + i)));
    partial[c] = s;
}

// offset = float(sequential fp64 sum of partials / nb); one thread does the
// chain, the block stages partials through shared memory.
__global__ void k_dq_total(const double *__restrict__ partial, int64_t nparts, int64_t nb, float *__restrict__ offset) {
    __shared__ double buf[1024];
    double total = 0.0;
    for (int64_t b0 = 0; b0 < nparts; b0 += 1024) {
        const int64_t cnt = nparts - b0 < 1024 ? nparts - b0 : 1024;
        __syncthreads();
        if (threadIdx.x < cnt) buf[threadIdx.x] = partial[b0 + threadIdx.x];
        __syncthreads();
        if (threadIdx.x == 0)
            for (int i = 0; i < cnt; ++i) total = __dadd_rn(total, buf[i]);
    }
    if (threadIdx.x == 0) *offset = float(__ddiv_rn(total, double(nb)));
}

// One warp per 256-entry block of absmax: absmax2 = max |absmax - offset|,
// absmax_q = #(255 midpoints) strictly below (absmax - offset) * rcp(absmax2).
__global__ void __launch_bounds__(kThreads) k_dq_quant(const float *__restrict__ absmax, int64_t nb,
                                                        const float *__restrict__ thresholds2,
                                                        const float *__restrict__ offset_p,
                                                        uint8_t *__restrict__ absmax_q, float *__restrict__ absmax2) {
    __shared__ float thr[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) thr[i] = i < 255 ? thresholds2[i] : __int_as_float(0x7f800000);
    __syncthreads();
    const float off = *offset_p;
    const int lane = threadIdx.x & 31;
    const int64_t nblk = (nb + 255) / 256;
    for (int64_t blk = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; blk < nblk;
         blk += (int64_t(gridDim.x) * blockDim.x) >> 5) {
        float c[8];
        float am = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int64_t i = blk * 256 + lane * 8 + k;
            c[k] = i < nb ? __fsub_rn(__ldg(absmax + i), off) : 0.f;
            am = fmaxf(am, fabsf(c[k]));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        const float inv = __frcp_rn(am);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int64_t i = blk * 256 + lane * 8 + k;
            const float x = __fmul_rn(c[k], inv);
            uint32_t q = 0;
#pragma unroll
            for (int step = 128; step > 0; step >>= 1) q += (x > thr[q + step - 1]) ? step : 0;
            if (i < nb) absmax_q[i] = uint8_t(q);
        }
        if (lane == 0) absmax2[blk] = am;
    }
}

}  // namespace
}  // namespace stratum

using namespace stratum;

extern "C" {

int stratum_abi_version(void) { return 1; }

const char *stratum_last_error(void) { return g_last_error; }

uint64_t stratum_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int stratum_set_device(int device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail(STRATUM_ERR_CUDA, "set_device(%d): %s", device, cudaGetErrorString(e));
    return STRATUM_OK;
}

int stratum_nf4_quantize(const void *src, int src_dtype, int64_t n, int blocksize, const float *thresholds,
                         uint8_t *packed, float *absmax, void *stream) {
    STRATUM_REQUIRE(n >= 0, "quantize: n < 0");
    if (n == 0) return STRATUM_OK;
    STRATUM_REQUIRE(src && thresholds && packed && absmax, "quantize: null pointer");
    const int esz = src_dtype == STRATUM_F32 ? 4 : 2;
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(src) % 16 == 0, "quantize: src must be 16-byte aligned");
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(packed) % 4 == 0, "quantize: packed must be 4-byte aligned");
    (void)esz;
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (src_dtype) {
        case STRATUM_F16: return launch_quantize(static_cast<const __half *>(src), n, blocksize, thresholds, packed, absmax, st);
        case STRATUM_BF16: return launch_quantize(static_cast<const __nv_bfloat16 *>(src), n, blocksize, thresholds, packed, absmax, st);
        case STRATUM_F32: return launch_quantize(static_cast<const float *>(src), n, blocksize, thresholds, packed, absmax, st);
        default: return fail(STRATUM_ERR_UNSUPPORTED, "quantize: unsupported src_dtype %d", src_dtype);
    }
}

size_t stratum_nf4_dq_workspace_bytes(int64_t nb) {
    const int64_t nparts = (nb + kMeanChunk - 1) / kMeanChunk;
    return size_t(nparts < 1 ? 1 : nparts) * sizeof(double);
}

int stratum_nf4_quantize_absmax_dq(const float *absmax, int64_t nb, int blocksize2, const float *thresholds2,
                                   uint8_t *absmax_q, float *absmax2, float *offset, void *workspace,
                                   size_t workspace_bytes, void *stream) {
    STRATUM_REQUIRE(nb > 0, "quantize_absmax_dq: nb must be > 0");
    STRATUM_REQUIRE(absmax && thresholds2 && absmax_q && absmax2 && offset && workspace, "quantize_absmax_dq: null pointer");
    if (blocksize2 != 256) return fail(STRATUM_ERR_UNSUPPORTED, "quantize_absmax_dq: blocksize2 %d != 256", blocksize2);
    STRATUM_REQUIRE(workspace_bytes >= stratum_nf4_dq_workspace_bytes(nb), "quantize_absmax_dq: workspace too small (%zu < %zu)",
                    workspace_bytes, stratum_nf4_dq_workspace_bytes(nb));
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 8 == 0, "quantize_absmax_dq: workspace must be 8-byte aligned");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    double *partial = static_cast<double *>(workspace);
    const int64_t nparts = (nb + kMeanChunk - 1) / kMeanChunk;
    k_dq_partial<<<int((nparts + 127) / 128), 128, 0, st>>>(absmax, nb, partial);
    int rc = check_launch("nf4_dq_partial");
    if (rc) return rc;
    k_dq_total<<<1, 1024, 0, st>>>(partial, nparts, nb, offset);
    rc = check_launch("nf4_dq_total");
    if (rc) return rc;
    const int64_t nblk = (nb + 255) / 256;
    const int64_t want = (nblk + (kThreads / 32) - 1) / (kThreads / 32);
    const int64_t cap = int64_t(sm_count()) * 8;
    k_dq_quant<<<int(want > cap ? cap : want), kThreads, 0, st>>>(absmax, nb, thresholds2, offset, absmax_q, absmax2);
    return check_launch("nf4_dq_quant");
}

// ------------------------------------------------------------------------
// Allocation-free double-quant quantizer.
//
// Some callers of this library cannot allocate device memory for a
// workspace: a host that binds the C ABI through an FFI and owns only the
// buffers it was handed (every tensor belongs to the caller's allocator,
// e.g. torch's caching allocator, and the library must not create device
// memory behind its back), or code running where an allocation is not
// allowed at that point.  NF4 quantization with double quantization needs
// two pieces of scratch -- the float32 absmax of every block and the
// chunk sums of the absmax mean -- so for those callers the scratch lives
// in one file-scope __device__ array of a fixed size instead.
//
// Limit: at most kNoAllocMaxBlocks NF4 blocks of 64 elements per call
// (64 Mi elements, e.g. a 14336 x 4096 weight).  The array costs 4 MiB +
// 8 KiB on every GPU that loads the library, held until the process exits.
constexpr int64_t kNoAllocMaxBlocks = int64_t(1) << 20;
constexpr size_t kNoAllocAbsmaxBytes = size_t(kNoAllocMaxBlocks) * sizeof(float);
constexpr size_t kNoAllocPartialBytes = size_t(kNoAllocMaxBlocks / kMeanChunk) * sizeof(double);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocAbsmaxBytes + kNoAllocPartialBytes];

// Device address of g_noalloc_scratch on the current device.  The name is
// only a host-side stand-in; the address comes from cudaGetSymbolAddress,
// looked up once per device (on that device's first call) and cached.  The
// cache entries are atomics: threads that race on a device's first call all
// store the same address.  The cache assumes the device's primary context
// lives as long as the process (a cudaDeviceReset would leave a stale entry).
static int noalloc_scratch(unsigned char **out) {
    static std::atomic<unsigned char *> ptrs[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64)
        return fail(STRATUM_ERR_CUDA, "quantize_dq_noalloc: no current device (%s)", cudaGetErrorString(e));
    unsigned char *cached = ptrs[dev].load(std::memory_order_acquire);
    if (cached == nullptr) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(STRATUM_ERR_CUDA, "quantize_dq_noalloc: cannot resolve the scratch array on device %d: %s", dev,
                        cudaGetErrorString(e));
        cached = static_cast<unsigned char *>(p);
        ptrs[dev].store(cached, std::memory_order_release);
    }
    *out = cached;
    return STRATUM_OK;
}

int stratum_nf4_quantize_dq_noalloc(const void *src, int src_dtype, int64_t n, const float *thresholds,
                                    const float *thresholds2, uint8_t *packed, uint8_t *absmax_q, float *absmax2,
                                    float *offset, void *stream) {
    STRATUM_REQUIRE(n >= 0, "quantize_dq_noalloc: n < 0");
    if (n == 0) return STRATUM_OK;  // as stratum_nf4_quantize: nothing to do, nothing written
    const int64_t nb = (n + 63) / 64;
    if (nb > kNoAllocMaxBlocks)
        return fail(STRATUM_ERR_INVALID,
                    "quantize_dq_noalloc: %lld elements need %lld NF4 blocks, above this entry point's fixed scratch "
                    "of %lld blocks (%lld elements); use stratum_nf4_quantize + stratum_nf4_quantize_absmax_dq with "
                    "a caller-provided workspace",
                    (long long)n, (long long)nb, (long long)kNoAllocMaxBlocks, (long long)(kNoAllocMaxBlocks * 64));
    STRATUM_BIND_STREAM(stream);
    unsigned char *scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    float *absmax = reinterpret_cast<float *>(scratch);
    double *partial = reinterpret_cast<double *>(scratch + kNoAllocAbsmaxBytes);
    // Both scratch regions are written in full before they are read (every
    // block's absmax, every chunk's sum), so nothing carries over between calls.
    rc = stratum_nf4_quantize(src, src_dtype, n, 64, thresholds, packed, absmax, stream);
    if (rc) return rc;
    return stratum_nf4_quantize_absmax_dq(absmax, nb, 256, thresholds2, absmax_q, absmax2, offset, partial,
                                          kNoAllocPartialBytes, stream);
}

int stratum_nf4_dequantize(const uint8_t *packed, const float *absmax, const float *code16, int64_t n, int blocksize,
                           void *out, int out_dtype, void *stream) {
    STRATUM_REQUIRE(n >= 0, "dequantize: n < 0");
    if (n == 0) return STRATUM_OK;
    STRATUM_REQUIRE(packed && absmax && code16 && out, "dequantize: null pointer");
    if (!is_pow2(blocksize) || blocksize < 32 || blocksize > 4096)
        return fail(STRATUM_ERR_UNSUPPORTED, "dequantize: blocksize %d not a power of two in [32, 4096]", blocksize);
    DequantArgs a{};
    a.packed = packed; a.absmax = absmax; a.code16 = code16; a.n = n; a.log2bs = ilog2(blocksize);
    STRATUM_BIND_STREAM(stream);
    return launch_dequant<false>(a, out, out_dtype, static_cast<cudaStream_t>(stream));
}

int stratum_nf4_dequantize_dq(const uint8_t *packed, const uint8_t *absmax_q, const float *absmax2, const float *code2,
                              const float *offset, int blocksize2, const float *code16, int64_t n, int blocksize,
                              void *out, int out_dtype, void *stream) {
    STRATUM_REQUIRE(n >= 0, "dequantize_dq: n < 0");
    if (n == 0) return STRATUM_OK;
    STRATUM_REQUIRE(packed && absmax_q && absmax2 && code2 && offset && code16 && out, "dequantize_dq: null pointer");
    if (!is_pow2(blocksize) || blocksize < 32 || blocksize > 4096)
        return fail(STRATUM_ERR_UNSUPPORTED, "dequantize_dq: blocksize %d not a power of two in [32, 4096]", blocksize);
    if (!is_pow2(blocksize2)) return fail(STRATUM_ERR_UNSUPPORTED, "dequantize_dq: blocksize2 %d not a power of two", blocksize2);
    DequantArgs a{};
    a.packed = packed; a.absmax_q = absmax_q; a.absmax2 = absmax2; a.code2 = code2; a.offset = offset;
    a.log2bs2 = ilog2(blocksize2); a.code16 = code16; a.n = n; a.log2bs = ilog2(blocksize);
    STRATUM_BIND_STREAM(stream);
    return launch_dequant<true>(a, out, out_dtype, static_cast<cudaStream_t>(stream));
}

int stratum_nf4_dequantize_many(const stratum_nf4_tensor *tensors, int count, const float *code16, int blocksize,
                                int blocksize2, int out_dtype, void *stream) {
    STRATUM_REQUIRE(count >= 0 && (count == 0 || tensors), "dequantize_many: bad tensor list");
    if (count == 0) return STRATUM_OK;
    STRATUM_REQUIRE(code16 != nullptr, "dequantize_many: null code16");
    if (!is_pow2(blocksize) || blocksize < 32 || blocksize > 4096)
        return fail(STRATUM_ERR_UNSUPPORTED, "dequantize_many: blocksize %d not a power of two in [32, 4096]", blocksize);
    for (int i = 0; i < count; ++i) {
        const stratum_nf4_tensor &t = tensors[i];
        STRATUM_REQUIRE(t.n >= 0, "dequantize_many: tensor %d: n < 0", i);
        if (t.n == 0) continue;
        STRATUM_REQUIRE(t.packed && t.out, "dequantize_many: tensor %d: null pointer", i);
        STRATUM_REQUIRE(t.absmax || (t.absmax_q && t.absmax2 && t.code2 && t.offset),
                        "dequantize_many: tensor %d: needs absmax or the double-quant set", i);
        if (!t.absmax && !is_pow2(blocksize2))
            return fail(STRATUM_ERR_UNSUPPORTED, "dequantize_many: blocksize2 %d not a power of two", blocksize2);
    }
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool wide = out_dtype == STRATUM_BF16 || out_dtype == STRATUM_F16;
    const int log2bs = ilog2(blocksize);
    // tensors the batched kernel takes; the rest go one by one through the single-tensor path
    DequantMany groups[2];
    for (auto &g : groups) {
        memset(&g, 0, sizeof(g));
        g.log2bs = log2bs;
        g.log2bs2 = ilog2(blocksize2 > 0 ? blocksize2 : 256);
        g.code16 = code16;
    }
    auto flush = [&](int dq) -> int {
        DequantMany &g = groups[dq];
        if (g.count == 0) return STRATUM_OK;
        const int64_t tiles = g.tile0[g.count];
        const int64_t want = (tiles + kThreads / 32 - 1) / (kThreads / 32);
        int64_t cap;
        if (out_dtype == STRATUM_BF16)
            cap = dq ? resident_grid<k_dequant_many<true, true>>(kThreads) : resident_grid<k_dequant_many<true, false>>(kThreads);
        else
            cap = dq ? resident_grid<k_dequant_many<false, true>>(kThreads) : resident_grid<k_dequant_many<false, false>>(kThreads);
        const int grid = int(want < 1 ? 1 : (want > cap ? cap : want));
        if (out_dtype == STRATUM_BF16) {
            if (dq) k_dequant_many<true, true><<<grid, kThreads, 0, st>>>(g);
            else k_dequant_many<true, false><<<grid, kThreads, 0, st>>>(g);
        } else {
            if (dq) k_dequant_many<false, true><<<grid, kThreads, 0, st>>>(g);
            else k_dequant_many<false, false><<<grid, kThreads, 0, st>>>(g);
        }
        const int rc = check_launch("nf4_dequantize_many");
        const int keep_log2bs2 = g.log2bs2;
        memset(&g, 0, sizeof(g));
        g.log2bs = log2bs;
        g.log2bs2 = keep_log2bs2;
        g.code16 = code16;
        return rc;
    };
    for (int i = 0; i < count; ++i) {
        const stratum_nf4_tensor &t = tensors[i];
        if (t.n == 0) continue;
        const bool dq = t.absmax == nullptr;
        const bool batchable = wide && t.n % 64 == 0 && log2bs >= 6 && reinterpret_cast<uintptr_t>(t.packed) % 16 == 0 &&
                               reinterpret_cast<uintptr_t>(t.out) % 16 == 0;
        int rc = STRATUM_OK;
        if (!batchable) {
            rc = dq ? stratum_nf4_dequantize_dq(t.packed, t.absmax_q, t.absmax2, t.code2, t.offset, blocksize2, code16,
                                                t.n, blocksize, t.out, out_dtype, stream)
                    : stratum_nf4_dequantize(t.packed, t.absmax, code16, t.n, blocksize, t.out, out_dtype, stream);
            if (rc) return rc;
            continue;
        }
        DequantMany &g = groups[dq];
        const int k = g.count;
        g.nseg[k] = t.n >> 6;
        g.tile0[k + 1] = g.tile0[k] + ((g.nseg[k] + 31) >> 5);
        g.packed[k] = t.packed;
        g.absmax[k] = t.absmax;
        g.absmax_q[k] = t.absmax_q;
        g.absmax2[k] = t.absmax2;
        g.code2[k] = t.code2;
        g.offset[k] = t.offset;
        g.out[k] = static_cast<uint4 *>(t.out);
        g.count = k + 1;
        if (g.count == kMaxMany && (rc = flush(dq))) return rc;
    }
    int rc = flush(0);
    if (rc) return rc;
    return flush(1);
}

}  // extern "C"
