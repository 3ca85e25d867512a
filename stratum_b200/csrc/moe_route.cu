// Token routing around the grouped NF4 expert GEMMs (B200, sm_100a).
//
// HF Qwen3MoeExperts.forward (transformers' modeling_qwen3_moe.py, the loop
// the reference runs with NF4-staged expert weights) walks the experts, gathers
// each expert's tokens with torch.where over a one-hot mask, runs the expert
// MLP, scales by the routing weight and index_adds the rows back.  Here the
// same work is laid out for one pass over HBM per step:
//   route      : stable counting sort of the T*k (token, slot) pairs by expert
//                -> order[p] (flat pair of sorted row p), inv[j] (sorted row of
//                pair j), token_of[p], offsets[E+1]
//   gather     : x_sorted[p] = x[token_of[p]]
//   combine    : out[t] = sum_k w[t,k] * rows[inv[t*k+k']]   (fp32 sum, fixed k order)
//   combine_grad (backward of combine for one weighted source):
//                dy_sorted[p] = w[order[p]] * dout[token_of[p]],
//                dw[order[p]] = <dout[token_of[p]], rows[p]>
//   swiglu_grad: d(gate|up) from dh and the saved gate|up (silu(g) * u).
// Every kernel is HBM-bound integer/elementwise work: 16-byte vector accesses,
// grids sized to the SM count, no tensor cores.
#include "common.cuh"

namespace stratum {
namespace route {

constexpr int kChunk = 1024;  // pairs per block in the count and scatter passes
constexpr int kMaxBuckets = 1024;  // experts + the dropped bucket (one scan thread each)

// Pass 1: per-block histogram of a contiguous chunk of pairs over E + 1
// buckets; bucket E collects dropped pairs (expert id outside [0, E), which
// includes HF's "expert_idx == num_experts" skip value).
__device__ __forceinline__ int bucket_of(int64_t e, int E) { return (e >= 0 && e < E) ? int(e) : E; }

__global__ void __launch_bounds__(kChunk)
k_route_count(const int64_t *__restrict__ experts, int64_t n, int E, int *__restrict__ blkcnt) {
    extern __shared__ int hist[];
    const int B = E + 1;
    for (int e = threadIdx.x; e < B; e += kChunk) hist[e] = 0;
    __syncthreads();
    const int64_t j = int64_t(blockIdx.x) * kChunk + threadIdx.x;
    if (j < n) atomicAdd(&hist[bucket_of(experts[j], E)], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < B; e += kChunk) blkcnt[int64_t(blockIdx.x) * B + e] = hist[e];
}

// Pass 2 (one block): exclusive scan of the bucket totals, giving offsets[0..E]
// (offsets[E] = pairs routed to a real expert); blkbase[b][e] = start of
// bucket e + its pairs in blocks before b.
__global__ void __launch_bounds__(kChunk)
k_route_scan(const int *__restrict__ blkcnt, int nblk, int E, int *__restrict__ blkbase, int *__restrict__ offsets) {
    __shared__ int wsum[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int e = threadIdx.x, B = E + 1;
    int total = 0;
    if (e < B)
        for (int b = 0; b < nblk; ++b) total += blkcnt[int64_t(b) * B + e];
    int v = total;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
    }
    if (lane == 31) wsum[wid] = v;
    __syncthreads();
    if (wid == 0) {
        int w = wsum[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, w, d);
            if (lane >= d) w += u;
        }
        wsum[lane] = w;
    }
    __syncthreads();
    const int excl = (wid ? wsum[wid - 1] : 0) + v - total;
    if (e < B) {
        if (e <= E) offsets[e] = excl;
        int run = excl;
        for (int b = 0; b < nblk; ++b) {
            blkbase[int64_t(b) * B + e] = run;
            run += blkcnt[int64_t(b) * B + e];
        }
    }
}

// Pass 3: stable scatter.  A pair's sorted row = its block's base for the
// bucket + same-bucket pairs in earlier warps of the block + earlier lanes of
// its warp (match_any groups the lanes by bucket).
__global__ void __launch_bounds__(kChunk)
k_route_scatter(const int64_t *__restrict__ experts, int64_t n, int E, int k, const int *__restrict__ blkbase,
                int *__restrict__ order, int *__restrict__ inv, int *__restrict__ token_of) {
    extern __shared__ int wcnt[];  // [32 warps][E + 1]
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, B = E + 1;
    for (int i = threadIdx.x; i < 32 * B; i += kChunk) wcnt[i] = 0;
    __syncthreads();
    const int64_t j = int64_t(blockIdx.x) * kChunk + threadIdx.x;
    const int e = j < n ? bucket_of(experts[j], E) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[wid * B + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
        int pos = blkbase[int64_t(blockIdx.x) * B + e] + rank;
        for (int w = 0; w < wid; ++w) pos += wcnt[w * B + e];
        order[pos] = int(j);
        inv[j] = pos;
        token_of[pos] = int(j / k);
    }
}

// x_sorted[p, :] = src[idx[p], :]; one warp per row, 16-byte vectors.
__global__ void k_gather_rows(const uint4 *__restrict__ src, const int *__restrict__ idx, int64_t rows, int vec_per_row,
                              uint4 *__restrict__ dst) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint4 *s = src + int64_t(ld_na(idx + r)) * vec_per_row;
        uint4 *d = dst + r * vec_per_row;
        for (int c = lane; c < vec_per_row; c += 32) st_na(d + c, ld_na(s + c));
    }
}

template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4 v, float f[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (BF16) {
            f[2 * i] = __uint_as_float(w[i] << 16);
            f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            const float2 h = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
            f[2 * i] = h.x;
            f[2 * i + 1] = h.y;
        }
    }
}

template <bool BF16>
__device__ __forceinline__ uint4 pack8(const float f[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (BF16) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&h);
        } else {
            const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&h);
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// out[t, :] = sum_{s<k} w[t*k+s] * rows[inv[t*k+s], :] over the pairs routed to a
// real expert (sorted row < offsets[E]); one warp per token.
template <bool BF16>
__global__ void k_combine(const uint4 *__restrict__ rows, const int *__restrict__ inv, const float *__restrict__ w,
                          const int *__restrict__ offsets, int E, int64_t T, int k, int vec_per_row,
                          uint4 *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int routed = ld_na(offsets + E);
    const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t t = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += warps) {
        for (int c = lane; c < vec_per_row; c += 32) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int s = 0; s < k; ++s) {
                const int64_t j = t * k + s;
                const int p = ld_na(inv + j);
                if (p >= routed) continue;
                const float ws = w ? ld_na(w + j) : 1.f;
                float f[8];
                unpack8<BF16>(ld_na(rows + int64_t(p) * vec_per_row + c), f);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(ws, f[i]));
            }
            st_na(out + t * vec_per_row + c, pack8<BF16>(acc));
        }
    }
}

// Backward of combine for sorted row p (pair j = order[p], token t = token_of[p]):
//   dy_sorted[p, :] = w[j] * dout[t, :];  dw[j] = <dout[t, :], rows[p, :]>  (fp32)
// Dropped pairs (p >= offsets[E]) get zero rows and a zero weight gradient.
// One warp per sorted row.
template <bool BF16>
__global__ void k_combine_grad(const uint4 *__restrict__ dout, const int *__restrict__ order,
                               const int *__restrict__ token_of, const float *__restrict__ w,
                               const int *__restrict__ offsets, int E, const uint4 *__restrict__ rows,
                               int64_t n_rows, int vec_per_row, uint4 *__restrict__ dy_sorted,
                               float *__restrict__ dw) {
    const int lane = threadIdx.x & 31;
    const int routed = ld_na(offsets + E);
    const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t p = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n_rows; p += warps) {
        const int j = ld_na(order + p);
        const int64_t t = ld_na(token_of + p);
        const bool live = p < routed;
        const float ws = live ? (w ? ld_na(w + j) : 1.f) : 0.f;
        float dot = 0.f;
        for (int c = lane; c < vec_per_row; c += 32) {
            float g[8], r[8], o[8];
            unpack8<BF16>(ld_na(dout + t * vec_per_row + c), g);
            if (rows && live) {
                unpack8<BF16>(ld_na(rows + p * vec_per_row + c), r);
#pragma unroll
                for (int i = 0; i < 8; ++i) dot = fmaf(g[i], r[i], dot);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = ws * g[i];
            st_na(dy_sorted + p * vec_per_row + c, pack8<BF16>(o));
        }
        if (dw) {
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, d);
            if (lane == 0) st_na(dw + j, dot);
        }
    }
}

// d(gate|up) for h = silu(g) * u:  dg = dh * u * s * (1 + g * (1 - s)),  du = dh * g * s,  s = sigmoid(g).
// gu and dgu are [rows, 2I] ([gate | up]); dh is [rows, I].
template <bool BF16>
__global__ void k_swiglu_grad(const uint4 *__restrict__ gu, const uint4 *__restrict__ dh, int64_t rows, int vec_i,
                              uint4 *__restrict__ dgu) {
    const int64_t n = rows * vec_i;
    for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < n; v += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = v / vec_i;
        const int c = int(v - r * vec_i);
        float g[8], u[8], d[8], dg[8], du[8];
        unpack8<BF16>(ld_na(gu + r * 2 * vec_i + c), g);
        unpack8<BF16>(ld_na(gu + r * 2 * vec_i + vec_i + c), u);
        unpack8<BF16>(ld_na(dh + v), d);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float s = 1.f / (1.f + __expf(-g[i]));
            du[i] = d[i] * g[i] * s;
            dg[i] = d[i] * u[i] * s * (1.f + g[i] * (1.f - s));
        }
        st_na(dgu + r * 2 * vec_i + c, pack8<BF16>(dg));
        st_na(dgu + r * 2 * vec_i + vec_i + c, pack8<BF16>(du));
    }
}

}  // namespace route
}  // namespace stratum

using namespace stratum;

namespace {
bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }
int warp_grid(int64_t rows) {
    const int64_t blocks = (rows + 7) / 8;  // 8 warps per block
    const int64_t cap = int64_t(sm_count()) * 8;
    return int(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}
}  // namespace

extern "C" {

size_t stratum_moe_route_workspace_bytes(int64_t n_pairs, int n_experts) {
    if (n_pairs < 0 || n_experts <= 0) return 0;
    const int64_t nblk = (n_pairs + route::kChunk - 1) / route::kChunk;
    return size_t(2 * nblk * (n_experts + 1)) * sizeof(int) + 256;
}

int stratum_moe_route(const int64_t *experts, int64_t T, int k, int E, int *order, int *inv, int *token_of,
                      int *offsets, void *workspace, size_t workspace_bytes, void *stream) {
    STRATUM_REQUIRE(T >= 0 && k > 0 && E > 0, "moe_route: bad sizes");
    if (E + 1 > route::kMaxBuckets)
        return fail(STRATUM_ERR_UNSUPPORTED, "moe_route: at most %d experts", route::kMaxBuckets - 1);
    const int64_t n = T * k;
    STRATUM_REQUIRE(n < (int64_t(1) << 31), "moe_route: T*k must fit in int32");
    STRATUM_REQUIRE(offsets != nullptr, "moe_route: null offsets");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n == 0) {
        if (cudaMemsetAsync(offsets, 0, sizeof(int) * (E + 1), st) != cudaSuccess)
            return fail(STRATUM_ERR_CUDA, "moe_route: memset failed");
        return STRATUM_OK;
    }
    STRATUM_REQUIRE(experts && order && inv && token_of && workspace, "moe_route: null pointer");
    const size_t need = stratum_moe_route_workspace_bytes(n, E);
    if (workspace_bytes < need)
        return fail(STRATUM_ERR_INVALID, "moe_route: workspace needs %zu bytes, got %zu", need, workspace_bytes);
    const int nblk = int((n + route::kChunk - 1) / route::kChunk);
    int *blkcnt = static_cast<int *>(workspace);
    int *blkbase = blkcnt + int64_t(nblk) * (E + 1);
    const int smem_cnt = (E + 1) * int(sizeof(int));
    const int smem_scatter = 32 * (E + 1) * int(sizeof(int));
    static bool attr_done[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(route::k_route_scatter, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 32 * route::kMaxBuckets * int(sizeof(int))) != cudaSuccess)
            return fail(STRATUM_ERR_CUDA, "moe_route: cannot set shared memory size");
        attr_done[dev] = true;
    }
    route::k_route_count<<<nblk, route::kChunk, smem_cnt, st>>>(experts, n, E, blkcnt);
    int rc = check_launch("moe_route_count");
    if (rc) return rc;
    route::k_route_scan<<<1, route::kChunk, 0, st>>>(blkcnt, nblk, E, blkbase, offsets);
    rc = check_launch("moe_route_scan");
    if (rc) return rc;
    route::k_route_scatter<<<nblk, route::kChunk, smem_scatter, st>>>(experts, n, E, k, blkbase, order, inv, token_of);
    return check_launch("moe_route_scatter");
}

int stratum_moe_gather_rows(const void *src, int64_t row_bytes, const int *idx, int64_t rows, void *dst, void *stream) {
    STRATUM_REQUIRE(rows >= 0 && row_bytes > 0, "moe_gather_rows: bad sizes");
    if (rows == 0) return STRATUM_OK;
    STRATUM_REQUIRE(src && idx && dst, "moe_gather_rows: null pointer");
    STRATUM_REQUIRE(row_bytes % 16 == 0 && aligned16(src) && aligned16(dst),
                    "moe_gather_rows: rows must be 16-byte multiples at 16-byte aligned addresses");
    STRATUM_BIND_STREAM(stream);
    route::k_gather_rows<<<warp_grid(rows), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4 *>(src), idx, rows, int(row_bytes / 16), static_cast<uint4 *>(dst));
    return check_launch("moe_gather_rows");
}

int stratum_moe_combine(const void *rows, int dtype, const int *inv, const float *weights, const int *offsets,
                        int E, int64_t T, int k, int64_t width, void *out, void *stream) {
    STRATUM_REQUIRE(T >= 0 && k > 0 && width > 0, "moe_combine: bad sizes");
    if (T == 0) return STRATUM_OK;
    STRATUM_REQUIRE(rows && inv && offsets && out && E > 0, "moe_combine: null pointer");
    if (dtype != STRATUM_BF16 && dtype != STRATUM_F16) return fail(STRATUM_ERR_UNSUPPORTED, "moe_combine: bf16 or fp16 rows");
    STRATUM_REQUIRE(width % 8 == 0 && aligned16(rows) && aligned16(out), "moe_combine: width % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int vpr = int(width / 8);
    if (dtype == STRATUM_BF16)
        route::k_combine<true><<<warp_grid(T), 256, 0, st>>>(static_cast<const uint4 *>(rows), inv, weights, offsets, E, T, k, vpr,
                                                             static_cast<uint4 *>(out));
    else
        route::k_combine<false><<<warp_grid(T), 256, 0, st>>>(static_cast<const uint4 *>(rows), inv, weights, offsets, E, T, k, vpr,
                                                              static_cast<uint4 *>(out));
    return check_launch("moe_combine");
}

int stratum_moe_combine_grad(const void *dout, int dtype, const int *order, const int *token_of, const float *weights,
                             const int *offsets, int E, const void *rows, int64_t n_rows, int64_t width,
                             void *dy_sorted, float *dweights, void *stream) {
    STRATUM_REQUIRE(n_rows >= 0 && width > 0, "moe_combine_grad: bad sizes");
    if (n_rows == 0) return STRATUM_OK;
    STRATUM_REQUIRE(dout && order && token_of && offsets && dy_sorted && E > 0, "moe_combine_grad: null pointer");
    STRATUM_REQUIRE(!dweights || rows, "moe_combine_grad: dweights needs the combined rows");
    if (dtype != STRATUM_BF16 && dtype != STRATUM_F16)
        return fail(STRATUM_ERR_UNSUPPORTED, "moe_combine_grad: bf16 or fp16 rows");
    STRATUM_REQUIRE(width % 8 == 0 && aligned16(dout) && aligned16(dy_sorted) && (!rows || aligned16(rows)),
                    "moe_combine_grad: width % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int vpr = int(width / 8);
    if (dtype == STRATUM_BF16)
        route::k_combine_grad<true><<<warp_grid(n_rows), 256, 0, st>>>(
            static_cast<const uint4 *>(dout), order, token_of, weights, offsets, E, static_cast<const uint4 *>(rows), n_rows, vpr,
            static_cast<uint4 *>(dy_sorted), dweights);
    else
        route::k_combine_grad<false><<<warp_grid(n_rows), 256, 0, st>>>(
            static_cast<const uint4 *>(dout), order, token_of, weights, offsets, E, static_cast<const uint4 *>(rows), n_rows, vpr,
            static_cast<uint4 *>(dy_sorted), dweights);
    return check_launch("moe_combine_grad");
}

int stratum_swiglu_grad(const void *gate_up, const void *dh, int dtype, int64_t rows, int64_t inter, void *dgate_up,
                        void *stream) {
    STRATUM_REQUIRE(rows >= 0 && inter > 0, "swiglu_grad: bad sizes");
    if (rows == 0) return STRATUM_OK;
    STRATUM_REQUIRE(gate_up && dh && dgate_up, "swiglu_grad: null pointer");
    if (dtype != STRATUM_BF16 && dtype != STRATUM_F16) return fail(STRATUM_ERR_UNSUPPORTED, "swiglu_grad: bf16 or fp16");
    STRATUM_REQUIRE(inter % 8 == 0 && aligned16(gate_up) && aligned16(dh) && aligned16(dgate_up),
                    "swiglu_grad: intermediate % 8 and 16-byte alignment");
    STRATUM_BIND_STREAM(stream);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int vi = int(inter / 8);
    const int grid = sm_count() * 8;
    if (dtype == STRATUM_BF16)
        route::k_swiglu_grad<true><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(gate_up),
                                                         static_cast<const uint4 *>(dh), rows, vi,
                                                         static_cast<uint4 *>(dgate_up));
    else
        route::k_swiglu_grad<false><<<grid, 256, 0, st>>>(static_cast<const uint4 *>(gate_up),
                                                          static_cast<const uint4 *>(dh), rows, vi,
                                                          static_cast<uint4 *>(dgate_up));
    return check_launch("swiglu_grad");
}

}  // extern "C"
