// Grouped NF4 GEMMs for routed MoE experts (B200, sm_100a).
//
// Replaces the per-expert loop of HF Qwen3MoeExperts.forward over NF4-staged
// 3-D weights (the reference stages them as [-1, last] 2-D payloads,
// stratum/upload.py:361-366; forward: transformers' Qwen3MoeExperts.forward):
//     gate, up = chunk(x_e . W_gu[e]^T, 2);  h = silu(gate) * up;
//     y_e = (h . W_d[e]^T) * routing_weight;  index_add back to token order.
// Tokens arrive sorted by expert with offsets[E+1].  A one-block kernel turns
// the offsets into a tile table {expert, weight-row tile, first token, end
// token}; the persistent GEMM kernels walk that table.  The mainloops are the
// single-GEMM ones (nf4_gemm.cu): the forward keeps the dequantized expert
// tile in TMEM as the A operand, the input-gradient kernel writes it MN-major
// into shared memory.  Token tiles may run into the next expert's tokens;
// those columns are computed and never stored (row-masked epilogues).
//
// Forward epilogues:
//   PLAIN  : y[t, n] (* rw[t] when given), stored row-masked through a
//            swizzled staging tile;
//   SWIGLU : a tile pairs 64 gate rows with the matching 64 up rows of W_gu, so
//            h[t, j] = silu(gate) * up is formed in the epilogue (from the 16-bit
//            gate and up, as HF's bf16 forward forms it) and only h -- half the
//            width of gate_up -- is written, plus gate|up when the backward needs it.
// An expert's tokens are split into equal token tiles (multiples of 16, at most
// 320 in the forward, 256 in the input gradient), and a tile's MMAs are only as
// wide as its tokens, so skewed routing costs tensor-core time in proportion to
// the tokens and no tile re-dequantizes a weight tile for a handful of them.
// The forward covers up to 320 tokens with two MMAs per K slice (N <= 256 into
// accumulator columns [0, 256), the rest into [256, 320)): at 4096 x top-8
// tokens over 128 experts (~256 per expert) every expert is one token tile.
#include "common.cuh"
#include "nf4_decode.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

namespace stratum {

namespace gemm {
int *status_ptr();  // the GEMM status word (nf4_gemm.cu), read by stratum_device_status
}

namespace grouped {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int DQG = 3;
constexpr int EPI_WARP0 = 4 + 4 * DQG;
constexpr int NUM_THREADS = (EPI_WARP0 + 4) * 32;
constexpr int X_BYTES = BN * BK * 2;

// ------------------------------------------------------------- tile table --

struct __align__(16) Tile {
    int e, m, t0, t_end;
};

// A CTA's tiles (first, first + stride, ...), read in increasing order by every
// warp role; each record is fetched one tile ahead, so a role's first use of a
// tile never waits on the table load (and the absmax address computed from it
// is ready one step later, as the dequant warps' prefetch expects).
struct TileCursor {
    const Tile *tiles;
    int first, stride, n, tl;
    Tile cur, next;
    __device__ __forceinline__ TileCursor(const Tile *t, int f, int s, int count)
        : tiles(t), first(f), stride(s), n(count), tl(-1), cur{0, 0, 0, 0}, next{0, 0, 0, 0} {
        if (count > 0) next = tiles[f];
    }
    __device__ __forceinline__ Tile at(int want) {
        if (want != tl) {
            cur = want == tl + 1 ? next : tiles[first + want * stride];
            tl = want;
            if (want + 1 < n) next = tiles[first + (want + 1) * stride];
        }
        return cur;
    }
};

// offsets[E+1] (device) -> tiles[]; order: expert, token tile, then weight-row
// tile innermost, so CTAs running at the same time share a token tile.  An
// expert's n tokens become ceil(n / cap) tiles of equal size rounded up to 16
// (the last one shorter).  One block: each thread counts one expert's tiles, a
// block scan places them.  Offsets that are not non-decreasing within
// [0, Ttot] set the status word and leave the table empty, so no kernel can
// store outside y.
constexpr int kTileThreads = 256;

__global__ void __launch_bounds__(kTileThreads)
k_build_tiles(const int *__restrict__ offsets, int E, int m_tiles, int cap, int64_t Ttot, Tile *__restrict__ tiles,
              int *__restrict__ ntiles, int max_tiles, int *__restrict__ status) {
    __shared__ int warp_sums[kTileThreads / 32];
    __shared__ int base_s;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x == 0) base_s = 0;
    int bad = 0;
    for (int e = threadIdx.x; e < E; e += kTileThreads) {
        const int a = ld_na(offsets + e), b = ld_na(offsets + e + 1);
        bad |= a < 0 || b < a || int64_t(b) > Ttot;
    }
    if (__syncthreads_or(bad)) {
        if (threadIdx.x == 0) {
            atomicCAS(status, 0, kErrBadOffsets);
            *ntiles = 0;
        }
        return;
    }
    for (int e0 = 0; e0 < E; e0 += kTileThreads) {
        const int e = e0 + threadIdx.x;
        int a = 0, b = 0, cnt = 0, sz = cap;
        if (e < E) {
            a = ld_na(offsets + e);
            b = ld_na(offsets + e + 1);
            if (b > a) {
                const int n = b - a, parts = (n + cap - 1) / cap;
                sz = ((n + parts - 1) / parts + 15) & ~15;  // <= cap (a multiple of 16)
                cnt = (n + sz - 1) / sz * m_tiles;
            }
        }
        int v = cnt;  // inclusive scan within the warp
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, v, d);
            if (lane >= d) v += u;
        }
        if (lane == 31) warp_sums[wid] = v;
        __syncthreads();
        if (wid == 0) {
            int w = lane < kTileThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
            for (int d = 1; d < kTileThreads / 32; d <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, w, d);
                if (lane >= d) w += u;
            }
            if (lane < kTileThreads / 32) warp_sums[lane] = w;
        }
        __syncthreads();
        const int start = base_s + (wid ? warp_sums[wid - 1] : 0) + v - cnt;
        int n = start;
        for (int t0 = a; t0 < b; t0 += sz)
            for (int m = 0; m < m_tiles; ++m, ++n)
                if (n < max_tiles)
                    st_na(reinterpret_cast<uint4 *>(tiles + n),
                          make_uint4(uint32_t(e), uint32_t(m), uint32_t(t0), uint32_t(t0 + sz < b ? t0 + sz : b)));
        __syncthreads();
        if (threadIdx.x == kTileThreads - 1) base_s = start + cnt;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        int n = base_s;
        if (n > max_tiles) {
            atomicCAS(status, 0, kErrTileTable);  // table too small: no tile is computed
            n = 0;
        }
        *ntiles = n;
    }
}

// Tokens of a tile (all of its expert; at most the table's cap), and the MMA
// width that covers them (a multiple of 16): a tile of a few tokens issues a
// narrow MMA instead of a full-width one.
__device__ __forceinline__ int tile_cols(const Tile &t) { return t.t_end - t.t0; }
__device__ __forceinline__ int tile_mma_n(const Tile &t) { return (tile_cols(t) + 15) & ~15; }

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
    for (int i = 0; i < 4; ++i) w[i] = BF16 ? pack_bf16x2(f[2 * i], f[2 * i + 1]) : pack_f16x2(f[2 * i], f[2 * i + 1]);
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// ------------------------------------------------------------- forward --

// Token tiles of up to F_TMAX tokens: accumulator columns [0, F_TMAX) (an N <= 256
// MMA into [0, 256) plus an N <= 64 one into [256, 320)), the dequantized A tiles
// from TMEM column F_TMAX on (32 columns per stage).  x arrives in 64-token boxes,
// only as many as the tile's MMA width needs.
constexpr int F_TMAX = 320;
constexpr int F_XBOX = 64;
constexpr int F_XBOX_BYTES = F_XBOX * BK * 2;
constexpr int F_X_BYTES = F_TMAX * BK * 2;
// stages: a token tile (40 KiB) and its dequantized weight tile (TMEM) share one
// full/empty barrier pair, so the MMA issuer waits and commits once per K step
constexpr int F_XS = 3, F_WS = 6, F_AS = F_XS;
constexpr int F_W_BYTES = BM * BK / 2;
constexpr int F_STAGE_BYTES = F_TMAX * BM * 2;  // [320 tokens][128 rows] 16-bit, 2 swizzled halves
constexpr int F_SMEM = 1024 + F_XS * F_X_BYTES + F_STAGE_BYTES + F_WS * F_W_BYTES + 512 + 1088;
static_assert(F_SMEM <= 232448, "smem");
static_assert(F_TMAX % F_XBOX == 0 && F_TMAX > BN && F_TMAX - BN <= BN && F_TMAX + 32 * F_AS <= 512,
              "forward tile shape");

struct FwdParams {
    const Tile *tiles;
    const int *ntiles;
    const float *absmax;
    const uint8_t *absmax_q;
    const float *absmax2;
    const float *code2;
    const float *offset;
    const float *code16;
    const float *rw;       // per sorted token routing weight (PLAIN, optional)
    uint16_t *y;           // PLAIN: [Ttot, N_e]; SWIGLU: [Ttot, N_e / 2]
    uint16_t *gu;          // SWIGLU, optional: gate and up [Ttot, N_e] for the backward
    int64_t Ttot;
    int N_e;               // weight rows per expert (2I for gate_up)
    int K;                 // contraction (H)
    int E, m_tiles, cap;   // bounds a tile record must respect (checked before any tile runs)
    int *status;
};

// Warp 3 (idle otherwise) checks this CTA's tile records before any role uses
// them: a record outside the bounds (a table overwritten after it was built, or
// built from bad offsets) would make an MMA that never completes.  On a bad
// record the status word gets kErrTileTable with the record beside it (block,
// tile index, e, m, t0, t_end) and the CTA runs no tile.  Returns through *bad
// (shared memory) after the caller's __syncthreads.
__device__ __forceinline__ void check_tiles(const Tile *tiles, int first, int stride, int n, int E, int m_tiles,
                                            int cap, int64_t Ttot, int *status, int *bad) {
    const int lane = threadIdx.x & 31;
    bool ok = true;
    for (int i = lane; i < n; i += 32) {
        const Tile t = tiles[first + i * stride];
        if (t.e < 0 || t.e >= E || t.m < 0 || t.m >= m_tiles || t.t0 < 0 || t.t_end <= t.t0 ||
            int64_t(t.t_end) > Ttot || t.t_end - t.t0 > cap) {
            ok = false;
            if (atomicCAS(status, 0, kErrTileTable) == 0) {
                volatile int *d = status;
                d[1] = first;
                d[2] = i;
                d[3] = t.e;
                d[4] = t.m;
                d[5] = t.t0;
                d[6] = t.t_end;
                __threadfence();
            }
        }
    }
    const bool all_ok = __all_sync(0xffffffffu, ok);
    if (lane == 0) *bad = all_ok ? 0 : 1;
}

template <bool BF16, bool DQ, bool SWIGLU>
__global__ void __launch_bounds__(NUM_THREADS, 1)
k_grouped_fwd(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w, const FwdParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *x0 = base;
    uint8_t *y0 = x0 + F_XS * F_X_BYTES;
    uint8_t *w0 = y0 + F_STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(w0 + F_WS * F_W_BYTES);
    // full[s]: stage s's token boxes landed (TMA bytes) and its weight tile is in TMEM
    // (128 dequant arrivals); empty[s]: the stage's MMAs completed (one commit)
    uint64_t *full = bars, *empty = full + F_XS, *wfull = empty + F_XS, *wempty = wfull + F_WS;
    uint64_t *accfull = wempty + F_WS, *accempty = accfull + 1;
    uint64_t *drain = accempty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    float *lv_s = reinterpret_cast<float *>(bars + 64);
    float *c2 = lv_s + 16;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.K / BK;
    const int ntiles = *p.ntiles;
    const int my_tiles0 = ntiles > int(blockIdx.x) ? (ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
    const int half_rows = p.N_e / 2;  // SWIGLU: I
    int *bad = reinterpret_cast<int *>(tmem_slot + 1);
    if (warp == 3) check_tiles(p.tiles, int(blockIdx.x), int(gridDim.x), my_tiles0, p.E, p.m_tiles, p.cap, p.Ttot,
                               p.status, bad);

    if (threadIdx.x == 0) {
        for (int i = 0; i < F_XS; ++i) { mbar_init(&full[i], 1 + 128); mbar_init(&empty[i], 1); }
        for (int i = 0; i < F_WS; ++i) { mbar_init(&wfull[i], 1); mbar_init(&wempty[i], 128); }
        mbar_init(accfull, 1);
        mbar_init(accempty, 128);
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 16) lv_s[threadIdx.x] = p.code16[threadIdx.x];
    if (DQ) for (int i = threadIdx.x; i < 256; i += NUM_THREADS) c2[i] = p.code2[i];
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int my_tiles = *bad ? 0 : my_tiles0;  // a bad tile record: run no tile (the status word says why)
    TileCursor cursor(p.tiles, int(blockIdx.x), int(gridDim.x), my_tiles);
    auto tile_at = [&](int tl) { return cursor.at(tl); };
    // first global weight row of the tile's rows r < 64 (and, in SWIGLU mode, r >= 64)
    auto row_lo = [&](const Tile &t) { return t.e * p.N_e + (SWIGLU ? t.m * 64 : t.m * BM); };
    auto row_hi = [&](const Tile &t) { return t.e * p.N_e + (SWIGLU ? half_rows + t.m * 64 : t.m * BM + 64); };

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tensormap(&tm_x);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const Tile t = tile_at(tl);
                const int nbox = (tile_mma_n(t) + F_XBOX - 1) / F_XBOX;  // 64-token boxes the MMAs read
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % F_XS;
                    if (!mbar_wait(&empty[s], ((it / F_XS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrGroupedFwdOffset)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], uint32_t(nbox * F_XBOX_BYTES));
                    for (int bx = 0; bx < nbox; ++bx)
                        tma_load_2d(x0 + s * F_X_BYTES + bx * F_XBOX_BYTES, &tm_x, ks * BK, t.t0 + bx * F_XBOX,
                                    &full[s]);
                }
            }
            for (uint32_t j = (it > F_XS ? it - F_XS : 0); j < it; ++j)
                mbar_wait_issued(&full[j % F_XS], (j / F_XS) & 1, p.status, kErrTimeoutTeardown + kErrGroupedFwdOffset);
            // the MMAs' last completion signals (commits into this CTA's shared memory)
            // land before the CTA exits: an arrival still in flight would hit the
            // shared memory of whichever CTA runs on this SM next
            if (ok)
                for (uint32_t j = (it > F_XS ? it - F_XS : 0); j < it; ++j)
                    mbar_wait(&empty[j % F_XS], (j / F_XS) & 1, p.status, kErrTimeoutTeardown + kErrGroupedFwdOffset);
        }
    } else if (warp == 2) {
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            uint32_t wt = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const Tile t = tile_at(tl);
                for (int ks = 0; ks < nk; ++ks, ++wt) {
                    const int s = wt % F_WS;
                    if (!mbar_wait(&wempty[s], ((wt / F_WS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrGroupedFwdOffset)) { ok = false; break; }
                    mbar_arrive_expect_tx(&wfull[s], F_W_BYTES);
                    // two 64-row boxes: rows [0, 64) and [64, 128) of the stage
                    tma_load_2d(w0 + s * F_W_BYTES, &tm_w, ks * (BK / 2), row_lo(t), &wfull[s]);
                    tma_load_2d(w0 + s * F_W_BYTES + 64 * 32, &tm_w, ks * (BK / 2), row_hi(t), &wfull[s]);
                }
            }
            for (uint32_t j = (wt > F_WS ? wt - F_WS : 0); j < wt; ++j)
                mbar_wait_issued(&wfull[j % F_WS], (j / F_WS) & 1, p.status, kErrTimeoutTeardown + kErrGroupedFwdOffset);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                // tokens [0, n0) into accumulator columns [0, n0), tokens [BN, BN + n1) into [BN, BN + n1)
                const int ntot = tile_mma_n(tile_at(tl));
                const int n0 = ntot < BN ? ntot : BN, n1 = ntot - n0;
                const uint32_t idesc0 = idesc_f16(BF16, BM, n0);
                const uint32_t idesc1 = n1 ? idesc_f16(BF16, BM, n1) : 0u;
                if (!mbar_wait(accempty, (tl & 1) ^ 1, p.status, kErrTimeoutMma + kErrGroupedFwdOffset)) { ok = false; break; }
                tc_fence_after();
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % F_XS, sa = s;
                    if (!mbar_wait(&full[s], (it / F_XS) & 1, p.status, kErrTimeoutMma + kErrGroupedFwdOffset)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bdesc0 = smem_desc_k_sw128(x0 + s * F_X_BYTES);
                    const uint64_t bdesc1 = smem_desc_k_sw128(x0 + s * F_X_BYTES + BN * BK * 2);
                    const uint32_t a0 = tmem + F_TMAX + sa * 32;
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j) {
                        mma_ts_f16(tmem, a0 + j * 8, bdesc0 + uint64_t(j * 2), idesc0, (ks | j) != 0);
                        if (n1) mma_ts_f16(tmem + BN, a0 + j * 8, bdesc1 + uint64_t(j * 2), idesc1, (ks | j) != 0);
                    }
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(accfull);
            }
            mma_commit(drain);
            mbar_wait_issued(drain, 0, p.status, kErrTimeoutTeardown + kErrGroupedFwdOffset);
        }
    } else if (warp >= 4 && warp < EPI_WARP0) {
        const int grp = (warp - 4) >> 2;
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        float lv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lv[i] = lv_s[i];
        const int64_t kb = p.K / BK;
        auto absmax_at = [&](int tl, int ks) -> float {
            if (tl >= my_tiles) return 0.f;
            const Tile t = tile_at(tl);
            const int64_t grow = row < 64 ? row_lo(t) + row : row_hi(t) + (row - 64);
            const int64_t b = grow * kb + ks;
            if constexpr (DQ) {
                return __fadd_rn(__fmul_rn(c2[__ldg(p.absmax_q + b)], __ldg(p.absmax2 + (b >> 8))), *p.offset);
            } else {
                return __ldg(p.absmax + b);
            }
        };
        const uint32_t total = uint32_t(my_tiles) * uint32_t(nk);
        // (tile, step) of the group's next owned step, advanced without division
        int ntl = 0, nks = grp;
        auto step = [&]() {
            while (nks >= nk) {
                nks -= nk;
                ++ntl;
            }
        };
        step();
        float am_next = absmax_at(ntl, nks);
        nks += DQG;
        step();
        for (uint32_t it = uint32_t(grp); it < total; it += DQG) {
            const float am = am_next;
            am_next = absmax_at(ntl, nks);  // one owned step ahead
            nks += DQG;
            step();
            const uint32_t wt = it;  // one weight tile per step (no LoRA chunks here)
            const int s = wt % F_WS;
            if (!__all_sync(0xffffffffu, mbar_wait(&wfull[s], (wt / F_WS) & 1, p.status, kErrTimeoutDequant + kErrGroupedFwdOffset))) break;
            const uint4 *src = reinterpret_cast<const uint4 *>(w0 + s * F_W_BYTES + row * 32);
            const int sw = (row >> 2) & 1;  // 32-byte swizzle
            const uint4 p0 = src[sw], p1 = src[sw ^ 1];
            const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            uint32_t vals[32];
            const Nf4Tables tb = nf4_build_tables<BF16>(lv, am);
            nf4_decode_block(tb, w, vals);
            fence_proxy_async_smem();  // generic reads before the stage's TMA refill
            mbar_arrive(&wempty[s]);
            const int sa = it % F_AS;
            if (!__all_sync(0xffffffffu, mbar_wait(&empty[sa], ((it / F_AS) & 1) ^ 1, p.status, kErrTimeoutDequant + kErrGroupedFwdOffset)))
                break;
            tc_fence_after();
            tmem_st_32x32b_x32(tmem + lane_addr + F_TMAX + sa * 32, vals);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&full[sa]);
        }
    } else if (warp >= EPI_WARP0) {  // warp 3 is idle: it must not join the epilogue's barriers
        // --------------------------------------------------------- epilogue
        const int q = warp & 3;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        const int etid = threadIdx.x - EPI_WARP0 * 32;  // 0..127
        for (int tl = 0; tl < my_tiles; ++tl) {
            if (!__all_sync(0xffffffffu, mbar_wait(accfull, tl & 1, p.status, kErrTimeoutEpilogue + kErrGroupedFwdOffset))) break;
            tc_fence_after();
            const Tile t = tile_at(tl);
            const int ncols = tile_cols(t);          // tokens of this expert in the tile
            const int nb = tile_mma_n(t) / 16;       // accumulator column blocks the MMA wrote
            // TMEM -> registers as 16x256b fragments (row = weight row, pairs of tokens)
            // -> 16-bit -> stmatrix.trans into the [token][row] staging tile (two
            // 128B-swizzled halves of 64 rows); the accumulator is released as soon as
            // it has been read, so the next tile's MMAs overlap the rest of the epilogue.
            named_bar_sync(1, 128);  // previous tile's readers are done with the staging tile
            const int kq = lane >> 3, jr = lane & 7;
            const int tok_in = jr + 8 * (kq >> 1);
            const int nrow = q * 32 + 8 * (kq & 1);
            auto stage_block = [&](int cb, const uint32_t (&v)[2][8]) {
                float s0 = 1.f, s1 = 1.f, s2 = 1.f, s3 = 1.f;  // routing weights of this thread's 4 tokens
                if (!SWIGLU && p.rw) {
                    const int tk = cb * 16 + 2 * (lane & 3);
                    s0 = tk < ncols ? p.rw[t.t0 + tk] : 0.f;
                    s1 = tk + 1 < ncols ? p.rw[t.t0 + tk + 1] : 0.f;
                    s2 = tk + 8 < ncols ? p.rw[t.t0 + tk + 8] : 0.f;
                    s3 = tk + 9 < ncols ? p.rw[t.t0 + tk + 9] : 0.f;
                }
                const int tok = cb * 16 + tok_in;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t x4[4];
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const float sa = (m < 2) ? s0 : s2, sb = (m < 2) ? s1 : s3;
                        const float lo = __uint_as_float(v[h][2 * m]) * sa;
                        const float hi = __uint_as_float(v[h][2 * m + 1]) * sb;
                        x4[m] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                    }
                    const int nr = nrow + 16 * h;
                    const int half = nr >> 6, chunk = (nr & 63) >> 3;
                    const uint8_t *dst = y0 + half * (F_STAGE_BYTES / 2) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
                    stmatrix_x4_trans(smem_u32(dst), x4[0], x4[1], x4[2], x4[3]);
                }
            };
            // two 16-token column blocks per TMEM load wait: half the round trips on
            // the path that holds the accumulator
#pragma unroll 1
            for (int cb = 0; cb < nb; cb += 2) {
                const bool pair = cb + 1 < nb;  // warp-uniform
                uint32_t v0[2][8], v1[2][8];
                tmem_ld_16x256b_x2(tmem + lane_addr + cb * 16, v0[0]);
                tmem_ld_16x256b_x2(tmem + lane_addr + (16u << 16) + cb * 16, v0[1]);
                if (pair) {
                    tmem_ld_16x256b_x2(tmem + lane_addr + (cb + 1) * 16, v1[0]);
                    tmem_ld_16x256b_x2(tmem + lane_addr + (16u << 16) + (cb + 1) * 16, v1[1]);
                }
                tmem_ld_wait();
                if (cb + 2 >= nb) {
                    tc_fence_before();
                    mbar_arrive(accempty);
                }
                stage_block(cb, v0);
                if (pair) stage_block(cb + 1, v1);
            }
            named_bar_sync(1, 128);
            if constexpr (SWIGLU) {
                // staging half 0 holds the tile's 64 gate rows, half 1 the matching 64 up
                // rows: h = silu(gate) * up from the 16-bit gate and up (the values HF's
                // bf16 forward multiplies), 8 columns per 16-byte chunk
                const int I = half_rows;
                for (int idx = etid; idx < ncols * 8; idx += 128) {
                    const int tok = idx >> 3, chunk = idx & 7;
                    const int off = tok * 128 + ((chunk ^ (tok & 7)) << 4);
                    const uint4 gv = *reinterpret_cast<const uint4 *>(y0 + off);
                    const uint4 uv = *reinterpret_cast<const uint4 *>(y0 + F_STAGE_BYTES / 2 + off);
                    float g[8], u[8], h[8];
                    unpack8<BF16>(gv, g);
                    unpack8<BF16>(uv, u);
#pragma unroll
                    for (int i = 0; i < 8; ++i) h[i] = g[i] / (1.f + __expf(-g[i])) * u[i];
                    const int64_t trow = t.t0 + tok;
                    *reinterpret_cast<uint4 *>(p.y + trow * I + t.m * 64 + chunk * 8) = pack8<BF16>(h);
                    if (p.gu) {  // gate and up themselves, in gate_up's [gate | up] column order
                        uint16_t *gr = p.gu + trow * (2 * I) + t.m * 64 + chunk * 8;
                        *reinterpret_cast<uint4 *>(gr) = gv;
                        *reinterpret_cast<uint4 *>(gr + I) = uv;
                    }
                }
            } else {
                // row-masked 16-byte copies to y (only this expert's tokens are stored):
                // 16 chunks of 16 B per token, 8 threads per 128-byte half row
                for (int idx = etid; idx < ncols * 16; idx += 128) {
                    const int tok = idx >> 4, hc = idx & 15, half = hc >> 3, chunk = hc & 7;
                    const uint4 val = *reinterpret_cast<const uint4 *>(y0 + half * (F_STAGE_BYTES / 2) + tok * 128 +
                                                                       ((chunk ^ (tok & 7)) << 4));
                    *reinterpret_cast<uint4 *>(p.y + int64_t(t.t0 + tok) * p.N_e + t.m * BM + half * 64 + chunk * 8) =
                        val;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// -------------------------------------------------------- input gradient --

constexpr int D_XS = 3, D_WS = 4, D_AS = D_XS;  // stages: dY tile + W^T tile, one barrier pair
constexpr int D_W_BYTES = BK * BM / 2;
constexpr int D_A_BYTES = BM * BK * 2;
constexpr int D_A_ATOM = BK * 128;
constexpr int D_STAGE_BYTES = BN * BM * 2;
constexpr int D_SMEM = 1024 + D_XS * X_BYTES + D_AS * D_A_BYTES + D_STAGE_BYTES + D_WS * D_W_BYTES + 512 + 1088;
static_assert(D_SMEM <= 232448, "smem");

struct DxParams {
    const Tile *tiles;
    const int *ntiles;
    const float *absmax;
    const uint8_t *absmax_q;
    const float *absmax2;
    const float *code2;
    const float *offset;
    const float *code16;
    uint16_t *dx;     // [Ttot, K]
    int N_e;          // contraction: weight rows per expert
    int K;            // weight columns (output width)
    int64_t Ttot;
    int E, m_tiles, cap;  // bounds a tile record must respect (checked before any tile runs)
    int *status;
};

template <bool BF16, bool DQ>
__global__ void __launch_bounds__(NUM_THREADS, 1)
k_grouped_dx(const __grid_constant__ CUtensorMap tm_dy, const __grid_constant__ CUtensorMap tm_w, const DxParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *x0 = base;
    uint8_t *a0 = x0 + D_XS * X_BYTES;
    uint8_t *y0 = a0 + D_AS * D_A_BYTES;
    uint8_t *w0 = y0 + D_STAGE_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(w0 + D_WS * D_W_BYTES);
    // full[s]: stage s's dY tile landed and its W^T tile is in shared memory (TMA bytes +
    // 128 dequant arrivals); empty[s]: the stage's MMAs completed (one commit)
    uint64_t *full = bars, *empty = full + D_XS, *wfull = empty + D_XS, *wempty = wfull + D_WS;
    uint64_t *accfull = wempty + D_WS, *accempty = accfull + 2;
    uint64_t *drain = accempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    // progress words beside the barriers (snapshotted by a timeout record): [0] dY steps
    // issued, [1] W steps issued, [2] steps the MMA consumed, [3..5] each decode
    // group's step + 1, [6] the epilogue's tile | its tile count << 16, [7] ntiles as read
    volatile int *prog = reinterpret_cast<volatile int *>(tmem_slot + 2);
    float *lv_s = reinterpret_cast<float *>(bars + 64);
    float *c2 = lv_s + 16;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = p.N_e / BK;
    const int ntiles = *p.ntiles;
    const int my_tiles0 = ntiles > int(blockIdx.x) ? (ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
    int *bad = reinterpret_cast<int *>(tmem_slot + 1);
    if (warp == 3) check_tiles(p.tiles, int(blockIdx.x), int(gridDim.x), my_tiles0, p.E, p.m_tiles, p.cap, p.Ttot,
                               p.status, bad);

    if (threadIdx.x == 0) {
        for (int i = 0; i < D_XS; ++i) { mbar_init(&full[i], 1 + 128); mbar_init(&empty[i], 1); }
        for (int i = 0; i < D_WS; ++i) { mbar_init(&wfull[i], 1); mbar_init(&wempty[i], 128); }
        for (int i = 0; i < 2; ++i) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], 128); }
        mbar_init(drain, 1);
        fence_barrier_init();
        for (int i = 0; i < 7; ++i) prog[i] = 0;
        prog[7] = ntiles;
    }
    if (threadIdx.x < 16) lv_s[threadIdx.x] = p.code16[threadIdx.x];
    if (DQ) for (int i = threadIdx.x; i < 256; i += NUM_THREADS) c2[i] = p.code2[i];
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int my_tiles = *bad ? 0 : my_tiles0;  // a bad tile record: run no tile (the status word says why)
    TileCursor cursor(p.tiles, int(blockIdx.x), int(gridDim.x), my_tiles);
    auto tile_at = [&](int tl) { return cursor.at(tl); };

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tensormap(&tm_dy);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const Tile t = tile_at(tl);
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % D_XS;
                    if (!mbar_wait(&empty[s], ((it / D_XS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrGroupedDxOffset)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], X_BYTES);
                    tma_load_2d(x0 + s * X_BYTES, &tm_dy, ks * BK, t.t0, &full[s]);
                    prog[0] = int(it) + 1;
                }
            }
            for (uint32_t j = (it > D_XS ? it - D_XS : 0); j < it; ++j)
                mbar_wait_issued(&full[j % D_XS], (j / D_XS) & 1, p.status, kErrTimeoutTeardown + kErrGroupedDxOffset);
            // the MMAs' last completion signals (commits into this CTA's shared memory)
            // land before the CTA exits: an arrival still in flight would hit the
            // shared memory of whichever CTA runs on this SM next
            if (ok)
                for (uint32_t j = (it > D_XS ? it - D_XS : 0); j < it; ++j)
                    mbar_wait(&empty[j % D_XS], (j / D_XS) & 1, p.status, kErrTimeoutTeardown + kErrGroupedDxOffset);
        }
    } else if (warp == 2) {
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            uint32_t wt = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const Tile t = tile_at(tl);
                for (int ks = 0; ks < nk; ++ks, ++wt) {
                    const int s = wt % D_WS;
                    if (!mbar_wait(&wempty[s], ((wt / D_WS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrGroupedDxOffset)) { ok = false; break; }
                    mbar_arrive_expect_tx(&wfull[s], D_W_BYTES);
                    tma_load_2d(w0 + s * D_W_BYTES, &tm_w, t.m * (BM / 2), t.e * p.N_e + ks * BK, &wfull[s]);
                    prog[1] = int(wt) + 1;
                }
            }
            for (uint32_t j = (wt > D_WS ? wt - D_WS : 0); j < wt; ++j)
                mbar_wait_issued(&wfull[j % D_WS], (j / D_WS) & 1, p.status, kErrTimeoutTeardown + kErrGroupedDxOffset);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const uint32_t idesc = idesc_f16_amn(BF16, BM, tile_mma_n(tile_at(tl)));
                const int ab = tl & 1;
                if (!mbar_wait(&accempty[ab], ((tl >> 1) & 1) ^ 1, p.status, kErrTimeoutMma + kErrGroupedDxOffset)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + uint32_t(ab * 256);
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % D_XS, sa = s;
                    if (!mbar_wait(&full[s], (it / D_XS) & 1, p.status, kErrTimeoutMma + kErrGroupedDxOffset)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_k_sw128(x0 + s * X_BYTES);
                    const uint64_t adesc = smem_desc_mn_sw128(a0 + sa * D_A_BYTES, D_A_ATOM, 1024);
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j)
                        mma_ss_f16(acc, adesc + uint64_t(j * (2048 >> 4)), bdesc + uint64_t(j * 2), idesc, (ks | j) != 0);
                    mma_commit(&empty[s]);
                    prog[2] = int(it) + 1;
                }
                if (ok) mma_commit(&accfull[ab]);
            }
            mma_commit(drain);
            mbar_wait_issued(drain, 0, p.status, kErrTimeoutTeardown + kErrGroupedDxOffset);
        }
    } else if (warp >= 4 && warp < EPI_WARP0) {
        const int grp = (warp - 4) >> 2;
        const int tid = (warp & 3) * 32 + lane;
        const int rl = tid & 63, kb = tid >> 6;
        float lv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lv[i] = lv_s[i];
        const int64_t kbl = p.K / 64;
        auto absmax_at = [&](int tl, int ks) -> float {
            if (tl >= my_tiles) return 0.f;
            const Tile t = tile_at(tl);
            const int64_t kblk = int64_t(t.m) * 2 + kb;
            if (kblk >= kbl) return 0.f;
            const int64_t b = (int64_t(t.e) * p.N_e + int64_t(ks) * BK + rl) * kbl + kblk;
            if constexpr (DQ) {
                return __fadd_rn(__fmul_rn(c2[__ldg(p.absmax_q + b)], __ldg(p.absmax2 + (b >> 8))), *p.offset);
            } else {
                return __ldg(p.absmax + b);
            }
        };
        const uint32_t total = uint32_t(my_tiles) * uint32_t(nk);
        // (tile, step) of the group's next owned step, advanced without division
        int ntl = 0, nks = grp;
        auto step = [&]() {
            while (nks >= nk) {
                nks -= nk;
                ++ntl;
            }
        };
        step();
        float am_next = absmax_at(ntl, nks);
        nks += DQG;
        step();
        for (uint32_t it = uint32_t(grp); it < total; it += DQG) {
            const float am = am_next;
            am_next = absmax_at(ntl, nks);  // one owned step ahead
            nks += DQG;
            step();
            const int s = it % D_WS;
            if (tid == 0) prog[3 + grp] = int(it) + 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&wfull[s], (it / D_WS) & 1, p.status, kErrTimeoutDequant + kErrGroupedDxOffset))) break;
            const uint4 *src = reinterpret_cast<const uint4 *>(w0 + s * D_W_BYTES + rl * 64);
            const int sw = (rl >> 1) & 3;  // 64-byte swizzle
            const uint4 p0 = src[(2 * kb) ^ sw], p1 = src[(2 * kb + 1) ^ sw];
            const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
            uint32_t vals[32];
            const Nf4Tables tb = nf4_build_tables<BF16>(lv, am);
            nf4_decode_block(tb, w, vals);
            fence_proxy_async_smem();
            mbar_arrive(&wempty[s]);
            const int sa = it % D_AS;
            if (!__all_sync(0xffffffffu, mbar_wait(&empty[sa], ((it / D_AS) & 1) ^ 1, p.status, kErrTimeoutDequant + kErrGroupedDxOffset)))
                break;
            uint8_t *dst = a0 + sa * D_A_BYTES + kb * D_A_ATOM + (rl >> 3) * 1024 + (rl & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4 *>(dst + ((c ^ (rl & 7)) << 4)) =
                    make_uint4(vals[4 * c], vals[4 * c + 1], vals[4 * c + 2], vals[4 * c + 3]);
            fence_proxy_async_smem();
            mbar_arrive(&full[sa]);
        }
    } else if (warp >= EPI_WARP0) {  // warp 3 is idle
        const int q = warp & 3;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        const int etid = threadIdx.x - EPI_WARP0 * 32;
        const int kq = lane >> 3, jr = lane & 7;
        const int tok_in = jr + 8 * (kq >> 1);
        const int nrow = q * 32 + 8 * (kq & 1);
        for (int tl = 0; tl < my_tiles; ++tl) {
            const int ab = tl & 1;
            if (etid == 0) prog[6] = tl | (my_tiles << 16);
            if (!__all_sync(0xffffffffu, mbar_wait(&accfull[ab], (tl >> 1) & 1, p.status, kErrTimeoutEpilogue + kErrGroupedDxOffset))) break;
            tc_fence_after();
            const Tile t = tile_at(tl);
            const int ncols = tile_cols(t);
            const int nb = tile_mma_n(t) / 16;  // accumulator column blocks the MMA wrote
            const uint32_t acc = tmem + lane_addr + uint32_t(ab * 256);
            named_bar_sync(1, 128);
#pragma unroll 1
            for (int cb = 0; cb < nb; ++cb) {
                uint32_t v[2][8];
                tmem_ld_16x256b_x2(acc + cb * 16, v[0]);
                tmem_ld_16x256b_x2(acc + (16u << 16) + cb * 16, v[1]);
                tmem_ld_wait();
                if (cb == nb - 1) {
                    tc_fence_before();
                    mbar_arrive(&accempty[ab]);
                }
                const int tok = cb * 16 + tok_in;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t x4[4];
#pragma unroll
                    for (int m = 0; m < 4; ++m) {
                        const float lo = __uint_as_float(v[h][2 * m]), hi = __uint_as_float(v[h][2 * m + 1]);
                        x4[m] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                    }
                    const int nr = nrow + 16 * h;
                    const int half = nr >> 6, chunk = (nr & 63) >> 3;
                    const uint8_t *dst = y0 + half * (D_STAGE_BYTES / 2) + tok * 128 + ((chunk ^ (tok & 7)) << 4);
                    stmatrix_x4_trans(smem_u32(dst), x4[0], x4[1], x4[2], x4[3]);
                }
            }
            named_bar_sync(1, 128);
            const int k0 = t.m * BM;
            for (int idx = etid; idx < ncols * 16; idx += 128) {
                const int tok = idx >> 4, hc = idx & 15, half = hc >> 3, chunk = hc & 7;
                const int col = k0 + half * 64 + chunk * 8;
                if (col < p.K) {
                    const uint4 val = *reinterpret_cast<const uint4 *>(y0 + half * (D_STAGE_BYTES / 2) + tok * 128 +
                                                                       ((chunk ^ (tok & 7)) << 4));
                    *reinterpret_cast<uint4 *>(p.dx + int64_t(t.t0 + tok) * p.K + col) = val;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------ host --

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

int make_map(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw, const char *what) {
    auto enc = encode_fn();
    if (!enc) return fail(STRATUM_ERR_CUDA, "%s: cuTensorMapEncodeTiled unavailable", what);
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(STRATUM_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, int(r));
    return STRATUM_OK;
}

template <typename K>
int set_smem(K kern, int bytes, bool *done, const char *what) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !done[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
            return fail(STRATUM_ERR_CUDA, "%s: cannot set %d bytes of shared memory", what, bytes);
        done[dev] = true;
    }
    return STRATUM_OK;
}

template <bool BF16, bool DQ, bool SWIGLU>
int launch_fwd(const CUtensorMap &mx, const CUtensorMap &mw, const FwdParams &p, int grid, cudaStream_t st) {
    static bool done[64] = {false};
    auto kern = k_grouped_fwd<BF16, DQ, SWIGLU>;
    int rc = set_smem(kern, F_SMEM, done, "nf4_grouped_fwd");
    if (rc) return rc;
    kern<<<grid, NUM_THREADS, F_SMEM, st>>>(mx, mw, p);
    return check_launch("nf4_grouped_fwd");
}

template <bool BF16, bool DQ>
int launch_dx(const CUtensorMap &mdy, const CUtensorMap &mw, const DxParams &p, int grid, cudaStream_t st) {
    static bool done[64] = {false};
    auto kern = k_grouped_dx<BF16, DQ>;
    int rc = set_smem(kern, D_SMEM, done, "nf4_grouped_dx");
    if (rc) return rc;
    kern<<<grid, NUM_THREADS, D_SMEM, st>>>(mdy, mw, p);
    return check_launch("nf4_grouped_dx");
}

}  // namespace grouped
}  // namespace stratum

using namespace stratum;

extern "C" {

static size_t table_bytes_for(int64_t total_tokens, int n_experts, int m_tiles) {
    const int64_t max_tiles = int64_t(m_tiles) * ((total_tokens + grouped::BN - 1) / grouped::BN + n_experts);
    return size_t(max_tiles) * sizeof(grouped::Tile) + 256;
}

size_t stratum_nf4_grouped_table_bytes(int64_t total_tokens, int n_experts, int64_t weight_dim) {
    if (total_tokens < 0 || n_experts <= 0 || weight_dim <= 0) return 0;
    return table_bytes_for(total_tokens, n_experts, int((weight_dim + grouped::BM - 1) / grouped::BM));
}

// Shared argument checks and tile-table build for the two grouped kernels.
// `cap`: most tokens in a token tile (a multiple of 16, at least 256, so the
// table size of stratum_nf4_grouped_table_bytes bounds the tile count).
static int build_table(const int *offsets, int E, int m_tiles, int cap, int64_t Ttot, void *table,
                       size_t table_bytes, int *status, cudaStream_t st, grouped::Tile **tiles, int **ntiles,
                       int *grid) {
    const size_t need = table_bytes_for(Ttot, E, m_tiles);
    if (table_bytes < need) return fail(STRATUM_ERR_INVALID, "grouped: tile table needs %zu bytes, got %zu", need, table_bytes);
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(table) % 16 == 0, "grouped: tile table must be 16-byte aligned");
    *ntiles = static_cast<int *>(table);
    *tiles = reinterpret_cast<grouped::Tile *>(static_cast<uint8_t *>(table) + 256);
    const int max_tiles = int((table_bytes - 256) / sizeof(grouped::Tile));
    grouped::k_build_tiles<<<1, grouped::kTileThreads, 0, st>>>(offsets, E, m_tiles, cap, Ttot, *tiles, *ntiles,
                                                                 max_tiles, status);
    int rc = check_launch("nf4_grouped_tiles");
    if (rc) return rc;
    *grid = sm_count();
    return STRATUM_OK;
}

int stratum_nf4_grouped_fwd(const void *x_sorted, int dtype, int64_t Ttot, int K, const int *offsets, int E,
                            const uint8_t *packed, const float *absmax, const uint8_t *absmax_q, const float *absmax2,
                            const float *code2, const float *offset, const float *code16, int N_e, int swiglu,
                            const float *rw, void *y, void *gate_up, void *table, size_t table_bytes,
                            void *stream) {
    STRATUM_REQUIRE(Ttot >= 0 && Ttot < (int64_t(1) << 31) && K > 0 && E > 0 && N_e > 0, "nf4_grouped_fwd: bad sizes");
    if (Ttot == 0) return STRATUM_OK;
    STRATUM_REQUIRE(x_sorted && offsets && packed && code16 && y && table, "nf4_grouped_fwd: null pointer");
    if (dtype != STRATUM_BF16 && dtype != STRATUM_F16) return fail(STRATUM_ERR_UNSUPPORTED, "nf4_grouped_fwd: x must be bf16 or fp16");
    if (K % 64) return fail(STRATUM_ERR_UNSUPPORTED, "nf4_grouped_fwd: K=%d must be a multiple of 64", K);
    if (N_e % 128) return fail(STRATUM_ERR_UNSUPPORTED, "nf4_grouped_fwd: N_e=%d must be a multiple of 128", N_e);
    STRATUM_REQUIRE(!swiglu || rw == nullptr, "nf4_grouped_fwd: the routing weight applies to the plain epilogue");
    STRATUM_REQUIRE(swiglu || gate_up == nullptr, "nf4_grouped_fwd: gate_up is written by the swiglu epilogue only");
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(gate_up) % 4 == 0, "nf4_grouped_fwd: gate_up must be 4-byte aligned");
    const bool dq = absmax == nullptr;
    STRATUM_REQUIRE(!dq || (absmax_q && absmax2 && code2 && offset), "nf4_grouped_fwd: need absmax or the double-quant set");
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(x_sorted) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 16 == 0 &&
                        reinterpret_cast<uintptr_t>(y) % 16 == 0,
                    "nf4_grouped_fwd: x, packed and y must be 16-byte aligned");
    STRATUM_BIND_STREAM(stream);
    int *status = gemm::status_ptr();
    if (!status) return fail(STRATUM_ERR_CUDA, "nf4_grouped_fwd: no status word");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // plain: 128 weight rows per tile; swiglu: 64 gate rows + the matching 64 up rows
    const int m_tiles = N_e / 128;
    grouped::Tile *tiles;
    int *ntiles, grid;
    int rc = build_table(offsets, E, m_tiles, grouped::F_TMAX, Ttot, table, table_bytes, status, st, &tiles, &ntiles,
                         &grid);
    if (rc) return rc;
    const CUtensorMapDataType xdt = dtype == STRATUM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap mx, mw;
    rc = grouped::make_map(&mx, xdt, x_sorted, uint64_t(K), uint64_t(Ttot), uint64_t(K) * 2, 64, grouped::F_XBOX,
                           CU_TENSOR_MAP_SWIZZLE_128B, "nf4_grouped_fwd x");
    if (rc) return rc;
    rc = grouped::make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, uint64_t(K / 2), uint64_t(E) * uint64_t(N_e),
                           uint64_t(K / 2), 32, 64, CU_TENSOR_MAP_SWIZZLE_32B, "nf4_grouped_fwd packed");
    if (rc) return rc;
    grouped::FwdParams p{};
    p.E = E; p.m_tiles = m_tiles; p.cap = grouped::F_TMAX;
    p.tiles = tiles; p.ntiles = ntiles; p.absmax = absmax; p.absmax_q = absmax_q; p.absmax2 = absmax2;
    p.code2 = code2; p.offset = offset; p.code16 = code16; p.rw = rw; p.y = static_cast<uint16_t *>(y);
    p.gu = static_cast<uint16_t *>(gate_up);
    p.Ttot = Ttot; p.N_e = N_e; p.K = K; p.status = status;
    const bool bf = dtype == STRATUM_BF16;
#define G_LAUNCH(B, D, S) return grouped::launch_fwd<B, D, S>(mx, mw, p, grid, st)
    if (bf) { if (dq) { if (swiglu) G_LAUNCH(true, true, true); else G_LAUNCH(true, true, false); }
              else { if (swiglu) G_LAUNCH(true, false, true); else G_LAUNCH(true, false, false); } }
    else { if (dq) { if (swiglu) G_LAUNCH(false, true, true); else G_LAUNCH(false, true, false); }
           else { if (swiglu) G_LAUNCH(false, false, true); else G_LAUNCH(false, false, false); } }
#undef G_LAUNCH
}

int stratum_nf4_grouped_dx(const void *dy_sorted, int dtype, int64_t Ttot, int N_e, const int *offsets, int E,
                           const uint8_t *packed, const float *absmax, const uint8_t *absmax_q, const float *absmax2,
                           const float *code2, const float *offset, const float *code16, int K, void *dx, void *table,
                           size_t table_bytes, void *stream) {
    STRATUM_REQUIRE(Ttot >= 0 && Ttot < (int64_t(1) << 31) && K > 0 && E > 0 && N_e > 0, "nf4_grouped_dx: bad sizes");
    if (Ttot == 0) return STRATUM_OK;
    STRATUM_REQUIRE(dy_sorted && offsets && packed && code16 && dx && table, "nf4_grouped_dx: null pointer");
    if (dtype != STRATUM_BF16 && dtype != STRATUM_F16) return fail(STRATUM_ERR_UNSUPPORTED, "nf4_grouped_dx: dy must be bf16 or fp16");
    if (K % 64) return fail(STRATUM_ERR_UNSUPPORTED, "nf4_grouped_dx: K=%d must be a multiple of 64", K);
    if (N_e % 64) return fail(STRATUM_ERR_UNSUPPORTED, "nf4_grouped_dx: N_e=%d must be a multiple of 64", N_e);
    const bool dq = absmax == nullptr;
    STRATUM_REQUIRE(!dq || (absmax_q && absmax2 && code2 && offset), "nf4_grouped_dx: need absmax or the double-quant set");
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(dy_sorted) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 16 == 0 &&
                        reinterpret_cast<uintptr_t>(dx) % 16 == 0,
                    "nf4_grouped_dx: dy, packed and dx must be 16-byte aligned");
    STRATUM_BIND_STREAM(stream);
    int *status = gemm::status_ptr();
    if (!status) return fail(STRATUM_ERR_CUDA, "nf4_grouped_dx: no status word");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int m_tiles = (K + grouped::BM - 1) / grouped::BM;
    grouped::Tile *tiles;
    int *ntiles, grid;
    int rc = build_table(offsets, E, m_tiles, grouped::BN, Ttot, table, table_bytes, status, st, &tiles, &ntiles,
                         &grid);
    if (rc) return rc;
    const CUtensorMapDataType xdt = dtype == STRATUM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap mdy, mw;
    rc = grouped::make_map(&mdy, xdt, dy_sorted, uint64_t(N_e), uint64_t(Ttot), uint64_t(N_e) * 2, 64, grouped::BN,
                           CU_TENSOR_MAP_SWIZZLE_128B, "nf4_grouped_dx dy");
    if (rc) return rc;
    rc = grouped::make_map(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, uint64_t(K / 2), uint64_t(E) * uint64_t(N_e),
                           uint64_t(K / 2), 64, 64, CU_TENSOR_MAP_SWIZZLE_64B, "nf4_grouped_dx packed");
    if (rc) return rc;
    grouped::DxParams p{};
    p.Ttot = Ttot; p.E = E; p.m_tiles = m_tiles; p.cap = grouped::BN;
    p.tiles = tiles; p.ntiles = ntiles; p.absmax = absmax; p.absmax_q = absmax_q; p.absmax2 = absmax2;
    p.code2 = code2; p.offset = offset; p.code16 = code16; p.dx = static_cast<uint16_t *>(dx);
    p.N_e = N_e; p.K = K; p.status = status;
    const bool bf = dtype == STRATUM_BF16;
    if (bf) return dq ? grouped::launch_dx<true, true>(mdy, mw, p, grid, st) : grouped::launch_dx<true, false>(mdy, mw, p, grid, st);
    return dq ? grouped::launch_dx<false, true>(mdy, mw, p, grid, st) : grouped::launch_dx<false, false>(mdy, mw, p, grid, st);
}

}  // extern "C"
