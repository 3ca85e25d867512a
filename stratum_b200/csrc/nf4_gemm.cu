// Fused NF4 GEMM for B200 (sm_100a): dequant-in-mainloop, tcgen05 tensor
// cores, TMEM accumulators, LoRA folded into the same accumulator.
//
// Forward (the reference's NF4Linear.forward + PEFT lora.Linear,
// stratum/nf4_linear.py:43-47, scripts/train.py:568-573):
//     y[T, N] = x[T, K] . W[N, K]^T + bias[N] + xa[T, r] . lora_B[N, r]^T
// with W stored NF4 (packed nibbles + per-64 absmax, optionally double
// quantized) and xa = scaling * x . lora_A^T computed beforehand.
//
// Layout of the work (swap-AB): the MMA computes D[n, t] = sum_k W[n, k] x[t, k]
// for a 128 (weight rows, TMEM lanes) x 384 (tokens: two MMAs of up to 192 that
// share the dequantized weight tile) tile, 64 K per stage; GEMMs with too few
// tiles to fill the GPU use 192-token tiles.
//   * the weight tile is the A operand and lives in TMEM: dequant warps turn
//     TMA-staged packed bytes into bf16/fp16 pairs in registers and
//     tcgen05.st them straight into TMEM, so the dequantized weight never
//     touches shared memory (shared-memory bandwidth is the scarce resource
//     once the tensor core runs at full rate);
//   * the token tile is the B operand, TMA-staged into 128B-swizzled shared
//     memory (K-major canonical layout);
//   * LoRA is one more K-chunk per 64 of rank: A = lora_B rows (staged into
//     TMEM by the same warps), B = the xa tile;
//   * the fp32 accumulator (384 TMEM columns) is drained by an epilogue
//     warpgroup that adds the bias, rounds and stores y, 192 tokens at a time.
// Warp roles (640 threads): w0 TMA producer of token tiles, w2 TMA producer
// of packed weight tiles (its own deep ring, so weights stream ahead of the
// MMA), w1 TMEM owner + MMA issuer, w4-15 dequant (three warpgroups taking
// turns by K-step; w%4 selects the TMEM lane quarter), w16-19 epilogue.
// Every wait is bounded; a timeout records a status word and unwinds.
#include "common.cuh"
#include "half8.cuh"
#include "nf4_decode.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>

namespace stratum {

// Status word of the GEMM kernels (0 = ok), one per device: [0] the code, then
// the record of the first wait that gave up (sm100::record_timeout) or of a
// rejected tile record (grouped::check_tiles); after the record, the wait limit
// (sm100::kLimitWord).
__device__ int g_gemm_status[sm100::kStatusAlloc];

namespace gemm {

using namespace sm100;


constexpr int BM = 128;       // weight rows per tile (TMEM lanes, MMA M)
constexpr int BN = 384;       // tokens per tile: two MMAs of up to BNH share each dequantized weight tile
constexpr int BNH = 192;      // tokens per MMA, per TMA box and per epilogue chunk
constexpr int BK = 64;        // K per step: one NF4 block per weight row
constexpr int XS = 3;         // stages: token tile (48 KiB) + dequantized weight tile (TMEM), released by MMA completion
constexpr int WS = 6;         // ring of packed weight tiles (4 KiB each), released by the dequant warps
constexpr int AS = XS;        // TMEM weight tiles (32 columns each), one per stage
constexpr int DQG = 3;        // dequant warpgroups; group g owns the steps with it % DQG == g
constexpr int X_BYTES = BN * BK * 2;    // 48 KiB: two [192 tokens][64] halves
constexpr int XH_BYTES = BNH * BK * 2;  // 24 KiB
constexpr int W_BYTES = BM * BK / 2;    // 4 KiB
constexpr int Y_HALF_BYTES = BNH * 64 * 2;  // staging of one 192-token chunk of y: two [192][64 rows] halves
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0;    // accumulator: columns [0, 384)
constexpr int A_COL0 = BN;    // A ring: columns [384, 384 + 32 * AS)
constexpr int EPI_WARP0 = 4 + 4 * DQG;
constexpr int NUM_THREADS = (EPI_WARP0 + 4) * 32;
constexpr int SMEM_BYTES = 1024 /*align slack*/ + XS * X_BYTES + WS * W_BYTES + 2 * Y_HALF_BYTES +
                           1024 /*barriers*/ + 2112 /*tables*/;
static_assert(A_COL0 + AS * 32 <= TMEM_COLS, "TMEM budget");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

// One NF4 weight's absmax (plain, or the double-quant set).
struct WeightScales {
    const float *absmax;      // [N, K/64] (plain)
    const uint8_t *absmax_q;  // [N, K/64] (double quant)
    const float *absmax2;     // [ceil(N*K/64 / 256)]
    const float *code2;       // [256]
    const float *offset;      // [1]
};

struct FwdParams {
    WeightScales w;           // the weight (SWIGLU: the gate projection's)
    WeightScales wu;          // SWIGLU: the up projection's
    const float *code16;      // [16]
    const void *bias;         // [N] or null
    int bias_dtype;
    const uint16_t *lora_b;   // [N, r] (bf16/fp16 bits) or null (SWIGLU: the gate projection's)
    const uint16_t *lora_bu;  // SWIGLU: the up projection's [N, r]
    int r;
    int lora_rp;              // SWIGLU: columns of xa per projection (r rounded up to 64)
    int lora_chunks;
    uint16_t *y;              // [T, N] (SWIGLU: h [T, N], N = the projections' width)
    uint16_t *gate, *up;      // SWIGLU, optional: the 16-bit gate and up [T, N] for the backward
    int64_t T, N, K;
    int n_tiles, t_tiles;
    int tile_tokens;          // tokens per tile: BN (two MMAs per K slice) or BNH (one)
    int tma_store;            // y stored through the staging tile + TMA (N % 8 == 0, 16-byte aligned)
    int *status;
};

// absmax of NF4 block b of a weight (plain, or rebuilt from the double-quant set
// with its code2 table in shared memory)
template <bool DQ>
__device__ __forceinline__ float block_scale(const WeightScales &w, const float *c2, int64_t b) {
    if constexpr (DQ) {
        return __fadd_rn(__fmul_rn(c2[__ldg(w.absmax_q + b)], __ldg(w.absmax2 + (b >> 8))), *w.offset);
    } else {
        return __ldg(w.absmax + b);
    }
}

struct Smem {
    uint8_t *x0;    // token tile i at x0 + i * X_BYTES (1024-byte aligned)
    uint8_t *w0;    // packed weight tile i at w0 + i * W_BYTES
    uint8_t *y0;    // y staging: two halves of Y_HALF_BYTES (1024-byte aligned)
    // full[s]: stage s's token tile landed (TMA bytes) and its weight tile is in TMEM
    // (128 dequant arrivals); empty[s]: the stage's MMAs completed (one commit)
    uint64_t *full, *empty, *wfull, *wempty, *accfull, *accempty, *drain;
    uint32_t *tmem_slot;
    float *lv, *c2, *c2u;
};

__device__ __forceinline__ Smem carve(uint8_t *raw) {
    Smem s;
    uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023);
    uint8_t *p = reinterpret_cast<uint8_t *>(base);
    s.x0 = p;
    p += XS * X_BYTES;
    s.y0 = p;
    p += 2 * Y_HALF_BYTES;
    s.w0 = p;
    p += WS * W_BYTES;
    uint64_t *b = reinterpret_cast<uint64_t *>(p);
    s.full = b; b += XS;
    s.empty = b; b += XS;
    s.wfull = b; b += WS;
    s.wempty = b; b += WS;
    s.accfull = b; b += 1;
    s.accempty = b; b += 1;
    s.drain = b; b += 1;
    s.tmem_slot = reinterpret_cast<uint32_t *>(b);
    s.lv = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(b) + 64);
    s.c2 = s.lv + 16;
    s.c2u = s.c2 + 256;
    return s;
}

__device__ __forceinline__ float load_bias(const void *bias, int dt, int64_t n) {
    if (dt == STRATUM_F32) return static_cast<const float *>(bias)[n];
    if (dt == STRATUM_BF16) return __bfloat162float(static_cast<const __nv_bfloat16 *>(bias)[n]);
    return __half2float(static_cast<const __half *>(bias)[n]);
}

template <bool BF16>
__device__ __forceinline__ uint16_t to16(float v) {
    if constexpr (BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return __half_as_ushort(__float2half_rn(v));
}

// SWIGLU: the tile's 128 weight rows are 64 rows of the gate projection (TMEM
// lanes 0-63, packed tiles from tm_w) and the same 64 rows of the up projection
// (lanes 64-127, from tm_w2); the epilogue forms h = silu(gate) * up from the
// 16-bit gate and up and writes h (and gate / up for the backward) -- the dense
// LlamaMLP up-projection in one pass over x.
template <bool BF16, bool DQ, bool SWIGLU>
__global__ void __launch_bounds__(NUM_THREADS, 1)
k_nf4_gemm_fwd(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
               const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_xa,
               const __grid_constant__ CUtensorMap tm_y, const FwdParams p) {
    extern __shared__ uint8_t smem_raw[];
    Smem sm = carve(smem_raw);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nkw = int(p.K / BK);
    const int nk = nkw + p.lora_chunks;
    const int ntiles = p.n_tiles * p.t_tiles;
    // tiles of this CTA: blockIdx.x + tl * gridDim.x, tl = 0 .. my_tiles - 1
    const int my_tiles = ntiles > int(blockIdx.x) ? (ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < XS; ++i) {
            mbar_init(&sm.full[i], 1 + 128);  // the token producer's expect-tx + the owning dequant warpgroup
            mbar_init(&sm.empty[i], 1);
        }
        for (int i = 0; i < WS; ++i) {
            mbar_init(&sm.wfull[i], 1);
            mbar_init(&sm.wempty[i], 128);  // the dequant warpgroup that owns the step
        }
        mbar_init(sm.accfull, 1);
        mbar_init(sm.accempty, 128);
        mbar_init(sm.drain, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 16) sm.lv[threadIdx.x] = p.code16[threadIdx.x];
    if (DQ) {
        for (int i = threadIdx.x; i < 256; i += NUM_THREADS) sm.c2[i] = p.w.code2[i];
        if (SWIGLU)
            for (int i = threadIdx.x; i < 256; i += NUM_THREADS) sm.c2u[i] = p.wu.code2[i];
    }
    if (warp == 1) tmem_alloc(sm.tmem_slot, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *sm.tmem_slot;

    if (warp == 0) {
        // ------------------------------------------- producer: token tiles
        if (lane == 0) {
            prefetch_tensormap(&tm_x);
            if (p.lora_chunks) prefetch_tensormap(&tm_xa);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const int t0 = ((int(blockIdx.x) + tl * int(gridDim.x)) / p.n_tiles) * p.tile_tokens;
                const bool second = p.T - t0 > BNH && p.tile_tokens > BNH;  // the tile has a second half
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % XS;
                    if (!mbar_wait(&sm.empty[s], ((it / XS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrFwdOffset)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.full[s], second ? X_BYTES : XH_BYTES);
                    const CUtensorMap *m = ks < nkw ? &tm_x : &tm_xa;
                    const int kc = (ks < nkw ? ks : ks - nkw) * BK;
                    // one or two 192-token boxes (zero-filled past the last token)
                    tma_load_2d(sm.x0 + s * X_BYTES, m, kc, t0, &sm.full[s]);
                    if (second) tma_load_2d(sm.x0 + s * X_BYTES + XH_BYTES, m, kc, t0 + BNH, &sm.full[s]);
                }
            }
            for (uint32_t j = (it > XS ? it - XS : 0); j < it; ++j)  // every copy lands before exit
                mbar_wait_issued(&sm.full[j % XS], (j / XS) & 1, p.status, kErrTimeoutTeardown + kErrFwdOffset);
            // the MMAs' last completion signals (commits into this CTA's shared memory)
            // land before the CTA exits: an arrival still in flight would hit the
            // shared memory of whichever CTA runs on this SM next
            if (ok)
                for (uint32_t j = (it > XS ? it - XS : 0); j < it; ++j)
                    mbar_wait(&sm.empty[j % XS], (j / XS) & 1, p.status, kErrTimeoutTeardown + kErrFwdOffset);
        }
    } else if (warp == 2) {
        // ---------------------------------- producer: packed weight tiles
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            if (SWIGLU) prefetch_tensormap(&tm_w2);
            uint32_t wt = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const int m = (int(blockIdx.x) + tl * int(gridDim.x)) % p.n_tiles;
                for (int ks = 0; ks < nkw; ++ks, ++wt) {
                    const int s = wt % WS;
                    if (!mbar_wait(&sm.wempty[s], ((wt / WS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrFwdOffset)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&sm.wfull[s], W_BYTES);
                    if constexpr (SWIGLU) {  // 64 gate rows, then the same 64 up rows
                        tma_load_2d(sm.w0 + s * W_BYTES, &tm_w, ks * (BK / 2), m * 64, &sm.wfull[s]);
                        tma_load_2d(sm.w0 + s * W_BYTES + W_BYTES / 2, &tm_w2, ks * (BK / 2), m * 64, &sm.wfull[s]);
                    } else {
                        tma_load_2d(sm.w0 + s * W_BYTES, &tm_w, ks * (BK / 2), m * BM, &sm.wfull[s]);
                    }
                }
            }
            for (uint32_t j = (wt > WS ? wt - WS : 0); j < wt; ++j)
                mbar_wait_issued(&sm.wfull[j % WS], (j / WS) & 1, p.status, kErrTimeoutTeardown + kErrFwdOffset);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                // the tile's two MMAs are only as wide as its tokens (multiples of 16)
                const int64_t t0 = int64_t((int(blockIdx.x) + tl * int(gridDim.x)) / p.n_tiles) * p.tile_tokens;
                const int ntok = int(p.T - t0 < p.tile_tokens ? p.T - t0 : p.tile_tokens);
                const int na = ((ntok < BNH ? ntok : BNH) + 15) & ~15;
                const int nb = ntok > BNH ? ((ntok - BNH + 15) & ~15) : 0;
                const uint32_t ida = idesc_f16(BF16, BM, na);
                const uint32_t idb = idesc_f16(BF16, BM, nb > 0 ? nb : 16);
                if (!mbar_wait(sm.accempty, (tl & 1) ^ 1, p.status, kErrTimeoutMma + kErrFwdOffset)) { ok = false; break; }
                tc_fence_after();
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    // one wait and one commit per stage: each costs the issuing thread
                    // ~100 cycles that the tensor pipe spends idle
                    const int s = it % XS;
                    if (!mbar_wait(&sm.full[s], (it / XS) & 1, p.status, kErrTimeoutMma + kErrFwdOffset)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t bda = smem_desc_k_sw128(sm.x0 + s * X_BYTES);
                    const uint64_t bdb = smem_desc_k_sw128(sm.x0 + s * X_BYTES + XH_BYTES);
                    const uint32_t a0 = tmem + A_COL0 + s * 32;
                    // each K slice of the dequantized weight tile feeds both token halves
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j) {
                        mma_ts_f16(tmem + ACC_COL, a0 + j * 8, bda + uint64_t(j * 2), ida, (ks | j) != 0);
                        if (nb) mma_ts_f16(tmem + ACC_COL + BNH, a0 + j * 8, bdb + uint64_t(j * 2), idb, (ks | j) != 0);
                    }
                    mma_commit(&sm.empty[s]);
                }
                if (ok) mma_commit(sm.accfull);
            }
            mma_commit(sm.drain);  // all issued MMAs complete before TMEM is released
            mbar_wait_issued(sm.drain, 0, p.status, kErrTimeoutTeardown + kErrFwdOffset);
        }
    } else if (warp >= 4 && warp < EPI_WARP0) {
        // ---------------------------------------------------- dequant warps
        const int grp = (warp - 4) >> 2;
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        // SWIGLU: lanes 64-127 hold up-projection rows (warp-uniform: q >= 2)
        const bool upper = SWIGLU && q >= 2;
        const WeightScales &ws = upper ? p.wu : p.w;
        const float *c2 = upper ? sm.c2u : sm.c2;
        float lv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lv[i] = sm.lv[i];
        const int64_t kb = p.K / BK;
        // weight row of this lane in tile tl (SWIGLU: row of its projection)
        auto row_of = [&](int tl) -> int64_t {
            const int m = (int(blockIdx.x) + tl * int(gridDim.x)) % p.n_tiles;
            return SWIGLU ? int64_t(m) * 64 + (row & 63) : int64_t(m) * BM + row;
        };
        // (tile turn, step) of a position in the group's walk, advanced DQG steps at a
        // time with no division (the row is recomputed only when the tile changes)
        struct Pos {
            int tl, ks;
            int64_t n;
        };
        auto norm = [&](Pos &q) {
            if (q.ks < nk) return;
            while (q.ks >= nk) {
                q.ks -= nk;
                ++q.tl;
            }
            if (q.tl < my_tiles) q.n = row_of(q.tl);
        };
        auto absmax_at = [&](const Pos &q) -> float {
            if (q.tl >= my_tiles || q.ks >= nkw || q.n >= p.N) return 0.f;
            return block_scale<DQ>(ws, c2, q.n * kb + q.ks);
        };
        const uint32_t total = uint32_t(my_tiles) * uint32_t(nk);
        Pos cur{0, grp, row_of(0)};
        norm(cur);
        Pos nxt{cur.tl, cur.ks + DQG, cur.n};
        norm(nxt);
        float am_next = absmax_at(cur);
        for (uint32_t it = uint32_t(grp); it < total; it += DQG, cur = nxt, nxt.ks += DQG, norm(nxt)) {
            const float am = am_next;
            am_next = absmax_at(nxt);  // one owned step ahead
            const int tl = cur.tl, ks = cur.ks;
            const int64_t n = cur.n;
            uint32_t vals[32];
            if (ks < nkw) {
                const uint32_t wt = uint32_t(tl) * uint32_t(nkw) + uint32_t(ks);
                const int s = wt % WS;
                // warp-uniform outcome: the tcgen05.st below is a warp collective
                if (!__all_sync(0xffffffffu, mbar_wait(&sm.wfull[s], (wt / WS) & 1, p.status, kErrTimeoutDequant + kErrFwdOffset)))
                    break;
                // 32-byte swizzled tile: row r's 16-byte halves are swapped when bit 2 of r is set
                const uint4 *src = reinterpret_cast<const uint4 *>(sm.w0 + s * W_BYTES + row * 32);
                const int sw = (row >> 2) & 1;
                const uint4 p0 = src[sw], p1 = src[sw ^ 1];
                const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                const Nf4Tables t = nf4_build_tables<BF16>(lv, am);
                nf4_decode_block(t, w, vals);
                // release the stage only once the words are consumed, and order these
                // generic-proxy reads before the TMA (async proxy) refill of the stage
                fence_proxy_async_smem();
                mbar_arrive(&sm.wempty[s]);
            } else {
                const int j0 = (ks - nkw) * BK;
                const bool valid = n < p.N;
                if constexpr (SWIGLU) {
                    // xa = [gate's xa | 0-pad | up's xa | 0-pad], lora_rp columns each: the gate
                    // rows take lora_b over columns [0, r), the up rows lora_bu over [rp, rp + r)
                    const uint16_t *lb = upper ? p.lora_bu : p.lora_b;
                    const int c0 = upper ? p.lora_rp : 0;
#pragma unroll
                    for (int m = 0; m < 32; ++m) {
                        const int j = j0 + 2 * m - c0;
                        vals[m] = (valid && j >= 0 && j < p.r)
                                      ? __ldg(reinterpret_cast<const uint32_t *>(lb + n * p.r + j)) : 0u;
                    }
                } else {
#pragma unroll
                    for (int m = 0; m < 32; ++m) {
                        const int j = j0 + 2 * m;
                        vals[m] = (valid && j < p.r) ? __ldg(reinterpret_cast<const uint32_t *>(p.lora_b + n * p.r + j))
                                                     : 0u;
                    }
                }
            }
            const int sa = it % AS;
            if (!__all_sync(0xffffffffu, mbar_wait(&sm.empty[sa], ((it / AS) & 1) ^ 1, p.status, kErrTimeoutDequant + kErrFwdOffset)))
                break;
            tc_fence_after();
            tmem_st_32x32b_x32(tmem + lane_addr + A_COL0 + sa * 32, vals);
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&sm.full[sa]);
        }
    } else if (warp >= EPI_WARP0) {
        // --------------------------------------------------------- epilogue
        const int q = warp & 3;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        const bool leader = warp == EPI_WARP0 && lane == 0;
        for (int tl = 0; tl < my_tiles; ++tl) {
            if (!__all_sync(0xffffffffu, mbar_wait(sm.accfull, tl & 1, p.status, kErrTimeoutEpilogue + kErrFwdOffset))) break;
            tc_fence_after();
            const int tile = int(blockIdx.x) + tl * int(gridDim.x);
            const int64_t n0 = int64_t(tile % p.n_tiles) * BM;
            const int64_t t0 = int64_t(tile / p.n_tiles) * p.tile_tokens;
            const int ntok = int(p.T - t0 < p.tile_tokens ? p.T - t0 : p.tile_tokens);
            const int nchunks = ntok > BNH ? 2 : 1;
            if (SWIGLU || p.tma_store) {
                // TMEM -> registers as 16x256b fragments (row = weight row, pairs of
                // tokens), + bias, -> 16-bit -> stmatrix.trans into the [token][row]
                // staging tile, then one TMA store per 64-row half; the tile's tokens go
                // through in chunks of 192 (one per MMA), the accumulator is released
                // once its last columns are read.
                float bias[2][2];
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int64_t n = n0 + q * 32 + h * 16 + (lane >> 2) + 8 * e;
                        bias[h][e] = (p.bias && n < p.N) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
                    }
                // this thread's stmatrix row: matrix k = lane/8, row j = lane%8
                const int k = lane >> 3, j = lane & 7;
                const int tok_in = j + 8 * (k >> 1);         // token offset within a 16-column block
                const int nrow = q * 32 + 8 * (k & 1);        // + 16h: first weight row of the 8x8 matrix
                auto stage_block = [&](int cb, const uint32_t (&v)[2][8]) {
                    const int tok = cb * 16 + tok_in;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t x4[4];
#pragma unroll
                        for (int m = 0; m < 4; ++m) {
                            const float b = bias[h][m & 1];
                            const float lo = __uint_as_float(v[h][2 * m]) + b;
                            const float hi = __uint_as_float(v[h][2 * m + 1]) + b;
                            x4[m] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                        }
                        // registers {0,1}: rows +0, tokens +0..7; {2,3}: rows +8; {4,5}/{6,7}: tokens +8
                        const int nr = nrow + 16 * h;
                        const int half = nr >> 6, chunk = (nr & 63) >> 3;
                        const uint8_t *dst = sm.y0 + half * Y_HALF_BYTES + tok * 128 + ((chunk ^ (tok & 7)) << 4);
                        stmatrix_x4_trans(smem_u32(dst), x4[0], x4[1], x4[2], x4[3]);
                    }
                };
#pragma unroll 1
                for (int c = 0; c < nchunks; ++c) {
                    const int ctok = (ntok - c * BNH < BNH ? ntok - c * BNH : BNH);  // tokens of this chunk
                    const int nblk = (ctok + 15) >> 4;
                    const uint32_t col0 = uint32_t(ACC_COL + c * BNH);
                    const int64_t tc0 = t0 + c * BNH;
                    if (leader) bulk_wait_read0();  // the previous store has read the staging tile
                    named_bar_sync(1, 128);
                    // two 16-token column blocks per TMEM load wait: half the round trips
                    // on the path that holds the accumulator
#pragma unroll 1
                    for (int cb = 0; cb < nblk; cb += 2) {
                        const bool pair = cb + 1 < nblk;  // warp-uniform
                        uint32_t v0[2][8], v1[2][8];
                        tmem_ld_16x256b_x2(tmem + lane_addr + col0 + cb * 16, v0[0]);
                        tmem_ld_16x256b_x2(tmem + lane_addr + (16u << 16) + col0 + cb * 16, v0[1]);
                        if (pair) {
                            tmem_ld_16x256b_x2(tmem + lane_addr + col0 + (cb + 1) * 16, v1[0]);
                            tmem_ld_16x256b_x2(tmem + lane_addr + (16u << 16) + col0 + (cb + 1) * 16, v1[1]);
                        }
                        tmem_ld_wait();
                        if (c == nchunks - 1 && cb + 2 >= nblk) {  // accumulator read: the next tile may start
                            tc_fence_before();
                            mbar_arrive(sm.accempty);
                        }
                        stage_block(cb, v0);
                        if (pair) stage_block(cb + 1, v1);
                    }
                    if constexpr (SWIGLU) {
                        // staging half 0 holds the chunk's 64 gate rows, half 1 the same 64 up
                        // rows (16-bit, as HF's bf16 projections round them): h = silu(gate) * up,
                        // 8 columns per 16-byte chunk, stored row by row with the gate and up
                        named_bar_sync(1, 128);
                        const int etid = int(threadIdx.x) - EPI_WARP0 * 32;
                        const int64_t colw = int64_t(tile % p.n_tiles) * 64;
                        for (int idx = etid; idx < ctok * 8; idx += 128) {
                            const int tok = idx >> 3, chunk = idx & 7;
                            const int64_t col = colw + chunk * 8;
                            if (col >= p.N) continue;
                            const int off = tok * 128 + ((chunk ^ (tok & 7)) << 4);
                            const uint4 gv = *reinterpret_cast<const uint4 *>(sm.y0 + off);
                            const uint4 uv = *reinterpret_cast<const uint4 *>(sm.y0 + Y_HALF_BYTES + off);
                            float g[8], u[8], h[8];
                            h16::unpack8<BF16>(gv, g);
                            h16::unpack8<BF16>(uv, u);
                            h16::swiglu_fwd8<BF16>(g, u, h);  // cheap on the SM the decode warps share
                            const int64_t at = (tc0 + tok) * p.N + col;
                            *reinterpret_cast<uint4 *>(p.y + at) = h16::pack8<BF16>(h);
                            if (p.gate) *reinterpret_cast<uint4 *>(p.gate + at) = gv;
                            if (p.up) *reinterpret_cast<uint4 *>(p.up + at) = uv;
                        }
                    } else {
                        fence_proxy_async_smem();
                        named_bar_sync(1, 128);
                        if (leader) {
                            tma_store_2d(&tm_y, int32_t(n0), int32_t(tc0), sm.y0);
                            if (n0 + 64 < p.N) tma_store_2d(&tm_y, int32_t(n0 + 64), int32_t(tc0), sm.y0 + Y_HALF_BYTES);
                            bulk_commit();
                        }
                    }
                }
            } else {
                // generic path (N % 8 != 0 or unaligned y): element stores
                const int row = q * 32 + lane;
                const int64_t n = n0 + row;
                const float bias = (n < p.N && p.bias) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
                const int nblk = (ntok + 31) >> 5;
#pragma unroll 1
                for (int c = 0; c < nblk; ++c) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem + lane_addr + ACC_COL + c * 32, v);
                    tmem_ld_wait();
                    if (c == nblk - 1) {
                        tc_fence_before();
                        mbar_arrive(sm.accempty);
                    }
                    if (n < p.N) {
                        const int64_t tcb = t0 + c * 32;
                        for (int i = 0; i < 32 && tcb + i < p.T; ++i)
                            p.y[(tcb + i) * p.N + n] = to16<BF16>(__uint_as_float(v[i]) + bias);
                    }
                }
            }
        }
        if (leader) bulk_wait0();  // stores complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// =================================================================== dX ===
//
// Input gradient (autograd of NF4Linear.forward / PEFT lora.Linear):
//     dX[T, K] = dY[T, N] . W[N, K] + dyb[T, r] . lora_A[r, K]
// with dyb = scaling * dY . lora_B computed beforehand.  Swap-AB again: the
// MMA computes D[k, t] = sum_n W[n, k] dY[t, n] for 128 columns of W (TMEM
// lanes) x 256 tokens, 64 rows of W per step.  The contraction now runs over
// W's rows, so the A operand is W^T: the dequant warps decode each (row,
// 64-column block) of W -- one NF4 block, exactly as in the forward -- and
// write the 64 values as one 128-byte row of an MN-major, 128B-swizzled
// shared-memory tile (conflict-free), which tcgen05.mma reads transposed.
// The kernel keeps no weight tile in TMEM, so the accumulator is double
// buffered (2 x 256 columns) and the epilogue of tile i overlaps the
// mainloop of tile i+1.
namespace dx {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int XS = 3;               // stages: dY tile (32 KiB) + dequantized W^T tile (16 KiB)
constexpr int WS = 4;               // packed weight tiles: 64 rows x 64 bytes (4 KiB)
constexpr int AS = XS;              // dequantized W^T tiles in shared memory, one per stage
constexpr int DQG = 3;
constexpr int X_BYTES = BN * BK * 2;
constexpr int W_BYTES = BK * BM / 2;
constexpr int A_BYTES = BM * BK * 2;
constexpr int A_ATOM = BK * 128;    // one 64-column MN atom: 64 K-rows x 128 B
constexpr int Y_HALF_BYTES = BN * 64 * 2;
constexpr int EPI_WARP0 = 4 + 4 * DQG;
constexpr int NUM_THREADS = (EPI_WARP0 + 4) * 32;
constexpr int SMEM_BYTES = 1024 + XS * X_BYTES + AS * A_BYTES + 2 * Y_HALF_BYTES + WS * W_BYTES + 512 + 1088;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Params {
    WeightScales w;          // the weight (PAIR: the first of the two stacked weights)
    WeightScales w1;         // PAIR: the second weight
    const float *code16;
    const uint16_t *lora_a;  // [r, K] or null
    int r;
    int lora_chunks;
    uint16_t *dx;            // [T, K]
    int64_t T, N, K;
    int nkw0;                // PAIR: contraction steps (64 rows each) over the first weight
    int k_tiles, t_tiles;
    int tma_store;
    int *status;
};

// PAIR: the contraction runs over two NF4 weights stacked along N (rows [0, N0)
// from tm_w, [N0, N) from tm_w2), e.g. the gate and up projections of an MLP whose
// dY is [dgate | dup].
template <bool BF16, bool DQ, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
k_nf4_gemm_dx(const __grid_constant__ CUtensorMap tm_dy, const __grid_constant__ CUtensorMap tm_w,
              const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_dyb,
              const __grid_constant__ CUtensorMap tm_dx, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *x0 = base;                              // XS x 32 KiB (1024-aligned)
    uint8_t *a0 = x0 + XS * X_BYTES;                 // AS x 16 KiB (1024-aligned)
    uint8_t *y0 = a0 + AS * A_BYTES;                 // 2 x 32 KiB (1024-aligned)
    uint8_t *w0 = y0 + 2 * Y_HALF_BYTES;             // WS x 4 KiB
    uint64_t *bars = reinterpret_cast<uint64_t *>(w0 + WS * W_BYTES);
    // full[s]: stage s's dY tile landed (TMA bytes) and its W^T tile is in shared memory
    // (128 dequant arrivals); empty[s]: the stage's MMAs completed (one commit)
    uint64_t *full = bars, *empty = full + XS, *wfull = empty + XS, *wempty = wfull + WS;
    uint64_t *accfull = wempty + WS, *accempty = accfull + 2;
    uint64_t *drain = accempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    float *lv_s = reinterpret_cast<float *>(bars + 64);
    float *c2 = lv_s + 16;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nkw = int((p.N + BK - 1) / BK);  // weight-row steps (ragged last step zero-filled)
    const int nk = nkw + p.lora_chunks;
    const int ntiles = p.k_tiles * p.t_tiles;
    const int my_tiles = ntiles > int(blockIdx.x) ? (ntiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < XS; ++i) { mbar_init(&full[i], 1 + 128); mbar_init(&empty[i], 1); }
        for (int i = 0; i < WS; ++i) { mbar_init(&wfull[i], 1); mbar_init(&wempty[i], 128); }
        for (int i = 0; i < 2; ++i) { mbar_init(&accfull[i], 1); mbar_init(&accempty[i], 128); }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 16) lv_s[threadIdx.x] = p.code16[threadIdx.x];
    if (DQ) {
        for (int i = threadIdx.x; i < 256; i += NUM_THREADS) c2[i] = p.w.code2[i];
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------- producer: dY (and dyb) tiles
        if (lane == 0) {
            prefetch_tensormap(&tm_dy);
            if (p.lora_chunks) prefetch_tensormap(&tm_dyb);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const int t0 = ((int(blockIdx.x) + tl * int(gridDim.x)) / p.k_tiles) * BN;
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % XS;
                    if (!mbar_wait(&empty[s], ((it / XS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrDxOffset)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], X_BYTES);
                    if (ks < nkw) tma_load_2d(x0 + s * X_BYTES, &tm_dy, ks * BK, t0, &full[s]);
                    else tma_load_2d(x0 + s * X_BYTES, &tm_dyb, (ks - nkw) * BK, t0, &full[s]);
                }
            }
            for (uint32_t j = (it > XS ? it - XS : 0); j < it; ++j)
                mbar_wait_issued(&full[j % XS], (j / XS) & 1, p.status, kErrTimeoutTeardown + kErrDxOffset);
            // the MMAs' last completion signals (commits into this CTA's shared memory)
            // land before the CTA exits: an arrival still in flight would hit the
            // shared memory of whichever CTA runs on this SM next
            if (ok)
                for (uint32_t j = (it > XS ? it - XS : 0); j < it; ++j)
                    mbar_wait(&empty[j % XS], (j / XS) & 1, p.status, kErrTimeoutTeardown + kErrDxOffset);
        }
    } else if (warp == 2) {
        // ------------------------------- producer: packed weight tiles (64 x 128)
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            if (PAIR) prefetch_tensormap(&tm_w2);
            uint32_t wt = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const int k0 = ((int(blockIdx.x) + tl * int(gridDim.x)) % p.k_tiles) * BM;
                for (int ks = 0; ks < nkw; ++ks, ++wt) {
                    const int s = wt % WS;
                    if (!mbar_wait(&wempty[s], ((wt / WS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrDxOffset)) { ok = false; break; }
                    mbar_arrive_expect_tx(&wfull[s], W_BYTES);
                    if (PAIR && ks >= p.nkw0) tma_load_2d(w0 + s * W_BYTES, &tm_w2, k0 / 2, (ks - p.nkw0) * BK, &wfull[s]);
                    else tma_load_2d(w0 + s * W_BYTES, &tm_w, k0 / 2, ks * BK, &wfull[s]);
                }
            }
            for (uint32_t j = (wt > WS ? wt - WS : 0); j < wt; ++j)
                mbar_wait_issued(&wfull[j % WS], (j / WS) & 1, p.status, kErrTimeoutTeardown + kErrDxOffset);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_amn(BF16, BM, BN);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                const int ab = tl & 1;
                if (!mbar_wait(&accempty[ab], ((tl >> 1) & 1) ^ 1, p.status, kErrTimeoutMma + kErrDxOffset)) { ok = false; break; }
                tc_fence_after();
                const uint32_t acc = tmem + uint32_t(ab * 256);
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % XS, sa = s;
                    if (!mbar_wait(&full[s], (it / XS) & 1, p.status, kErrTimeoutMma + kErrDxOffset)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_k_sw128(x0 + s * X_BYTES);
                    const uint64_t adesc = smem_desc_mn_sw128(a0 + sa * A_BYTES, A_ATOM, 1024);
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j)  // 16 K-rows = two 8-row groups = 2 KiB further
                        mma_ss_f16(acc, adesc + uint64_t(j * (2048 >> 4)), bdesc + uint64_t(j * 2), idesc, (ks | j) != 0);
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&accfull[ab]);
            }
            mma_commit(drain);
            mbar_wait_issued(drain, 0, p.status, kErrTimeoutTeardown + kErrDxOffset);
        }
    } else if (warp >= 4 && warp < EPI_WARP0) {
        // ---------------------------------------------------- dequant warps
        // thread -> (weight row rl = tid % 64 of the step, 64-column block kb = tid / 64)
        const int grp = (warp - 4) >> 2;
        const int tid = (warp & 3) * 32 + lane;
        const int rl = tid & 63, kb = tid >> 6;
        float lv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lv[i] = lv_s[i];
        const int64_t kbl = p.K / 64;  // NF4 blocks per weight row
        // (tile turn, step) of a position in the group's walk, advanced DQG steps at a
        // time with no division (the column block is recomputed only when the tile changes)
        struct Pos {
            int tl, ks;
            int64_t kb0;  // first NF4 column block of the tile
        };
        auto kb0_of = [&](int tl) { return int64_t((int(blockIdx.x) + tl * int(gridDim.x)) % p.k_tiles) * 2; };
        auto norm = [&](Pos &q) {
            if (q.ks < nk) return;
            while (q.ks >= nk) {
                q.ks -= nk;
                ++q.tl;
            }
            if (q.tl < my_tiles) q.kb0 = kb0_of(q.tl);
        };
        auto block_at = [&](const Pos &q, int64_t &wrow, int64_t &kblk) {
            wrow = int64_t(q.ks) * BK + rl;
            kblk = q.kb0 + kb;
            return q.ks;
        };
        auto absmax_at = [&](const Pos &q) -> float {
            if (q.tl >= my_tiles) return 0.f;
            int64_t wrow, kblk;
            const int ks = block_at(q, wrow, kblk);
            if (ks >= nkw || wrow >= p.N || kblk >= kbl) return 0.f;
            if (PAIR && ks >= p.nkw0)  // a row of the second weight (step-uniform choice); its code2
                // table is read from global memory (shared memory has room for one table only)
                return block_scale<DQ>(p.w1, p.w1.code2, (wrow - int64_t(p.nkw0) * BK) * kbl + kblk);
            return block_scale<DQ>(p.w, c2, wrow * kbl + kblk);
        };
        const uint32_t total = uint32_t(my_tiles) * uint32_t(nk);
        Pos cur{0, grp, kb0_of(0)};
        norm(cur);
        Pos nxt{cur.tl, cur.ks + DQG, cur.kb0};
        norm(nxt);
        float am_next = absmax_at(cur);
        for (uint32_t it = uint32_t(grp); it < total; it += DQG, cur = nxt, nxt.ks += DQG, norm(nxt)) {
            const float am = am_next;
            am_next = absmax_at(nxt);  // one owned step ahead
            int64_t wrow, kblk;
            const int ks = block_at(cur, wrow, kblk);
            const int tl = cur.tl;
            uint32_t vals[32];
            if (ks < nkw) {
                const uint32_t wt = uint32_t(tl) * uint32_t(nkw) + uint32_t(ks);
                const int s = wt % WS;
                if (!__all_sync(0xffffffffu, mbar_wait(&wfull[s], (wt / WS) & 1, p.status, kErrTimeoutDequant + kErrDxOffset))) break;
                // 64-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3)
                const uint4 *src = reinterpret_cast<const uint4 *>(w0 + s * W_BYTES + rl * 64);
                const int sw = (rl >> 1) & 3;
                const uint4 p0 = src[(2 * kb) ^ sw], p1 = src[(2 * kb + 1) ^ sw];
                const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                const Nf4Tables t = nf4_build_tables<BF16>(lv, am);
                nf4_decode_block(t, w, vals);
                // release the stage only once the words are consumed, and order these
                // generic-proxy reads before the TMA (async proxy) refill of the stage
                fence_proxy_async_smem();
                mbar_arrive(&wempty[s]);
            } else {
                // LoRA chunk: rank row j of lora_A, 64 columns (zero beyond r / K)
                const int j = (ks - nkw) * BK + rl;
                const bool ok_row = j < p.r && kblk < kbl;
                const uint4 *src = reinterpret_cast<const uint4 *>(p.lora_a + int64_t(j) * p.K + kblk * 64);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 v = ok_row ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
                    vals[4 * c] = v.x; vals[4 * c + 1] = v.y; vals[4 * c + 2] = v.z; vals[4 * c + 3] = v.w;
                }
            }
            const int sa = it % AS;
            if (!__all_sync(0xffffffffu, mbar_wait(&empty[sa], ((it / AS) & 1) ^ 1, p.status, kErrTimeoutDequant + kErrDxOffset))) break;
            // MN-major atom kb, K-row rl: 8 chunks of 16 B, XOR-swizzled by rl % 8
            uint8_t *dst = a0 + sa * A_BYTES + kb * A_ATOM + (rl >> 3) * 1024 + (rl & 7) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4 *>(dst + ((c ^ (rl & 7)) << 4)) =
                    make_uint4(vals[4 * c], vals[4 * c + 1], vals[4 * c + 2], vals[4 * c + 3]);
            fence_proxy_async_smem();  // generic-proxy writes -> visible to tcgen05.mma
            mbar_arrive(&full[sa]);
        }
    } else if (warp >= EPI_WARP0) {
        // --------------------------------------------------------- epilogue
        const int q = warp & 3;
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        const bool leader = warp == EPI_WARP0 && lane == 0;
        const int kq = lane >> 3, jr = lane & 7;
        const int tok_in = jr + 8 * (kq >> 1);
        const int nrow = q * 32 + 8 * (kq & 1);
        for (int tl = 0; tl < my_tiles; ++tl) {
            const int ab = tl & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&accfull[ab], (tl >> 1) & 1, p.status, kErrTimeoutEpilogue + kErrDxOffset))) break;
            tc_fence_after();
            const int tile = int(blockIdx.x) + tl * int(gridDim.x);
            const int64_t k0 = int64_t(tile % p.k_tiles) * BM;
            const int64_t t0 = int64_t(tile / p.k_tiles) * BN;
            const uint32_t acc = tmem + lane_addr + uint32_t(ab * 256);
            if (p.tma_store) {
                if (leader) bulk_wait_read0();
                named_bar_sync(1, 128);
#pragma unroll 1
                for (int cb = 0; cb < BN / 16; ++cb) {
                    uint32_t v[2][8];
                    tmem_ld_16x256b_x2(acc + cb * 16, v[0]);
                    tmem_ld_16x256b_x2(acc + (16u << 16) + cb * 16, v[1]);
                    tmem_ld_wait();
                    if (cb == BN / 16 - 1) {
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
                        const uint8_t *dst = y0 + half * Y_HALF_BYTES + tok * 128 + ((chunk ^ (tok & 7)) << 4);
                        stmatrix_x4_trans(smem_u32(dst), x4[0], x4[1], x4[2], x4[3]);
                    }
                }
                fence_proxy_async_smem();
                named_bar_sync(1, 128);
                if (leader) {
                    tma_store_2d(&tm_dx, int32_t(k0), int32_t(t0), y0);
                    if (k0 + 64 < p.K) tma_store_2d(&tm_dx, int32_t(k0 + 64), int32_t(t0), y0 + Y_HALF_BYTES);
                    bulk_commit();
                }
            } else {
                const int64_t k = k0 + q * 32 + lane;
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(acc + c * 32, v);
                    tmem_ld_wait();
                    if (c == BN / 32 - 1) {
                        tc_fence_before();
                        mbar_arrive(&accempty[ab]);
                    }
                    if (k < p.K) {
                        const int64_t tc0 = t0 + c * 32;
                        for (int i = 0; i < 32 && tc0 + i < p.T; ++i)
                            p.dx[(tc0 + i) * p.K + k] = to16<BF16>(__uint_as_float(v[i]));
                    }
                }
            }
        }
        if (leader) bulk_wait0();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace dx

// ================================================ CTA-pair GEMMs (2 SMs) ===
//
// The forward and the input gradient on CTA pairs (clusters of two) sharing
// 2-SM tcgen05 MMAs.  A pair tile is 256 output columns (the MMA's M: weight
// rows for the forward, weight columns for dX; each CTA decodes its own 128
// into a 128B-swizzled shared-memory A tile) x 512 tokens (two MMAs of N = 256
// per 16-wide K slice; each CTA stages half of each MMA's tokens).
// Why: one thread issuing tcgen05.mma costs ~95 cycles per instruction (~120
// with ALU-heavy warps on its sub-partition) whatever the instruction's size,
// so only N = 256 instructions (128 tensor cycles per SM) leave the issuing
// thread slack, and eight of them per 64-wide K step (1024 tensor cycles)
// amortise the step's one barrier wait and one commit.  A 512-token tile on one
// SM would need 80 KiB per stage; the pair halves the token bytes per SM.
// With the weight tile in shared memory the decode warps are not tied to TMEM
// lane quarters (see dq_index for their placement).  The fp32 accumulator fills
// TMEM (2 x 256 columns): a tile's epilogue runs before the next tile's
// mainloop, so the epilogue streams: TMEM loads software-pipelined by 16-token
// blocks, each warp's 32 x 32 chunk transposed through 2 KiB of shared memory
// and written with 16-byte global stores (no store-completion waits).
// The decoded tile has one physical layout in both directions: decode thread t
// writes 128-byte row t (8-row groups of 1024 bytes, 16-byte chunk c at chunk
// position c ^ (t % 8)).  The forward's thread t decodes weight row t (64
// values along K) and the MMA reads the tile K-major; dX's thread t decodes
// weight row t % 64 over columns 64 * (t / 64) .. + 63, i.e. two 64-column
// MN atoms of 8 KiB, and the MMA reads it MN-major (W^T).
// Barriers (each waited on by threads of the CTA that holds it): the first
// CTA's full[s] counts its producer's expect_tx (both CTAs' token bytes: each
// CTA's TMA signals it) and one arrival per decode warp of both CTAs, its
// accempty one per epilogue warp of both CTAs; empty[s], accfull and drain are
// arrived on in both CTAs by multicast commits.  Arrivals
// from the second CTA use the default (CTA-scope release) semantics, as
// cluster barriers between the CTAs of a 2-SM MMA are signalled; a
// cluster-scope release costs the arriving thread ~1500 cycles.
// Every wait is bounded, as in the single-CTA kernels.
#ifndef PAIR_DQG
#define PAIR_DQG 3
#endif
#ifndef PAIR_EPI
#define PAIR_EPI 4
#endif
namespace pair {

constexpr int BM = 128;                        // output columns per CTA; the pair's MMA M is 256
constexpr int BN = 512;                        // tokens per pair tile: two MMAs of NH
constexpr int NH = 256;                        // tokens per MMA (N)
constexpr int CT = NH / 2;                     // tokens of each MMA staged by each CTA
constexpr int BK = 64;                         // contraction per step: one NF4 block per decode thread
constexpr int XS = 4;                          // stages: this CTA's two 128-token halves (32 KiB) + its A tile (16 KiB)
constexpr int WS = 4;                          // packed weight tiles (4 KiB), released by the decode warps
constexpr int X_HALF = CT * BK * 2;            // 16 KiB: [128 tokens][64] of one MMA
constexpr int X_BYTES = 2 * X_HALF;
constexpr int A_BYTES = BM * BK * 2;           // 16 KiB
constexpr int A_ATOM = BK * 128;               // dX: one 64-column MN atom (64 K-rows x 128 B)
constexpr int W_BYTES = BM * BK / 2;           // 4 KiB
constexpr int CH = 32;                         // tokens per epilogue chunk
constexpr int YW_BYTES = CH * 32 * 2;          // one epilogue warp's chunk: [32 tokens][32 columns], 64B swizzle
constexpr int EPI_WARPS = PAIR_EPI;            // epilogue warps: 4 (one per TMEM lane quarter) or 8 (two)
constexpr int PART_TOK = BN / (EPI_WARPS / 4); // tokens of a tile drained by one warp
constexpr int Y_BUF_BYTES = EPI_WARPS * YW_BYTES;  // the epilogue warps' chunks
constexpr int DQG = PAIR_DQG;                  // decode groups (four warps each) taking turns by K step
constexpr int EPI_WARP0 = 16;
constexpr int NUM_THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES =
    1024 + XS * (X_BYTES + A_BYTES) + Y_BUF_BYTES + WS * W_BYTES + BAR_BYTES + (16 + 256) * 4;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");
static_assert((2 * XS + 2 * WS + 3) * 8 + 8 <= BAR_BYTES, "barrier area");

struct Params {
    WeightScales w;            // the weight (dX over two stacked weights: the first)
    WeightScales w1;           // dX over two stacked weights: the second
    const float *code16;
    const void *bias;          // forward: [M] or null
    int bias_dtype;
    const uint16_t *lora;      // forward: lora_b [M, r]; dX: lora_a [r, M]; null when r == 0
    int r, lora_chunks;
    uint16_t *y;               // output [T, M]
    int64_t T;
    int64_t M;                 // output columns (forward: N; dX: K)
    int64_t C;                 // contraction over the weight (forward: K; dX: N)
    int64_t kbl;               // NF4 blocks per weight row (the weight's K / 64)
    int nkw0;                  // dX over two weights: contraction steps over the first
    int m_tiles, t_tiles;
    int tma_store;             // the output takes 16-byte vector stores (aligned, M % 8 == 0)
    int *status;
};

// Decode warps (-1 for the others): with three groups, warps 4..15 on all four
// sub-partitions; with two, the eight among them not on sub-partition 1, which
// then keeps the MMA thread to itself.  Three measured faster: the MMA thread
// issues its eight MMAs in ~500 of a step's 1024 tensor cycles, so sharing its
// sub-partition costs less than a third stage of decode slack gains.
__device__ __forceinline__ int dq_index(int warp) {
    if (warp < 4 || warp >= EPI_WARP0) return -1;
    if (DQG == 3) return warp - 4;  // warps 4..15 on all four sub-partitions
    if ((warp & 3) == 1) return -1;
    const int a = warp - 4;
    const int idx = a - (a + 3) / 4;
    return idx < 4 * DQG ? idx : -1;
}

// DX: input gradient (A = W^T, MN-major); TWO_W: its contraction runs over two
// NF4 weights stacked along N (rows [0, N0) from tm_w, the rest from tm_w2).
template <bool BF16, bool DQ, bool DX, bool TWO_W>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
k_nf4_gemm_pair(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_xl,
                const __grid_constant__ CUtensorMap tm_y /* unused: y is written with vector stores */,
                const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *x0 = base;                       // XS x 32 KiB (1024-aligned)
    uint8_t *a0 = x0 + XS * X_BYTES;          // XS x 16 KiB (1024-aligned)
    uint8_t *y0 = a0 + XS * A_BYTES;          // 4 x 2 KiB (1024-aligned)
    uint8_t *w0 = y0 + Y_BUF_BYTES;           // WS x 4 KiB
    uint64_t *bars = reinterpret_cast<uint64_t *>(w0 + WS * W_BYTES);
    // full[s] (first CTA): stage s's token bytes of both CTAs landed and its A tile is
    // decoded in both CTAs; empty[s]: the stage's MMAs completed
    uint64_t *full = bars, *empty = full + XS;
    uint64_t *wfull = empty + XS, *wempty = wfull + WS;
    uint64_t *accfull = wempty + WS, *accempty = accfull + 1, *drain = accempty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    float *lv_s = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + BAR_BYTES);
    float *c2 = lv_s + 16;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool first = rank == 0;
    const int cluster = int(cluster_id_x()), nclusters = int(n_clusters_x());
    const int nkw = int((p.C + BK - 1) / BK);  // weight steps (dX: a ragged last step is zero-filled)
    const int nk = nkw + p.lora_chunks;
    const int ntiles = p.m_tiles * p.t_tiles;
    const int my_tiles = ntiles > cluster ? (ntiles - cluster + nclusters - 1) / nclusters : 0;
    // pair tile of this cluster's tl-th turn: output columns from m * 256, tokens from t0
    auto tile_of = [&](int tl, int &m, int64_t &t0, int &ntok) {
        const int tile = cluster + tl * nclusters;
        m = tile % p.m_tiles;
        t0 = int64_t(tile / p.m_tiles) * BN;
        ntok = int(p.T - t0 < BN ? p.T - t0 : BN);
    };

    if (threadIdx.x == 0) {
        for (int i = 0; i < XS; ++i) {
            mbar_init(&full[i], 1 + 2 * 4);  // the first producer's expect-tx + the owning decode warps of both CTAs
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < WS; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&wempty[i], 4);  // the owning group's four warps
        }
        mbar_init(accfull, 1);
        mbar_init(accempty, 2 * EPI_WARPS);  // both CTAs' epilogue warps
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 16) lv_s[threadIdx.x] = p.code16[threadIdx.x];
    if (DQ) {
        for (int i = threadIdx.x; i < 256; i += NUM_THREADS) c2[i] = p.w.code2[i];
    }
    cluster_sync();  // both CTAs' barriers exist before any remote arrival or TMA completion
    if (warp == 1) tmem_alloc_pair(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the first CTA's full[0] / accempty as shared::cluster addresses (8 bytes per stage)
    const uint32_t full_c = mapa_shared(full, 0);
    const uint32_t accempty_c = mapa_shared(accempty, 0);

    if (warp == 0) {
        // ------------------ producer: this CTA's token halves (and the LoRA chunks)
        if (lane == 0) {
            prefetch_tensormap(&tm_x);
            if (p.lora_chunks) prefetch_tensormap(&tm_xl);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                int m, ntok;
                int64_t t0;
                tile_of(tl, m, t0, ntok);
                const bool two = ntok > NH;  // the tile has a second MMA
                const int ta = int(t0) + int(rank) * CT, tb = ta + NH;
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % XS;
                    if (!mbar_wait(&empty[s], ((it / XS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrPairOffset)) {
                        ok = false;
                        break;
                    }
                    if (first) mbar_arrive_expect_tx(&full[s], uint32_t((two ? 2 : 1) * 2 * X_HALF));  // both CTAs
                    const CUtensorMap *map = ks < nkw ? &tm_x : &tm_xl;
                    const int kc = (ks < nkw ? ks : ks - nkw) * BK;
                    // zero-filled past the last token (and, for dX, past the last row of W)
                    tma_load_2d_pair(x0 + s * X_BYTES, map, kc, ta, full_c + 8u * uint32_t(s));
                    if (two) tma_load_2d_pair(x0 + s * X_BYTES + X_HALF, map, kc, tb, full_c + 8u * uint32_t(s));
                }
            }
            if (first)  // the pair's copies land before either CTA exits
                for (uint32_t j = (it > XS ? it - XS : 0); j < it; ++j)
                    mbar_wait_issued(&full[j % XS], (j / XS) & 1, p.status, kErrTimeoutTeardown + kErrPairOffset);
            // the MMAs' last completion signals (multicast commits into both CTAs' shared memory)
            // land before the CTA exits: an arrival still in flight would hit the
            // shared memory of whichever CTA runs on this SM next
            if (ok)
                for (uint32_t j = (it > XS ? it - XS : 0); j < it; ++j)
                    mbar_wait(&empty[j % XS], (j / XS) & 1, p.status, kErrTimeoutTeardown + kErrPairOffset);
        }
    } else if (warp == 2) {
        // ------------------------------ producer: this CTA's packed weight tiles
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            if (TWO_W) prefetch_tensormap(&tm_w2);
            uint32_t wt = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                int m, ntok;
                int64_t t0;
                tile_of(tl, m, t0, ntok);
                const int c0 = m * (2 * BM) + int(rank) * BM;  // this CTA's first output column
                for (int ks = 0; ks < nkw; ++ks, ++wt) {
                    const int s = wt % WS;
                    if (!mbar_wait(&wempty[s], ((wt / WS) & 1) ^ 1, p.status, kErrTimeoutProducer + kErrPairOffset)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&wfull[s], W_BYTES);
                    if constexpr (DX) {  // 64 weight rows x 128 columns (64 bytes)
                        if (TWO_W && ks >= p.nkw0)
                            tma_load_2d(w0 + s * W_BYTES, &tm_w2, c0 / 2, (ks - p.nkw0) * BK, &wfull[s]);
                        else
                            tma_load_2d(w0 + s * W_BYTES, &tm_w, c0 / 2, ks * BK, &wfull[s]);
                    } else {  // 128 weight rows x 64 columns (32 bytes)
                        tma_load_2d(w0 + s * W_BYTES, &tm_w, ks * (BK / 2), c0, &wfull[s]);
                    }
                }
            }
            for (uint32_t j = (wt > WS ? wt - WS : 0); j < wt; ++j)
                mbar_wait_issued(&wfull[j % WS], (j / WS) & 1, p.status, kErrTimeoutTeardown + kErrPairOffset);
        }
    } else if (warp == 1) {
        // ------------------------------------ MMA issuer (first CTA of the pair)
        if (lane == 0 && first) {
            constexpr uint32_t idesc = DX ? idesc_f16_amn(BF16, 2 * BM, NH) : idesc_f16(BF16, 2 * BM, NH);
            uint32_t it = 0;
            bool ok = true;
            for (int tl = 0; ok && tl < my_tiles; ++tl) {
                int m, ntok;
                int64_t t0;
                tile_of(tl, m, t0, ntok);
                const bool two = ntok > NH;
                if (!mbar_wait(accempty, (tl & 1) ^ 1, p.status, kErrTimeoutMma + kErrPairOffset)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int ks = 0; ks < nk; ++ks, ++it) {
                    const int s = it % XS;
                    if (!mbar_wait(&full[s], (it / XS) & 1, p.status, kErrTimeoutMma + kErrPairOffset)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // 16 contraction rows per MMA: 32 bytes along a K-major row, or two
                    // 8-row groups (2 KiB) of the MN-major atoms
                    const uint64_t ad = DX ? smem_desc_mn_sw128(a0 + s * A_BYTES, A_ATOM, 1024)
                                           : smem_desc_k_sw128(a0 + s * A_BYTES);
                    constexpr uint64_t a_step = DX ? (2048 >> 4) : 2;
                    const uint64_t bd = smem_desc_k_sw128(x0 + s * X_BYTES);
#pragma unroll
                    for (int j = 0; j < BK / 16; ++j) {
                        mma_ss_f16_pair(tmem, ad + j * a_step, bd + uint64_t(j * 2), idesc, (ks | j) != 0);
                        if (two)
                            mma_ss_f16_pair(tmem + NH, ad + j * a_step, bd + uint64_t((X_HALF >> 4) + j * 2), idesc,
                                            (ks | j) != 0);
                    }
                    mma_commit_pair(&empty[s], 0x3);
                }
                if (ok) mma_commit_pair(accfull, 0x3);
            }
            mma_commit_pair(drain, 0x3);  // every MMA done before either CTA frees TMEM
        }
    } else if (dq_index(warp) >= 0) {
        // ------------------------------------------ decode warps (both CTAs)
        const int di = dq_index(warp);
        const int grp = di >> 2;
        const int tid = (di & 3) * 32 + lane;  // this thread's 128-byte row of the A tile
        // forward: weight row tid of the CTA's 128; dX: weight row rl of the step over
        // the 64 columns of block kb of the CTA's 128
        const int rl = tid & 63, kb = tid >> 6;
        // A position in this group's walk over (tile turn tl, step ks): advanced
        // by DQG steps at a time with no division in the loop (one per tile change)
        struct Pos {
            int tl, ks;
            int64_t c0;  // this CTA's first output column in tile turn tl
        };
        auto set_tile = [&](Pos &q) {
            const int tile = cluster + q.tl * nclusters;
            q.c0 = int64_t(tile % p.m_tiles) * (2 * BM) + int64_t(rank) * BM;
        };
        auto advance = [&](Pos &q) {
            q.ks += DQG;
            if (q.ks >= nk) {
                while (q.ks >= nk) {
                    q.ks -= nk;
                    ++q.tl;
                }
                if (q.tl < my_tiles) set_tile(q);
            }
        };
        // (weight row, NF4 block) this thread decodes at q (the row may be past the weight)
        auto block_at = [&](const Pos &q, int64_t &wrow, int64_t &blk) {
            if constexpr (DX) {
                wrow = int64_t(q.ks) * BK + rl;
                blk = q.c0 / 64 + kb;
            } else {
                wrow = q.c0 + tid;
                blk = q.ks;
            }
        };
        auto absmax_at = [&](const Pos &q) -> float {
            if (q.tl >= my_tiles || q.ks >= nkw) return 0.f;
            int64_t wrow, blk;
            block_at(q, wrow, blk);
            if constexpr (DX) {
                if (wrow >= p.C || blk >= p.kbl) return 0.f;
                if (TWO_W && q.ks >= p.nkw0)  // the second weight's code2 table is read from global memory
                    return block_scale<DQ>(p.w1, p.w1.code2, (wrow - int64_t(p.nkw0) * BK) * p.kbl + blk);
            } else {
                if (wrow >= p.M) return 0.f;
            }
            return block_scale<DQ>(p.w, c2, wrow * p.kbl + blk);
        };
        const int arow = (tid >> 3) * 1024 + (tid & 7) * 128;
        Pos cur{0, grp - DQG, 0};
        advance(cur);  // normalises (tiles with fewer steps than the groups)
        if (cur.tl < my_tiles) set_tile(cur);
        Pos nxt = cur;
        advance(nxt);
        float am_next = absmax_at(cur);
        uint32_t it = uint32_t(cur.tl) * uint32_t(nk) + uint32_t(cur.ks);
        for (; cur.tl < my_tiles; it += DQG, cur = nxt, advance(nxt)) {
            const float am = am_next;
            am_next = absmax_at(nxt);  // one owned step ahead
            int64_t wrow, blk;
            block_at(cur, wrow, blk);
            const int ks = cur.ks, tl = cur.tl;
            uint32_t vals[32];
            if (ks < nkw) {
                const uint32_t wt = uint32_t(tl) * uint32_t(nkw) + uint32_t(ks);
                const int s = wt % WS;
                if (!__all_sync(0xffffffffu, mbar_wait(&wfull[s], (wt / WS) & 1, p.status, kErrTimeoutDequant + kErrPairOffset)))
                    break;
                uint4 p0, p1;
                if constexpr (DX) {
                    // 64-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ ((r >> 1) & 3)
                    const uint4 *src = reinterpret_cast<const uint4 *>(w0 + s * W_BYTES + rl * 64);
                    const int sw = (rl >> 1) & 3;
                    p0 = src[(2 * kb) ^ sw];
                    p1 = src[(2 * kb + 1) ^ sw];
                } else {
                    // 32-byte swizzle: row r's 16-byte halves are swapped when bit 2 of r is set
                    const uint4 *src = reinterpret_cast<const uint4 *>(w0 + s * W_BYTES + tid * 32);
                    const int sw = (tid >> 2) & 1;
                    p0 = src[sw];
                    p1 = src[sw ^ 1];
                }
                const uint32_t w[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
                const Nf4Tables t = nf4_build_tables<BF16>(lv_s, am);  // levels read from shared memory
                nf4_decode_block(t, w, vals);
                // release the packed tile once every lane has read it; order these
                // generic-proxy reads before the TMA refill of the slot
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&wempty[s]);
            } else if constexpr (DX) {
                // LoRA chunk: rank row j of lora_A, 64 columns (zero beyond r / the weight's K)
                const int j = (ks - nkw) * BK + rl;
                const bool ok_row = j < p.r && blk < p.kbl;
                const uint4 *src = reinterpret_cast<const uint4 *>(p.lora + int64_t(j) * p.M + blk * 64);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 v = ok_row ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
                    vals[4 * c] = v.x;
                    vals[4 * c + 1] = v.y;
                    vals[4 * c + 2] = v.z;
                    vals[4 * c + 3] = v.w;
                }
            } else {
                // LoRA chunk: lora_b row wrow, rank columns j0 .. j0 + 63 (zero beyond r / N)
                const int j0 = (ks - nkw) * BK;
                const bool valid = wrow < p.M;
#pragma unroll
                for (int m = 0; m < 32; ++m) {
                    const int j = j0 + 2 * m;
                    vals[m] = (valid && j < p.r) ? __ldg(reinterpret_cast<const uint32_t *>(p.lora + wrow * p.r + j))
                                                 : 0u;
                }
            }
            const int sa = it % XS;
            if (!__all_sync(0xffffffffu, mbar_wait(&empty[sa], ((it / XS) & 1) ^ 1, p.status, kErrTimeoutDequant + kErrPairOffset)))
                break;
            uint8_t *dst = a0 + sa * A_BYTES + arow;
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4 *>(dst + ((c ^ (tid & 7)) << 4)) =
                    make_uint4(vals[4 * c], vals[4 * c + 1], vals[4 * c + 2], vals[4 * c + 3]);
            fence_proxy_async_smem();  // generic-proxy writes -> visible to the pair's tcgen05.mma
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(full_c + 8u * uint32_t(sa));
        }
    } else if (warp >= EPI_WARP0) {
        // -------------------------------------------------- epilogue (both CTAs)
        const int q = warp & 3;
        const int ew = warp - EPI_WARP0;
        const int tok_lo = (ew >> 2) * PART_TOK;  // this warp's tokens of a tile: [tok_lo, tok_lo + PART_TOK)
        const uint32_t lane_addr = uint32_t(q * 32) << 16;
        // this thread's stmatrix row: matrix k = lane/8, row j = lane%8
        const int kq = lane >> 3, jr = lane & 7;
        const int tok_in = jr + 8 * (kq >> 1);  // token offset within a 16-column block
        auto release = [&]() {                   // this warp's accumulator reads are done
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(accempty_c);
        };
        for (int tl = 0; tl < my_tiles; ++tl) {
            if (!__all_sync(0xffffffffu, mbar_wait(accfull, tl & 1, p.status, kErrTimeoutEpilogue + kErrPairOffset))) break;
            tc_fence_after();
            int m, ntok;
            int64_t t0;
            tile_of(tl, m, t0, ntok);
            const int64_t n0 = int64_t(m) * (2 * BM) + int64_t(rank) * BM;
            if (p.tma_store) {
                // Each warp stages its own 32 output columns: TMEM -> registers as
                // 16x256b fragments, + bias, -> 16-bit -> stmatrix.trans into a [token][32]
                // chunk of 64 tokens (64-byte rows, 64B swizzle), then its own TMA store;
                // two buffers per warp alternate, so no warp waits for another
                float bias[2][2];
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int64_t n = n0 + q * 32 + h * 16 + (lane >> 2) + 8 * e;
                        bias[h][e] = (p.bias && n < p.M) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
                    }
                const int64_t nw = n0 + q * 32;  // this warp's first output column
                // 16-token blocks: block b's TMEM load is in flight while block b - 1 is
                // converted and staged (one wait covers all loads issued, so two register
                // buffers alternate).  A 32-token chunk (two blocks) is transposed through
                // this warp's 2 KiB of shared memory and written with 16-byte global
                // stores, which need no completion wait before the buffer is reused.
                const int ptok = ntok - tok_lo < PART_TOK ? ntok - tok_lo : PART_TOK;  // may be <= 0
                const int nblk = ptok > 0 ? (ptok + 15) >> 4 : 0;
                uint8_t *yb = y0 + ew * YW_BYTES;
                uint32_t va[2][8], vb[2][8];
                auto ld = [&](int blk, uint32_t (&v)[2][8]) {
                    const uint32_t col = uint32_t(tok_lo + blk * 16);
                    tmem_ld_16x256b_x2(tmem + lane_addr + col, v[0]);
                    tmem_ld_16x256b_x2(tmem + lane_addr + (16u << 16) + col, v[1]);
                };
                auto stage = [&](int blk, const uint32_t (&v)[2][8]) {
                    const int tok = (blk & 1) * 16 + tok_in;  // token row of the 32-token chunk
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t x4[4];
#pragma unroll
                        for (int mm = 0; mm < 4; ++mm) {
                            const float bb = bias[h][mm & 1];
                            const float lo = __uint_as_float(v[h][2 * mm]) + bb;
                            const float hi = __uint_as_float(v[h][2 * mm + 1]) + bb;
                            x4[mm] = BF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
                        }
                        // registers {0,1}: columns +0, tokens +0..7; {2,3}: columns +8; {4,5}/{6,7}: tokens +8;
                        // 16-byte chunk (kq & 1) + 2h of the token's 64-byte row, 64B swizzle
                        const int cw = (kq & 1) + 2 * h;
                        const uint8_t *dst = yb + tok * 64 + ((cw ^ ((tok >> 1) & 3)) << 4);
                        stmatrix_x4_trans(smem_u32(dst), x4[0], x4[1], x4[2], x4[3]);
                    }
                };
                auto flush = [&](int b0) {  // the staged chunk -> y (tokens from t0 + 16 b0)
                    __syncwarp();
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int piece = lane + 32 * r;  // 128 pieces of 16 bytes: 4 per token row
                        const int tok = piece >> 2, cw = piece & 3;
                        const uint4 v4 = *reinterpret_cast<const uint4 *>(yb + tok * 64 + ((cw ^ ((tok >> 1) & 3)) << 4));
                        const int64_t t = t0 + tok_lo + b0 * 16 + tok, n = nw + cw * 8;
                        if (t < p.T && n < p.M) *reinterpret_cast<uint4 *>(p.y + t * p.M + n) = v4;
                    }
                    __syncwarp();  // every lane has read the chunk before it is overwritten
                };
                if (nblk == 0) {
                    release();
                    continue;
                }
                ld(0, va);
                tmem_ld_wait();
                if (nblk == 1) release();  // the next tile may start
#pragma unroll 1
                for (int b0 = 0; b0 < nblk; b0 += 2) {
                    const bool has1 = b0 + 1 < nblk, has2 = b0 + 2 < nblk;  // warp-uniform
                    if (has1) ld(b0 + 1, vb);
                    stage(b0, va);
                    if (has1) {
                        tmem_ld_wait();
                        if (b0 + 2 >= nblk) release();
                    }
                    if (has2) ld(b0 + 2, va);
                    if (has1) stage(b0 + 1, vb);
                    flush(b0);
                    if (has2) {
                        tmem_ld_wait();
                        if (b0 + 3 >= nblk) release();
                    }
                }
            } else {
                // generic path (columns % 8 != 0 or unaligned output): element stores
                const int64_t n = n0 + q * 32 + lane;
                const float bias = (n < p.M && p.bias) ? load_bias(p.bias, p.bias_dtype, n) : 0.f;
                const int ptok = ntok - tok_lo < PART_TOK ? ntok - tok_lo : PART_TOK;  // may be <= 0
                const int nblk = ptok > 0 ? (ptok + 31) >> 5 : 0;
                if (nblk == 0) release();
#pragma unroll 1
                for (int c = 0; c < nblk; ++c) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem + lane_addr + tok_lo + c * 32, v);
                    tmem_ld_wait();
                    if (c == nblk - 1) release();
                    if (n < p.M) {
                        const int64_t tcb = t0 + tok_lo + c * 32;
                        for (int i = 0; i < 32 && tcb + i < p.T; ++i)
                            p.y[(tcb + i) * p.M + n] = to16<BF16>(__uint_as_float(v[i]) + bias);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1 && lane == 0) {  // the pair's MMAs into this CTA's TMEM are complete
        mbar_wait_issued(drain, 0, p.status, kErrTimeoutTeardown + kErrPairOffset);
        // the second CTA's epilogue releases of the last accumulator (remote arrivals
        // on this CTA's barrier) have landed before this CTA's shared memory is reused
        if (first && my_tiles > 0)
            mbar_wait(accempty, (my_tiles & 1) ^ 1, p.status, kErrTimeoutTeardown + kErrPairOffset);
    }
    __syncwarp();
    cluster_sync();  // neither CTA leaves while the peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
    // the pair's TMEM is released on both SMs before either CTA exits and its SM
    // takes the next CTA (the 2-SM deallocation spans both)
    cluster_sync();
}

}  // namespace pair


// ------------------------------------------------------- wait self-test --

// One warp: lane 0 waits on an mbarrier that nothing arrives on, through the same
// bounded wait as the GEMMs, so the wait gives up after the limit in force and
// writes kErrWaitSelfTest and its record to the status word; the kernel then
// returns.  The barrier sits inside zeroed words, as the record's snapshot
// expects shared memory on both sides of a waited barrier.
__global__ void __launch_bounds__(32) k_wait_selftest(int *status) {
    __shared__ __align__(8) uint64_t bars[sm100::kBarSnap];
    if (threadIdx.x < sm100::kBarSnap) bars[threadIdx.x] = 0;
    __syncwarp();
    if (threadIdx.x == 0) {
        sm100::mbar_init(&bars[sm100::kBarBelow], 1);
        sm100::fence_barrier_init();
        sm100::mbar_wait(&bars[sm100::kBarBelow], 0, status, sm100::kErrWaitSelfTest);
    }
    __syncwarp();
}

// ------------------------------------------------------------------- host --

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

int make_map_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
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

// Device address of g_gemm_status on the current device, resolved on the
// device's first call and cached (atomics: racing first calls store the same value).
int *status_ptr() {
    static std::atomic<int *> ptrs[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    int *cached = ptrs[dev].load(std::memory_order_acquire);
    if (!cached) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_gemm_status) != cudaSuccess) return nullptr;
        cached = static_cast<int *>(p);
        ptrs[dev].store(cached, std::memory_order_release);
    }
    return cached;
}

// Tokens per forward tile.  384 (two MMAs per K slice) decodes each weight tile
// for 1.5x the tokens of 256 and runs ~3-8% faster per FLOP on large GEMMs; 192
// (one MMA) halves the work per tile, which wins when the GEMM has too few tiles
// to fill the GPU.  Pick the one with the shorter estimated makespan (waves x
// tile length); the narrow tile is charged 1.4x per token, its measured cost on
// B200 (twice the decode work per FLOP).
int fwd_tile_tokens(int64_t T, int n_tiles) {
    const int64_t sms = sm_count();
    auto est = [&](int64_t tt, double slow) {
        const int64_t tiles = int64_t(n_tiles) * ((T + tt - 1) / tt);
        return double((tiles + sms - 1) / sms) * double(tt) * slow;
    };
    return est(BNH, 1.4) < est(BN, 1.0) ? BNH : BN;
}

template <bool BF16, bool DQ, bool SWIGLU>
int launch_fwd(const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mw2, const CUtensorMap &mxa,
               const CUtensorMap &my, const FwdParams &p, cudaStream_t st) {
    auto kern = k_nf4_gemm_fwd<BF16, DQ, SWIGLU>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) != cudaSuccess)
            return fail(STRATUM_ERR_CUDA, "nf4_gemm_fwd: cannot set %d bytes of shared memory", SMEM_BYTES);
        attr_set[dev] = true;
    }
    const int ntiles = p.n_tiles * p.t_tiles;
    const int grid = ntiles < sm_count() ? ntiles : sm_count();
    kern<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(mx, mw, mw2, mxa, my, p);
    return check_launch(SWIGLU ? "nf4_gemm_swiglu_fwd" : "nf4_gemm_fwd");
}

// CTA pairs of a 2-SM GEMM that fit on the device at once; sets the kernel's
// shared-memory attribute first (0 on failure).
template <typename Kern>
int pair_count_query(Kern kern) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pair::SMEM_BYTES) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(sm_count()), 1, 1);
    cfg.blockDim = dim3(pair::NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = pair::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = sm_count() / 2;
    }
    return n;
}

template <bool BF16, bool DQ, bool DX, bool TWO_W>
int launch_pair(const CUtensorMap &mx, const CUtensorMap &mw, const CUtensorMap &mw2, const CUtensorMap &mxl,
                const CUtensorMap &my, const pair::Params &p, cudaStream_t st, const char *what) {
    auto kern = pair::k_nf4_gemm_pair<BF16, DQ, DX, TWO_W>;
    static std::atomic<int> cached[64];  // per instantiation and device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return fail(STRATUM_ERR_CUDA, "%s: device %d out of range", what, dev);
    int pairs = cached[dev].load(std::memory_order_acquire);
    if (pairs <= 0) {
        pairs = pair_count_query(kern);
        if (pairs <= 0) return fail(STRATUM_ERR_CUDA, "%s: cannot set %d bytes of shared memory", what, pair::SMEM_BYTES);
        cached[dev].store(pairs, std::memory_order_release);
    }
    const int ntiles = p.m_tiles * p.t_tiles;
    const int grid = 2 * (ntiles < pairs ? ntiles : pairs);
    kern<<<grid, pair::NUM_THREADS, pair::SMEM_BYTES, st>>>(mx, mw, mw2, mxl, my, p);
    return check_launch(what);
}

// GEMM kernel selection: STRATUM_GEMM_AUTO, _PAIR or _SINGLE (set by
// stratum_nf4_gemm_set_kernel; initially from STRATUM_NF4_GEMM=pair|single).
std::atomic<int> g_gemm_kernel{-1};

int gemm_kernel_setting() {
    int v = g_gemm_kernel.load(std::memory_order_relaxed);
    if (v >= 0) return v;
    const char *e = getenv("STRATUM_NF4_GEMM");
    v = STRATUM_GEMM_AUTO;
    if (e && !strcmp(e, "pair")) v = STRATUM_GEMM_PAIR;
    if (e && !strcmp(e, "single")) v = STRATUM_GEMM_SINGLE;
    int expected = -1;
    g_gemm_kernel.compare_exchange_strong(expected, v);
    return g_gemm_kernel.load(std::memory_order_relaxed);
}

// Whether the CTA-pair kernel runs a GEMM of T tokens and M output columns: by
// estimated makespan.  A pair tile is 512 tokens x 256 columns on two SMs (512 x
// 128 per SM); the single-CTA tile is `tile_tokens` x 128 at relative cost
// `single_cost` per token-column, the pair tile kPairCost, in units of the
// single-CTA forward's 384-token tile (fitted to B200 measurements over T = 1024
// .. 8192 and 2048 .. 14336-wide weights: the one-SM forward's 192-token tile
// costs 1.4, the one-SM input gradient's 256-token tile 1.28).
constexpr double kPairCost = 0.93;
bool use_pair(int64_t T, int64_t M, int tile_tokens, double single_cost) {
    const int forced = gemm_kernel_setting();
    if (forced != STRATUM_GEMM_AUTO) return forced == STRATUM_GEMM_PAIR;
    const int64_t sms = sm_count(), pairs = sms / 2;
    const int64_t tiles1 = ((M + BM - 1) / BM) * ((T + tile_tokens - 1) / tile_tokens);
    const int64_t tiles2 = ((M + 2 * pair::BM - 1) / (2 * pair::BM)) * ((T + pair::BN - 1) / pair::BN);
    const double t1 = double((tiles1 + sms - 1) / sms) * tile_tokens * single_cost;
    const double t2 = double((tiles2 + pairs - 1) / pairs) * pair::BN * kPairCost;
    return t2 < t1;
}

template <bool BF16, bool DQ, bool PAIR>
int launch_dx(const CUtensorMap &mdy, const CUtensorMap &mw, const CUtensorMap &mw2, const CUtensorMap &mdyb,
              const CUtensorMap &mdx, const dx::Params &p, cudaStream_t st) {
    auto kern = dx::k_nf4_gemm_dx<BF16, DQ, PAIR>;
    static bool attr_set[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dx::SMEM_BYTES) != cudaSuccess)
            return fail(STRATUM_ERR_CUDA, "nf4_gemm_dx: cannot set %d bytes of shared memory", dx::SMEM_BYTES);
        attr_set[dev] = true;
    }
    const int ntiles = p.k_tiles * p.t_tiles;
    const int grid = ntiles < sm_count() ? ntiles : sm_count();
    kern<<<grid, dx::NUM_THREADS, dx::SMEM_BYTES, st>>>(mdy, mw, mw2, mdyb, mdx, p);
    return check_launch(PAIR ? "nf4_gemm_dx_pair" : "nf4_gemm_dx");
}

// Shared set-up of the input-gradient entry points: validation, tensor maps,
// parameters and the launch.  w1 != NULL: PAIR (w0's N0 rows, then w1's N - N0).
int dx_run(const void *dy, int dtype, int64_t T, int64_t N, const stratum_nf4_weight &w0, const stratum_nf4_weight *w1,
           int64_t N0, const float *code16, int64_t K, const void *lora_dyb, const void *lora_a, int r, void *dx_out,
           void *stream, const char *what) {
    const bool pair = w1 != nullptr;
    STRATUM_REQUIRE(T >= 0 && N >= 0 && K >= 0, "%s: negative size", what);
    if (T == 0 || K == 0) return STRATUM_OK;
    STRATUM_REQUIRE(dy && w0.packed && code16 && dx_out && (!pair || w1->packed), "%s: null pointer", what);
    if (dtype != STRATUM_BF16 && dtype != STRATUM_F16) return fail(STRATUM_ERR_UNSUPPORTED, "%s: dy must be bf16 or fp16", what);
    if (K % 64 != 0) return fail(STRATUM_ERR_UNSUPPORTED, "%s: K=%lld must be a multiple of 64", what, (long long)K);
    if (N % 8 != 0 || N == 0)
        return fail(STRATUM_ERR_UNSUPPORTED, "%s: N=%lld must be a positive multiple of 8", what, (long long)N);
    const bool dq = w0.absmax == nullptr;
    STRATUM_REQUIRE(!dq || (w0.absmax_q && w0.absmax2 && w0.code2 && w0.offset), "%s: need absmax or the double-quant "
                                                                                 "set", what);
    if (pair) {
        STRATUM_REQUIRE((w1->absmax == nullptr) == dq, "%s: both weights must be plain or both double quantized", what);
        STRATUM_REQUIRE(!dq || (w1->absmax_q && w1->absmax2 && w1->offset && w1->code2),
                        "%s: the second weight needs its double-quant set", what);
    }
    STRATUM_REQUIRE(r >= 0 && r <= 256, "%s: lora rank %d out of range", what, r);
    STRATUM_REQUIRE(r == 0 || (lora_dyb && lora_a), "%s: lora needs dyb and A", what);
    auto a16 = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    STRATUM_REQUIRE(a16(dy) && a16(w0.packed) && (!pair || a16(w1->packed)) && (r == 0 || a16(lora_a)),
                    "%s: dy, packed and lora_A must be 16-byte aligned", what);
    STRATUM_BIND_STREAM(stream);
    int *status = status_ptr();
    if (!status) return fail(STRATUM_ERR_CUDA, "%s: no status word", what);
    const bool bf16 = dtype == STRATUM_BF16;
    const CUtensorMapDataType xdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap mdy, mw, mw2, mdyb, mdx;
    int rc = make_map_2d(&mdy, xdt, dy, uint64_t(N), uint64_t(T), uint64_t(N) * 2, dx::BK, dx::BN,
                         CU_TENSOR_MAP_SWIZZLE_128B, what);
    if (rc) return rc;
    // packed W viewed as [rows][K/2 bytes]; box 64 bytes (128 columns) x 64 rows, 64-byte swizzle
    const int64_t rows0 = pair ? N0 : N;
    rc = make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w0.packed, uint64_t(K / 2), uint64_t(rows0), uint64_t(K / 2),
                     64, dx::BK, CU_TENSOR_MAP_SWIZZLE_64B, what);
    if (rc) return rc;
    mw2 = mw;
    if (pair) {
        rc = make_map_2d(&mw2, CU_TENSOR_MAP_DATA_TYPE_UINT8, w1->packed, uint64_t(K / 2), uint64_t(N - N0),
                         uint64_t(K / 2), 64, dx::BK, CU_TENSOR_MAP_SWIZZLE_64B, what);
        if (rc) return rc;
    }
    const int lora_chunks = (r + 63) / 64;
    if (r > 0) {
        STRATUM_REQUIRE(a16(lora_dyb), "%s: dyb must be 16-byte aligned", what);
        rc = make_map_2d(&mdyb, xdt, lora_dyb, uint64_t(lora_chunks * 64), uint64_t(T), uint64_t(lora_chunks * 64) * 2,
                         64, dx::BN, CU_TENSOR_MAP_SWIZZLE_128B, what);
        if (rc) return rc;
    } else {
        mdyb = mdy;
    }
    dx::Params p{};
    p.w = WeightScales{w0.absmax, w0.absmax_q, w0.absmax2, w0.code2, w0.offset};
    if (pair) p.w1 = WeightScales{w1->absmax, w1->absmax_q, w1->absmax2, w1->code2, w1->offset};
    p.code16 = code16;
    p.lora_a = static_cast<const uint16_t *>(lora_a);
    p.r = r;
    p.lora_chunks = lora_chunks;
    p.dx = static_cast<uint16_t *>(dx_out);
    p.T = T; p.N = N; p.K = K;
    p.nkw0 = pair ? int(N0 / dx::BK) : 0;
    p.k_tiles = int((K + dx::BM - 1) / dx::BM);
    p.t_tiles = int((T + dx::BN - 1) / dx::BN);
    p.status = status;
    p.tma_store = a16(dx_out);
    mdx = mdy;
    if (p.tma_store) {
        rc = make_map_2d(&mdx, xdt, dx_out, uint64_t(K), uint64_t(T), uint64_t(K) * 2, 64, dx::BN,
                         CU_TENSOR_MAP_SWIZZLE_128B, what);
        if (rc) return rc;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (use_pair(T, K, dx::BN, 1.28)) {
        // CTA-pair kernel: 512-token x 256-column tiles, each CTA stages 128-token boxes
        pair::Params q{};
        q.w = p.w;
        q.w1 = p.w1;
        q.code16 = code16;
        q.lora = p.lora_a;
        q.r = r;
        q.lora_chunks = lora_chunks;
        q.y = p.dx;
        q.T = T;
        q.M = K;
        q.C = N;
        q.kbl = K / 64;
        q.nkw0 = p.nkw0;
        q.m_tiles = int((K + 2 * pair::BM - 1) / (2 * pair::BM));
        q.t_tiles = int((T + pair::BN - 1) / pair::BN);
        q.tma_store = p.tma_store;
        q.status = status;
        rc = make_map_2d(&mdy, xdt, dy, uint64_t(N), uint64_t(T), uint64_t(N) * 2, pair::BK, pair::CT,
                         CU_TENSOR_MAP_SWIZZLE_128B, what);
        if (rc) return rc;
        if (r > 0) {
            rc = make_map_2d(&mdyb, xdt, lora_dyb, uint64_t(lora_chunks * 64), uint64_t(T),
                             uint64_t(lora_chunks * 64) * 2, 64, pair::CT, CU_TENSOR_MAP_SWIZZLE_128B, what);
            if (rc) return rc;
        } else {
            mdyb = mdy;
        }
        mdx = mdy;  // dx is written with 16-byte stores (q.tma_store: 16-byte aligned)
#define STRATUM_DX2(B, D)                                                                  \
    (pair ? launch_pair<B, D, true, true>(mdy, mw, mw2, mdyb, mdx, q, st, what)           \
          : launch_pair<B, D, true, false>(mdy, mw, mw2, mdyb, mdx, q, st, what))
        if (bf16) return dq ? STRATUM_DX2(true, true) : STRATUM_DX2(true, false);
        return dq ? STRATUM_DX2(false, true) : STRATUM_DX2(false, false);
#undef STRATUM_DX2
    }
#define STRATUM_DX(B, D) \
    (pair ? launch_dx<B, D, true>(mdy, mw, mw2, mdyb, mdx, p, st) : launch_dx<B, D, false>(mdy, mw, mw2, mdyb, mdx, p, st))
    if (bf16) return dq ? STRATUM_DX(true, true) : STRATUM_DX(true, false);
    return dq ? STRATUM_DX(false, true) : STRATUM_DX(false, false);
#undef STRATUM_DX
}

}  // namespace gemm
}  // namespace stratum

using namespace stratum;

extern "C" {

int stratum_device_status(int *out, int reset, void *stream) {
    STRATUM_REQUIRE(out != nullptr, "device_status: null out");
    STRATUM_BIND_STREAM(stream);
    int *dp = gemm::status_ptr();
    if (!dp) return fail(STRATUM_ERR_CUDA, "device_status: cannot resolve the status word");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(out, dp, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(STRATUM_ERR_CUDA, "device_status: copy failed: %s", cudaGetErrorString(cudaGetLastError()));
    if (reset && *out != 0) {
        if (cudaMemsetAsync(dp, 0, sm100::kStatusWords * sizeof(int), st) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            return fail(STRATUM_ERR_CUDA, "device_status: reset failed");
    }
    return STRATUM_OK;
}

int stratum_device_status_detail(int *out8, void *stream) {
    STRATUM_REQUIRE(out8 != nullptr, "device_status_detail: null out");
    STRATUM_BIND_STREAM(stream);
    int *dp = gemm::status_ptr();
    if (!dp) return fail(STRATUM_ERR_CUDA, "device_status_detail: cannot resolve the status word");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(out8, dp, 8 * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(STRATUM_ERR_CUDA, "device_status_detail: copy failed: %s", cudaGetErrorString(cudaGetLastError()));
    return STRATUM_OK;
}

int stratum_device_status_record(int *out, int n, void *stream) {
    STRATUM_REQUIRE(out != nullptr && n > 0, "device_status_record: null out or n <= 0");
    STRATUM_BIND_STREAM(stream);
    int *dp = gemm::status_ptr();
    if (!dp) return fail(STRATUM_ERR_CUDA, "device_status_record: cannot resolve the status word");
    const int m = n < sm100::kStatusWords ? n : sm100::kStatusWords;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(out, dp, size_t(m) * sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(STRATUM_ERR_CUDA, "device_status_record: copy failed: %s", cudaGetErrorString(cudaGetLastError()));
    for (int i = m; i < n; ++i) out[i] = 0;
    return STRATUM_OK;
}

int stratum_set_wait_limit_ns(uint64_t ns, void *stream) {
    STRATUM_REQUIRE(ns == 0 || (ns >= 1000000ull && ns <= 60000000000ull),
                    "set_wait_limit_ns: %llu ns outside [1 ms, 60 s] (0 restores the default)",
                    (unsigned long long)ns);
    STRATUM_BIND_STREAM(stream);
    int *dp = gemm::status_ptr();
    if (!dp) return fail(STRATUM_ERR_CUDA, "set_wait_limit_ns: cannot resolve the status word");
    const uint32_t words[2] = {uint32_t(ns), uint32_t(ns >> 32)};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(dp + sm100::kLimitWord, words, sizeof(words), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return fail(STRATUM_ERR_CUDA, "set_wait_limit_ns: copy failed: %s", cudaGetErrorString(cudaGetLastError()));
    return STRATUM_OK;
}

int stratum_wait_selftest(void *stream) {
    STRATUM_BIND_STREAM(stream);
    int *dp = gemm::status_ptr();
    if (!dp) return fail(STRATUM_ERR_CUDA, "wait_selftest: cannot resolve the status word");
    gemm::k_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dp);
    return check_launch("wait_selftest");
}

int stratum_nf4_gemm_set_kernel(int which) {
    STRATUM_REQUIRE(which == STRATUM_GEMM_AUTO || which == STRATUM_GEMM_PAIR || which == STRATUM_GEMM_SINGLE,
                    "nf4_gemm_set_kernel: unknown kernel %d", which);
    gemm::g_gemm_kernel.store(which, std::memory_order_relaxed);
    return STRATUM_OK;
}

int stratum_nf4_gemm_fwd(const void *x, int x_dtype, int64_t T, int64_t K, const uint8_t *packed, const float *absmax,
                         const uint8_t *absmax_q, const float *absmax2, const float *code2, const float *offset,
                         const float *code16, int64_t N, const void *bias, int bias_dtype, const void *lora_xa,
                         const void *lora_b, int r, void *y, void *stream) {
    STRATUM_REQUIRE(T >= 0 && N >= 0 && K >= 0, "nf4_gemm_fwd: negative size");
    if (T == 0 || N == 0) return STRATUM_OK;
    STRATUM_REQUIRE(x && packed && code16 && y, "nf4_gemm_fwd: null pointer");
    if (x_dtype != STRATUM_BF16 && x_dtype != STRATUM_F16)
        return fail(STRATUM_ERR_UNSUPPORTED, "nf4_gemm_fwd: x must be bf16 or fp16");
    if (K % gemm::BK != 0 || K == 0)
        return fail(STRATUM_ERR_UNSUPPORTED, "nf4_gemm_fwd: K=%lld must be a positive multiple of 64", (long long)K);
    const bool dq = absmax == nullptr;
    STRATUM_REQUIRE(!dq || (absmax_q && absmax2 && code2 && offset), "nf4_gemm_fwd: need absmax or the double-quant set");
    STRATUM_REQUIRE(r >= 0 && r <= 256, "nf4_gemm_fwd: lora rank %d out of range", r);
    STRATUM_REQUIRE(r == 0 || (lora_xa && lora_b && r % 2 == 0), "nf4_gemm_fwd: lora needs xa, B and an even rank");
    STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(packed) % 16 == 0,
                    "nf4_gemm_fwd: x and packed must be 16-byte aligned");
    STRATUM_REQUIRE(T <= (int64_t(1) << 31) && N <= (int64_t(1) << 31), "nf4_gemm_fwd: size too large");
    STRATUM_BIND_STREAM(stream);
    int *status = gemm::status_ptr();
    if (!status) return fail(STRATUM_ERR_CUDA, "nf4_gemm_fwd: no status word");

    const bool bf16 = x_dtype == STRATUM_BF16;
    const CUtensorMapDataType xdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap mx, mw, mxa;
    int rc = gemm::make_map_2d(&mx, xdt, x, uint64_t(K), uint64_t(T), uint64_t(K) * 2, gemm::BK, gemm::BNH,
                               CU_TENSOR_MAP_SWIZZLE_128B, "nf4_gemm_fwd x");
    if (rc) return rc;
    // 32-byte swizzle: rows r and r+4 trade 16-byte halves, so the dequant
    // warps' row-per-lane 16-byte reads are bank-conflict free
    rc = gemm::make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, packed, uint64_t(K / 2), uint64_t(N), uint64_t(K / 2),
                           gemm::BK / 2, gemm::BM, CU_TENSOR_MAP_SWIZZLE_32B, "nf4_gemm_fwd packed");
    if (rc) return rc;
    const int lora_chunks = (r + gemm::BK - 1) / gemm::BK;
    if (r > 0) {
        STRATUM_REQUIRE(reinterpret_cast<uintptr_t>(lora_xa) % 16 == 0, "nf4_gemm_fwd: xa must be 16-byte aligned");
        rc = gemm::make_map_2d(&mxa, xdt, lora_xa, uint64_t(lora_chunks * gemm::BK), uint64_t(T),
                               uint64_t(lora_chunks * gemm::BK) * 2, gemm::BK, gemm::BNH, CU_TENSOR_MAP_SWIZZLE_128B,
                               "nf4_gemm_fwd xa");
        if (rc) return rc;
    } else {
        mxa = mx;
    }
    gemm::FwdParams p{};
    p.w = gemm::WeightScales{absmax, absmax_q, absmax2, code2, offset};
    p.code16 = code16;
    p.bias = bias;
    p.bias_dtype = bias_dtype;
    p.lora_b = static_cast<const uint16_t *>(lora_b);
    p.r = r;
    p.lora_chunks = lora_chunks;
    p.y = static_cast<uint16_t *>(y);
    p.T = T;
    p.N = N;
    p.K = K;
    p.n_tiles = int((N + gemm::BM - 1) / gemm::BM);
    p.tile_tokens = gemm::fwd_tile_tokens(T, p.n_tiles);
    p.t_tiles = int((T + p.tile_tokens - 1) / p.tile_tokens);
    p.status = status;
    p.tma_store = (reinterpret_cast<uintptr_t>(y) % 16 == 0) && (N % 8 == 0);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (gemm::use_pair(T, N, p.tile_tokens, p.tile_tokens == gemm::BNH ? 1.4 : 1.0)) {
        // CTA-pair kernel: 512-token x 256-row tiles, each CTA stages 128-token boxes
        namespace pr = gemm::pair;
        pr::Params q{};
        q.w = p.w;
        q.code16 = code16;
        q.bias = bias;
        q.bias_dtype = bias_dtype;
        q.lora = p.lora_b;
        q.r = r;
        q.lora_chunks = lora_chunks;
        q.y = p.y;
        q.T = T;
        q.M = N;
        q.C = K;
        q.kbl = K / 64;
        q.m_tiles = int((N + 2 * pr::BM - 1) / (2 * pr::BM));
        q.t_tiles = int((T + pr::BN - 1) / pr::BN);
        q.tma_store = p.tma_store;
        q.status = status;
        rc = gemm::make_map_2d(&mx, xdt, x, uint64_t(K), uint64_t(T), uint64_t(K) * 2, pr::BK, pr::CT,
                               CU_TENSOR_MAP_SWIZZLE_128B, "nf4_gemm_fwd x");
        if (rc) return rc;
        if (r > 0) {
            rc = gemm::make_map_2d(&mxa, xdt, lora_xa, uint64_t(lora_chunks * pr::BK), uint64_t(T),
                                   uint64_t(lora_chunks * pr::BK) * 2, pr::BK, pr::CT, CU_TENSOR_MAP_SWIZZLE_128B,
                                   "nf4_gemm_fwd xa");
            if (rc) return rc;
        } else {
            mxa = mx;
        }
        const CUtensorMap &my = mx;  // y is written with 16-byte stores (q.tma_store: aligned, N % 8 == 0)
        if (bf16)
            return dq ? gemm::launch_pair<true, true, false, false>(mx, mw, mw, mxa, my, q, st, "nf4_gemm_fwd")
                      : gemm::launch_pair<true, false, false, false>(mx, mw, mw, mxa, my, q, st, "nf4_gemm_fwd");
        return dq ? gemm::launch_pair<false, true, false, false>(mx, mw, mw, mxa, my, q, st, "nf4_gemm_fwd")
                  : gemm::launch_pair<false, false, false, false>(mx, mw, mw, mxa, my, q, st, "nf4_gemm_fwd");
    }
    CUtensorMap my = mx;
    if (p.tma_store) {
        rc = gemm::make_map_2d(&my, xdt, y, uint64_t(N), uint64_t(T), uint64_t(N) * 2, 64, gemm::BNH,
                               CU_TENSOR_MAP_SWIZZLE_128B, "nf4_gemm_fwd y");
        if (rc) return rc;
    }
    if (bf16)
        return dq ? gemm::launch_fwd<true, true, false>(mx, mw, mw, mxa, my, p, st)
                  : gemm::launch_fwd<true, false, false>(mx, mw, mw, mxa, my, p, st);
    return dq ? gemm::launch_fwd<false, true, false>(mx, mw, mw, mxa, my, p, st)
              : gemm::launch_fwd<false, false, false>(mx, mw, mw, mxa, my, p, st);
}

int stratum_nf4_gemm_swiglu_fwd(const void *x, int x_dtype, int64_t T, int64_t K, const stratum_nf4_weight *gate,
                                const stratum_nf4_weight *up, const float *code16, int64_t I, const void *lora_xa,
                                const void *lora_b_gate, const void *lora_b_up, int r, void *h, void *gate_out,
                                void *up_out, void *stream) {
    STRATUM_REQUIRE(T >= 0 && I >= 0 && K >= 0, "nf4_gemm_swiglu_fwd: negative size");
    if (T == 0 || I == 0) return STRATUM_OK;
    STRATUM_REQUIRE(x && gate && up && gate->packed && up->packed && code16 && h, "nf4_gemm_swiglu_fwd: null pointer");
    if (x_dtype != STRATUM_BF16 && x_dtype != STRATUM_F16)
        return fail(STRATUM_ERR_UNSUPPORTED, "nf4_gemm_swiglu_fwd: x must be bf16 or fp16");
    if (K % gemm::BK != 0 || K == 0)
        return fail(STRATUM_ERR_UNSUPPORTED, "nf4_gemm_swiglu_fwd: K=%lld must be a positive multiple of 64",
                    (long long)K);
    if (I % 64 != 0)
        return fail(STRATUM_ERR_UNSUPPORTED, "nf4_gemm_swiglu_fwd: I=%lld must be a multiple of 64", (long long)I);
    const bool dq = gate->absmax == nullptr;
    STRATUM_REQUIRE((up->absmax == nullptr) == dq, "nf4_gemm_swiglu_fwd: gate and up must both be plain or both "
                                                   "double quantized");
    STRATUM_REQUIRE(!dq || (gate->absmax_q && gate->absmax2 && gate->code2 && gate->offset && up->absmax_q &&
                            up->absmax2 && up->code2 && up->offset),
                    "nf4_gemm_swiglu_fwd: need absmax or the double-quant set for both weights");
    STRATUM_REQUIRE(r >= 0 && r <= 256 && r % 2 == 0, "nf4_gemm_swiglu_fwd: lora rank %d must be even, <= 256", r);
    STRATUM_REQUIRE(r == 0 || (lora_xa && lora_b_gate && lora_b_up), "nf4_gemm_swiglu_fwd: lora needs xa and both B");
    auto a16 = [](const void *q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    STRATUM_REQUIRE(a16(x) && a16(gate->packed) && a16(up->packed) && a16(h) && a16(gate_out) && a16(up_out),
                    "nf4_gemm_swiglu_fwd: x, packed and the outputs must be 16-byte aligned");
    STRATUM_REQUIRE(T <= (int64_t(1) << 31) && I <= (int64_t(1) << 30), "nf4_gemm_swiglu_fwd: size too large");
    STRATUM_BIND_STREAM(stream);
    int *status = gemm::status_ptr();
    if (!status) return fail(STRATUM_ERR_CUDA, "nf4_gemm_swiglu_fwd: no status word");

    const bool bf16 = x_dtype == STRATUM_BF16;
    const CUtensorMapDataType xdt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap mx, mw, mw2, mxa;
    int rc = gemm::make_map_2d(&mx, xdt, x, uint64_t(K), uint64_t(T), uint64_t(K) * 2, gemm::BK, gemm::BNH,
                               CU_TENSOR_MAP_SWIZZLE_128B, "nf4_gemm_swiglu_fwd x");
    if (rc) return rc;
    // each weight contributes 64 rows per tile: boxes of 32 bytes x 64 rows
    rc = gemm::make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, gate->packed, uint64_t(K / 2), uint64_t(I),
                           uint64_t(K / 2), gemm::BK / 2, 64, CU_TENSOR_MAP_SWIZZLE_32B, "nf4_gemm_swiglu_fwd gate");
    if (rc) return rc;
    rc = gemm::make_map_2d(&mw2, CU_TENSOR_MAP_DATA_TYPE_UINT8, up->packed, uint64_t(K / 2), uint64_t(I),
                           uint64_t(K / 2), gemm::BK / 2, 64, CU_TENSOR_MAP_SWIZZLE_32B, "nf4_gemm_swiglu_fwd up");
    if (rc) return rc;
    const int rp = (r + gemm::BK - 1) / gemm::BK * gemm::BK;
    const int lora_chunks = 2 * rp / gemm::BK;
    if (r > 0) {
        STRATUM_REQUIRE(a16(lora_xa), "nf4_gemm_swiglu_fwd: xa must be 16-byte aligned");
        rc = gemm::make_map_2d(&mxa, xdt, lora_xa, uint64_t(2 * rp), uint64_t(T), uint64_t(2 * rp) * 2, gemm::BK,
                               gemm::BNH, CU_TENSOR_MAP_SWIZZLE_128B, "nf4_gemm_swiglu_fwd xa");
        if (rc) return rc;
    } else {
        mxa = mx;
    }
    gemm::FwdParams p{};
    p.w = gemm::WeightScales{gate->absmax, gate->absmax_q, gate->absmax2, gate->code2, gate->offset};
    p.wu = gemm::WeightScales{up->absmax, up->absmax_q, up->absmax2, up->code2, up->offset};
    p.code16 = code16;
    p.lora_b = static_cast<const uint16_t *>(lora_b_gate);
    p.lora_bu = static_cast<const uint16_t *>(lora_b_up);
    p.r = r;
    p.lora_rp = rp;
    p.lora_chunks = lora_chunks;
    p.y = static_cast<uint16_t *>(h);
    p.gate = static_cast<uint16_t *>(gate_out);
    p.up = static_cast<uint16_t *>(up_out);
    p.T = T;
    p.N = I;
    p.K = K;
    p.n_tiles = int(I / 64);
    p.tile_tokens = gemm::fwd_tile_tokens(T, p.n_tiles);
    p.t_tiles = int((T + p.tile_tokens - 1) / p.tile_tokens);
    p.status = status;
    p.tma_store = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (bf16)
        return dq ? gemm::launch_fwd<true, true, true>(mx, mw, mw2, mxa, mx, p, st)
                  : gemm::launch_fwd<true, false, true>(mx, mw, mw2, mxa, mx, p, st);
    return dq ? gemm::launch_fwd<false, true, true>(mx, mw, mw2, mxa, mx, p, st)
              : gemm::launch_fwd<false, false, true>(mx, mw, mw2, mxa, mx, p, st);
}

int stratum_nf4_gemm_dx(const void *dy, int dtype, int64_t T, int64_t N, const uint8_t *packed, const float *absmax,
                        const uint8_t *absmax_q, const float *absmax2, const float *code2, const float *offset,
                        const float *code16, int64_t K, const void *lora_dyb, const void *lora_a, int r, void *dx_out,
                        void *stream) {
    const stratum_nf4_weight w{packed, absmax, absmax_q, absmax2, code2, offset};
    return gemm::dx_run(dy, dtype, T, N, w, nullptr, 0, code16, K, lora_dyb, lora_a, r, dx_out, stream,
                        "nf4_gemm_dx");
}

int stratum_nf4_gemm_dx_pair(const void *dy, int dtype, int64_t T, const stratum_nf4_weight *w0, int64_t N0,
                             const stratum_nf4_weight *w1, int64_t N1, const float *code16, int64_t K,
                             const void *lora_dyb, const void *lora_a, int r, void *dx_out, void *stream) {
    STRATUM_REQUIRE(w0 && w1, "nf4_gemm_dx_pair: null weight");
    STRATUM_REQUIRE(N0 > 0 && N1 > 0 && N0 % 64 == 0 && N1 % 64 == 0,
                    "nf4_gemm_dx_pair: N0=%lld and N1=%lld must be positive multiples of 64", (long long)N0,
                    (long long)N1);
    return gemm::dx_run(dy, dtype, T, N0 + N1, *w0, w1, N0, code16, K, lora_dyb, lora_a, r, dx_out, stream,
                        "nf4_gemm_dx_pair");
}

}  // extern "C"
