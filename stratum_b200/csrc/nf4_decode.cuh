// Register-only NF4 decoding of one 64-element block (32 packed bytes, one
// absmax) into 32 packed 16-bit pairs, shared by the standalone dequantizer
// and the GEMMs' dequant warps.
//
// Per block the thread builds the 16 scaled levels once,
//     T[i] = round16(fp32(level[i] * absmax)),
// (exactly the value bitsandbytes' dequantizer produces for code i), splits
// them into a low-byte and a high-byte table of 16 bytes each (4 registers
// apiece), and then decodes 4 codes per byte-permute: prmt selects with a
// 3-bit index per output byte from 8 table bytes, so each table half is
// looked up once and a per-byte mask built from the code's bit 3 picks the
// half.  Cost: 32 ops to build the tables per block, 22 ops per 8 codes.
#pragma once

#include <stdint.h>

#include "sm100.cuh"

namespace stratum {

struct Nf4Tables {
    uint32_t lo[4];  // byte j of lo[r] = low byte of T[4r + j]
    uint32_t hi[4];  // byte j of hi[r] = high byte of T[4r + j]
};

// levels: the 16 fp32 levels (registers or shared memory), am: block absmax.
template <bool BF16>
__device__ __forceinline__ Nf4Tables nf4_build_tables(const float *levels, float am) {
    uint32_t p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float a = __fmul_rn(levels[2 * j], am);
        const float b = __fmul_rn(levels[2 * j + 1], am);
        p[j] = BF16 ? sm100::pack_bf16x2(a, b) : sm100::pack_f16x2(a, b);  // T[2j] in bits 0-15
    }
    Nf4Tables t;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        t.lo[r] = sm100::prmt(p[2 * r], p[2 * r + 1], 0x6420);
        t.hi[r] = sm100::prmt(p[2 * r], p[2 * r + 1], 0x7531);
    }
    return t;
}

// Decode one little-endian packed word (bytes b0..b3 = elements e0..e7, the
// first element of each byte in its high nibble) into 4 pairs
// out[m] = {e[2m] in bits 0-15, e[2m+1] in bits 16-31}.
__device__ __forceinline__ void nf4_decode_word(const Nf4Tables &t, uint32_t w, uint32_t out[4]) {
    const uint32_t w4 = w << 4;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // selector nibbles j = 0..3 hold codes [e1, e0, e3, e2] (h = 0) or [e5, e4, e7, e6] (h = 1)
        const uint32_t sel = (h == 0 ? w : (w >> 16)) & 0x7777u;
        // byte j of m = 0xFF where the code of selector nibble j has bit 3 set
        // (sign-replicate mode of prmt on the byte holding that bit)
        const uint32_t m = sm100::prmt(w, w4, h == 0 ? 0x9D8Cu : 0xBFAEu);
        const uint32_t l = (sm100::prmt(t.lo[0], t.lo[1], sel) & ~m) | (sm100::prmt(t.lo[2], t.lo[3], sel) & m);
        const uint32_t g = (sm100::prmt(t.hi[0], t.hi[1], sel) & ~m) | (sm100::prmt(t.hi[2], t.hi[3], sel) & m);
        out[2 * h] = sm100::prmt(l, g, 0x4051u);      // {e0|e4 : lo byte, hi byte, e1|e5 : lo, hi}
        out[2 * h + 1] = sm100::prmt(l, g, 0x6273u);  // {e2|e6, e3|e7}
    }
}

// 32 packed bytes (8 words) -> 32 pairs (64 elements).
__device__ __forceinline__ void nf4_decode_block(const Nf4Tables &t, const uint32_t (&w)[8], uint32_t (&out)[32]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        uint32_t o[4];
        nf4_decode_word(t, w[i], o);
        out[4 * i + 0] = o[0];
        out[4 * i + 1] = o[1];
        out[4 * i + 2] = o[2];
        out[4 * i + 3] = o[3];
    }
}

}  // namespace stratum
