/* CPU oracle for the NF4 codec, plain C + OpenMP.  TEST INFRASTRUCTURE ONLY.
 *
 * Same algorithm as oracle/nf4_oracle.py (which documents the sources and the
 * "parity unpinned" status in full): bitsandbytes' blockwise NF4 quantizer and
 * dequantizer as called by the reference at stratum/upload.py:355-369 and
 * :1021-1040, restated.  This C version exists so that the CPU baseline in
 * bench.py can be timed on all host cores; tests check it against the numpy
 * restatement.  Nothing in the product links it.
 *
 * Build: make -C oracle   (-> oracle/_build/libnf4_oracle.so)
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

enum { NF4O_F32 = 0, NF4O_F16 = 1, NF4O_BF16 = 2 };

static float load_elem(const void *src, int dtype, int64_t i) {
    if (dtype == NF4O_F32) return ((const float *)src)[i];
    if (dtype == NF4O_F16) return (float)((const _Float16 *)src)[i];
    uint32_t b = (uint32_t)((const uint16_t *)src)[i] << 16;
    float f;
    memcpy(&f, &b, 4);
    return f;
}

static uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if (isnan(f)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static void store_elem(void *dst, int dtype, int64_t i, float v) {
    if (dtype == NF4O_F32) ((float *)dst)[i] = v;
    else if (dtype == NF4O_F16) ((_Float16 *)dst)[i] = (_Float16)v;
    else ((uint16_t *)dst)[i] = f32_to_bf16(v);
}

/* number of thresholds strictly below x (NaN -> 0) */
static inline int count_below(float x, const float *thr, int nthr) {
    int lo = 0, hi = nthr; /* binary search on sorted thresholds */
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (x > thr[mid]) lo = mid + 1; else hi = mid;
    }
    return lo;
}

/* NF4 quantize: packed[ceil(n/2)], absmax[ceil(n/blocksize)].  thr = 15 fp32 midpoints. */
void nf4o_quantize(const void *src, int dtype, int64_t n, int blocksize, const float *thr,
                   uint8_t *packed, float *absmax, int nthreads) {
    int64_t nb = (n + blocksize - 1) / blocksize;
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t b = 0; b < nb; ++b) {
        int64_t s = b * blocksize, e = s + blocksize < n ? s + blocksize : n;
        float am = 0.f;
        for (int64_t i = s; i < e; ++i) {
            float a = fabsf(load_elem(src, dtype, i));
            am = a > am ? a : am;
        }
        absmax[b] = am;
        float inv = 1.0f / am;
        /* blocksize is even, so a block owns whole bytes; a ragged odd tail pads with 0.0 */
        int64_t pe = e + ((e - s) & 1);
        for (int64_t i = s; i < pe; i += 2) {
            float x0 = load_elem(src, dtype, i) * inv;
            float x1 = (i + 1 < e) ? load_elem(src, dtype, i + 1) * inv : 0.0f * inv;
            packed[i >> 1] = (uint8_t)((count_below(x0, thr, 15) << 4) | count_below(x1, thr, 15));
        }
    }
}

void nf4o_dequantize(const uint8_t *packed, const float *absmax, const float *levels, int64_t n,
                     int blocksize, void *out, int out_dtype, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint8_t byte = packed[i >> 1];
        int q = (i & 1) ? (byte & 0xF) : (byte >> 4);
        float v = levels[q] * absmax[i / blocksize];
        store_elem(out, out_dtype, i, v);
    }
}

/* Deterministic double-quant offset: chunked sequential fp64 sums (chunk 1024). */
float nf4o_dq_mean(const float *absmax, int64_t nb) {
    double total = 0.0;
    for (int64_t c0 = 0; c0 < nb; c0 += 1024) {
        double part = 0.0;
        int64_t c1 = c0 + 1024 < nb ? c0 + 1024 : nb;
        for (int64_t i = c0; i < c1; ++i) part += (double)absmax[i];
        total += part;
    }
    return (float)(total / (double)nb);
}

/* Double-quantize absmax: absmax_q[nb], absmax2[ceil(nb/bs2)], offset.  thr2 = 255 midpoints of code2. */
void nf4o_quantize_absmax_dq(const float *absmax, int64_t nb, int bs2, const float *thr2,
                             uint8_t *absmax_q, float *absmax2, float *offset_out, int nthreads) {
    float off = nf4o_dq_mean(absmax, nb);
    *offset_out = off;
    int64_t nb2 = (nb + bs2 - 1) / bs2;
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t b = 0; b < nb2; ++b) {
        int64_t s = b * bs2, e = s + bs2 < nb ? s + bs2 : nb;
        float am = 0.f;
        for (int64_t i = s; i < e; ++i) {
            float a = fabsf(absmax[i] - off);
            am = a > am ? a : am;
        }
        absmax2[b] = am;
        float inv = 1.0f / am;
        for (int64_t i = s; i < e; ++i) absmax_q[i] = (uint8_t)count_below((absmax[i] - off) * inv, thr2, 255);
    }
}

void nf4o_dequantize_dq(const uint8_t *packed, const uint8_t *absmax_q, const float *absmax2,
                        const float *code2, float offset, int bs2, const float *levels, int64_t n,
                        int blocksize, void *out, int out_dtype, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        int64_t b = i / blocksize;
        float am = code2[absmax_q[b]] * absmax2[b / bs2];
        am = am + offset;
        uint8_t byte = packed[i >> 1];
        int q = (i & 1) ? (byte & 0xF) : (byte >> 4);
        store_elem(out, out_dtype, i, levels[q] * am);
    }
}
