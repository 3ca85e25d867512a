// Shared helpers for the libstratum_nf4 C ABI: status/error reporting,
// launch accounting and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <atomic>

#include "../../include/stratum_nf4.h"

namespace stratum {

// Per-thread message of the last failing call (read by stratum_last_error()).
extern thread_local char g_last_error[512];
extern std::atomic<uint64_t> g_launches;

inline int fail(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

// Checks the launch that was just enqueued; counts it on success.
inline int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(STRATUM_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return STRATUM_OK;
}

inline int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (cached[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

// This library links its own CUDA runtime, whose current device is separate
// from the caller's (torch's).  Every entry point makes the device of the
// stream it was given current; a NULL stream (the legacy default stream) keeps
// the library's current device, which stratum_set_device() selects.  A stream
// that is being captured into a CUDA graph cannot be asked for its device (the
// query is not permitted during capture and would invalidate it), so while a
// stream captures, the library's current device is used as well: callers that
// capture on a device other than the last one used select it with
// stratum_set_device() first.
inline int bind_stream_device(void *stream) {
    if (stream == nullptr) return STRATUM_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(STRATUM_ERR_CUDA, "cannot query the stream's capture state: %s", cudaGetErrorString(e));
    }
    if (cs != cudaStreamCaptureStatusNone) return STRATUM_OK;
    int dev = -1;
    e = cudaStreamGetDevice(st, &dev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(STRATUM_ERR_CUDA, "cannot query the stream's device: %s", cudaGetErrorString(e));
    }
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev && (e = cudaSetDevice(dev)) != cudaSuccess) {
        cudaGetLastError();
        return fail(STRATUM_ERR_CUDA, "cannot select device %d: %s", dev, cudaGetErrorString(e));
    }
    return STRATUM_OK;
}

#define STRATUM_BIND_STREAM(stream) \
    do { int rc_ = ::stratum::bind_stream_device(stream); if (rc_) return rc_; } while (0)

// Resident CTAs of `kernel` on the whole GPU (SM count x occupancy), cached per kernel.
template <auto Kernel>
inline int64_t resident_grid(int threads, size_t smem = 0) {
    static int64_t cached = 0;
    if (cached == 0) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, Kernel, threads, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        cached = int64_t(per_sm) * sm_count();
    }
    return cached;
}

inline bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }
inline int ilog2(int64_t v) { int l = 0; while ((int64_t(1) << l) < v) ++l; return l; }

#define STRATUM_REQUIRE(cond, ...) \
    do { if (!(cond)) return ::stratum::fail(STRATUM_ERR_INVALID, __VA_ARGS__); } while (0)

// ----------------------------------------------------------------- device --

__device__ __forceinline__ float load_as_f32(const float *p, int64_t i) { return p[i]; }
__device__ __forceinline__ float load_as_f32(const __half *p, int64_t i) { return __half2float(p[i]); }
__device__ __forceinline__ float load_as_f32(const __nv_bfloat16 *p, int64_t i) { return __bfloat162float(p[i]); }

// Global accesses that allocate no L1 line, for the small kernels that run right
// before the grouped NF4 GEMMs.  Those GEMMs' CTAs take the whole of the SM's
// shared memory (the SRAM that L1 shares), and 128-byte lines the preceding kernel
// had touched (bf16 rows of dy_sorted, routing weights) were found in a grouped
// GEMM's barrier words.  The loads are for data no thread of the kernel writes
// (the non-coherent path), so they carry no ordering and the compiler may move them.
__device__ __forceinline__ uint4 ld_na(const uint4 *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ int ld_na(const int *p) {
    int v;
    asm("ld.global.nc.L1::no_allocate.b32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_na(const float *p) {
    float v;
    asm("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void st_na(uint4 *p, uint4 v) {
    asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_na(float *p, float v) {
    asm volatile("st.global.L1::no_allocate.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Index of the level for a scaled value: number of thresholds strictly below x.
// thr[0..14] sorted, thr[15] = +inf padding; NaN fails every test -> 0.
__device__ __forceinline__ uint32_t nf4_code(float x, const float *thr, float t7) {
    uint32_t i = (x > t7) ? 8u : 0u;
    i += (x > thr[i + 3]) ? 4u : 0u;
    i += (x > thr[i + 1]) ? 2u : 0u;
    i += (x > thr[i]) ? 1u : 0u;
    return i;
}

}  // namespace stratum
