// Thin inline-PTX wrappers for the sm_100a features the NF4 GEMMs use:
// mbarriers (with bounded waits), TMA tile loads (per-CTA, no broadcast), TMEM
// allocation, tcgen05.mma with the A operand in TMEM, commits, TMEM
// loads/stores and the tcgen05 ordering fences.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace stratum {
namespace sm100 {

// Status word written by a kernel whose bounded wait gave up (0 = fine).
// Host code reads it with stratum_device_status().
enum DeviceError : int {
    kErrNone = 0,
    kErrTimeoutProducer = 0x101,
    kErrTimeoutMma = 0x102,
    kErrTimeoutDequant = 0x103,
    kErrTimeoutEpilogue = 0x104,
    kErrTimeoutTeardown = 0x105,
    // added to the five codes above, so the status word names the kernel family
    kErrPairOffset = 0x10,     // CTA-pair GEMMs
    kErrFwdOffset = 0x20,      // one-SM forward GEMM
    kErrDxOffset = 0x30,       // one-SM input-gradient GEMM
    kErrGroupedFwdOffset = 0x40,  // grouped expert forward
    kErrGroupedDxOffset = 0x50,   // grouped expert input gradient
    kErrBadOffsets = 0x201,  // grouped GEMM: expert offsets outside [0, total tokens]
    kErrTileTable = 0x202,   // grouped GEMM: tile table smaller than the offsets need
    kErrWaitSelfTest = 0x1f0,  // stratum_wait_selftest: its wait on a barrier nothing completes gave up
};

// A wait that takes longer than this is a hang, never a slow pipeline stage
// (one stage is microseconds); the kernel then records an error and unwinds.
// The default; stratum_set_wait_limit_ns changes it per device.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;
// Suspend-time hint for a blocked mbarrier wait (the thread wakes when the phase completes).
constexpr uint32_t kSuspendHintNs = 1000000u;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait that lets the hardware suspend the thread (up to `hint_ns`) until
// the phase completes, instead of spinning on the issue slots that the
// working warps of the same sub-partition need.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Words of the status record (err): [0] code, [1] block, [2] thread, [3] parity,
// [4] the barrier's shared-memory offset, [5..6] its 64-bit state, [7] the SM,
// [8..9] nanoseconds and [10] SM clock cycles the wait lasted (%globaltimer and
// clock64 each, so a clock that jumped shows as the two disagreeing), and from
// [12] kBarSnap 64-bit shared-memory words (two ints each, low first): the
// kBarBelow words below the barrier waited on, that barrier, and kBarAbove words
// above it -- the CTA's other stage barriers and the progress words some
// kernels keep beside them, which say which role stopped.  Every kernel keeps at
// least 16 KiB of tiles below its barrier area and at least 1 KiB of tables
// above it, so the snapshot stays inside the CTA's shared memory.
constexpr int kBarBelow = 17, kBarAbove = 9;
constexpr int kBarSnap = kBarBelow + 1 + kBarAbove;
constexpr int kStatusWords = 72;
static_assert(12 + 2 * kBarSnap <= kStatusWords, "status record");
// Two more words after the record hold the wait limit in nanoseconds (0 =
// kWaitTimeoutNs), set by stratum_set_wait_limit_ns; clearing the record keeps them.
constexpr int kLimitWord = kStatusWords;
constexpr int kStatusAlloc = kStatusWords + 2;

// The wait limit in force (read from memory on every slow-path check, so the
// loop holds no extra register for it).
__device__ __forceinline__ uint64_t wait_limit_ns(const int *err) {
    const volatile uint32_t *w = reinterpret_cast<const volatile uint32_t *>(err + kLimitWord);
    const uint64_t v = uint64_t(w[0]) | (uint64_t(w[1]) << 32);
    return v ? v : kWaitTimeoutNs;
}

__device__ __forceinline__ uint32_t sm_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint64_t ld_shared_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(smem_u32(p)));
    return v;
}

// Record a wait that gave up: the first such thread of the grid writes `code` to
// err[0] and the rest of the record above (err points to kStatusWords ints);
// t0 is %globaltimer and c0 the low word of clock64 when the wait began (a wait
// gives up after ~2 s, fewer than 2^32 cycles at B200 clocks, so the 32-bit
// difference is exact).
__device__ __forceinline__ void record_timeout(int *err, int code, uint64_t *bar, uint32_t parity, uint64_t t0,
                                               uint32_t c0) {
    if (atomicCAS(err, 0, code) != 0) return;
    const uint64_t t1 = globaltimer();
    const uint32_t dc = uint32_t(clock64()) - c0;
    volatile int *d = err;
    const uint64_t state = ld_shared_u64(bar);
    d[1] = int(blockIdx.x);
    d[2] = int(threadIdx.x);
    d[3] = int(parity);
    d[4] = int(smem_u32(bar));
    d[5] = int(uint32_t(state));
    d[6] = int(uint32_t(state >> 32));
    d[7] = int(sm_id());
    d[8] = int(uint32_t(t1 - t0));
    d[9] = int(uint32_t((t1 - t0) >> 32));
    d[10] = int(dc);
    d[11] = 0;
    for (int i = 0; i < kBarSnap; ++i) {
        const uint64_t v = ld_shared_u64(bar - kBarBelow + i);
        d[12 + 2 * i] = int(uint32_t(v));
        d[13 + 2 * i] = int(uint32_t(v >> 32));
    }
    __threadfence();
}

// Bounded wait for the phase with the given parity.  Returns false (after
// recording `code` in *err) on timeout, or when another thread of the grid
// already recorded an error, so every role unwinds instead of spinning.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    const uint32_t c0 = uint32_t(clock64());
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
        if (*reinterpret_cast<volatile int *>(err) != 0) return false;
        if (globaltimer() - t0 > wait_limit_ns(err)) {
            record_timeout(err, code, bar, parity, t0, c0);
            return false;
        }
    }
}

// Bounded wait for work this CTA already issued (teardown): unlike mbar_wait it
// does not give up when another thread recorded an error, so a CTA that unwinds
// still waits -- up to the time limit -- for its own copies and MMAs before it
// frees shared memory or TMEM.
__device__ __forceinline__ bool mbar_wait_issued(uint64_t *bar, uint32_t parity, int *err, int code) {
    const uint64_t t0 = globaltimer();
    const uint32_t c0 = uint32_t(clock64());
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, kSuspendHintNs)) return true;
        if (globaltimer() - t0 > wait_limit_ns(err)) {
            record_timeout(err, code, bar, parity, t0, c0);
            return false;
        }
    }
}

// 2-D TMA tile load into shared memory, completion counted on `bar` (bytes).
// Every CTA fetches its own tiles (no cluster-wide broadcast form).
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int32_t c0, int32_t c1,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- TMEM -------------------------------------------------------------------

// Whole-warp collective: allocate `ncols` (power of two >= 32) TMEM columns and
// write the base address to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem desc]; kind::f16 (fp16/bf16 in, fp32 accumulate).
__device__ __forceinline__ void mma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; kind::f16.
__device__ __forceinline__ void mma_ss_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Instruction descriptor for kind::f16: fp32 accumulate, A/B both fp16 or
// both bf16, both K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N) {
    return (1u << 4)                              // D format: f32
           | ((bf16 ? 1u : 0u) << 7)              // A format
           | ((bf16 ? 1u : 0u) << 10)             // B format
           | (uint32_t(N >> 3) << 17)             // N / 8
           | (uint32_t(M >> 4) << 24);            // M / 16
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), tile base 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(const void *tile) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = 0;
    d |= (addr & 0x3FFFFull) >> 4;       // start address
    d |= uint64_t(1) << 16;              // LBO (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;      // SBO
    d |= uint64_t(1) << 46;              // descriptor version (sm100)
    d |= uint64_t(2) << 61;              // SWIZZLE_128B
    return d;
}

// Shared-memory matrix descriptor: MN-major, 128-byte swizzle.  Atoms of 8
// K-rows x 128 bytes (64 16-bit MN elements); `lbo` = byte stride between
// 64-element MN atoms, `sbo` = byte stride between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_mn_sw128(const void *tile, uint32_t lbo, uint32_t sbo) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = 0;
    d |= (addr & 0x3FFFFull) >> 4;
    d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor for kind::f16 with A MN-major (transposed), B K-major.
__host__ __device__ constexpr uint32_t idesc_f16_amn(bool bf16, int M, int N) {
    return idesc_f16(bf16, M, N) | (1u << 15);
}

// 32 lanes x 32 columns of 32-bit: thread t <-> lane (base + t), 32 registers.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 lanes x 256 bits, twice along columns (16 columns): thread t gets
// {lane t/4: col 2(t%4), 2(t%4)+1}, {lane t/4+8: same}, then the same for columns +8.
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

// Four 8x8 16-bit matrices, stored transposed: the row addressed by thread
// 8k + j receives column j of matrix k.
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t smem_addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("stmatrix.sync.aligned.x4.trans.m8n8.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(smem_addr), "r"(a),
                 "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Generic-proxy shared-memory writes become visible to the TMA (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 2-D TMA tile store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int32_t c0, int32_t c1, const void *smem_src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(smem_u32(smem_src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// at most one bulk store group still reading its shared-memory source
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

// ---- CTA pairs (clusters of two CTAs sharing 2-SM tcgen05 MMAs) ------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t n_clusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Every thread of both CTAs: release this CTA's prior writes, wait for the peer's.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

// `count` arrivals on an mbarrier given by its shared::cluster address (this CTA's
// or the peer's), releasing this thread's prior writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr, uint32_t count) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr), "r"(count)
                 : "memory");
}

// One arrival on an mbarrier of either CTA of the pair (shared::cluster address)
// with the default semantics (release at CTA scope), as cluster barriers are
// signalled between the CTAs of a 2-SM MMA: cheap, unlike a cluster-scope release,
// which makes the arriving thread wait ~1500 cycles for its stores to drain.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// try_wait that acquires at cluster scope (phases completed by the peer CTA's
// arrivals), with the same suspend hint as mbar_try_wait_sleep.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded cluster-scope wait: gives up on timeout or once another thread of the
// grid recorded an error (as mbar_wait).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int *err, int code) {
    if (mbar_try_wait_cluster(bar, parity, 0u)) return true;
    const uint64_t t0 = globaltimer();
    const uint32_t c0 = uint32_t(clock64());
    while (true) {
        if (mbar_try_wait_cluster(bar, parity, kSuspendHintNs)) return true;
        if (*reinterpret_cast<volatile int *>(err) != 0) return false;
        if (globaltimer() - t0 > wait_limit_ns(err)) {
            record_timeout(err, code, bar, parity, t0, c0);
            return false;
        }
    }
}

// Bounded cluster-scope wait for work already issued (teardown): does not give
// up on another thread's error, only on the time limit (as mbar_wait_issued).
__device__ __forceinline__ bool mbar_wait_cluster_issued(uint64_t *bar, uint32_t parity, int *err, int code) {
    const uint64_t t0 = globaltimer();
    const uint32_t c0 = uint32_t(clock64());
    while (true) {
        if (mbar_try_wait_cluster(bar, parity, kSuspendHintNs)) return true;
        if (globaltimer() - t0 > wait_limit_ns(err)) {
            record_timeout(err, code, bar, parity, t0, c0);
            return false;
        }
    }
}

// 2-D TMA tile load into this CTA's shared memory whose completion (bytes) is
// counted on an mbarrier of either CTA of the pair (`bar_cluster`, a
// shared::cluster address), as the 2-SM MMA's producers need.  Every CTA loads
// its own tiles: no cluster-wide broadcast form.
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map, int32_t c0, int32_t c1,
                                                 uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
        : "memory");
}

// TMEM allocation shared by the CTA pair: the same warp of both CTAs executes it.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 2-SM MMA issued by the pair's first CTA: D (M = 256: 128 rows in each CTA's
// TMEM, all N columns) (+)= A (each CTA's shared memory holds its 128 rows) * B
// (each CTA's shared memory holds N/2 of the rows of B^T); kind::f16.
__device__ __forceinline__ void mma_ss_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One arrival on the mbarrier at the same offset in every CTA of `cta_mask` when
// all 2-SM MMAs issued so far by this thread complete (a completion signal, not a load).
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// Pack two fp32 into 16-bit pairs (lo in bits 0-15), round-to-nearest-even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

}  // namespace sm100
}  // namespace stratum
