// Device-side building blocks shared by every sm_100a kernel in libdotl.
//
// Everything here is a thin, named wrapper over one PTX instruction (mbarrier,
// TMA bulk-tensor copies, tcgen05 MMA / TMEM traffic) plus the two descriptor
// encoders the tensor cores read. The library is one translation unit
// (dotl.cu includes every kernel header), so the device error word below has a
// single definition.
//
// Every spin-wait in this library is bounded: a wait that has not completed
// after kWaitLimitNs sets a CTA-wide abort flag and a bit in g_dotl_dev_error,
// and every role of the kernel then drains to its teardown, frees its TMEM and
// returns. The host reads the error word with dotl_device_error().

#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace dotl {

// Sticky device error word, or-ed by kernels that gave up a wait.
__device__ unsigned int g_dotl_dev_error = 0;

enum DevError : unsigned int {
    kDevErrWaitTimeout = 1u,   // an mbarrier phase did not complete in time
    kDevErrBadLaunch = 2u,     // a kernel was launched with arguments it rejects
};

// Two seconds of wall time. Nothing a correct launch waits for comes within
// three orders of magnitude of this.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier --

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes initialised barriers visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrives `count` times at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with parity `parity` to complete. Returns false
// (and raises the CTA abort flag) if it has not completed within kWaitLimitNs,
// or at once if another thread of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            atomicOr(&g_dotl_dev_error, kDevErrWaitTimeout);
            return false;
        }
    }
}

// Same wait, without looking at the abort flag: teardown uses it to drain
// copies that are still in flight after an abort.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// ----------------------------------------------------- thread-block clusters --
// Distributed shared memory: a CTA reaches a peer's shared memory through the
// shared::cluster window (mapa), stores there, and arrives on the peer's
// mbarriers with release semantics at cluster scope; the peer waits on its own
// barrier with acquire at cluster scope. Every CTA loads its own tiles.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of local shared address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void st_cluster_v2f32(uint32_t caddr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(caddr), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ void st_cluster_v4f32(uint32_t caddr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(caddr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

// Arrives on an mbarrier of a peer CTA (shared::cluster address), ordering this
// thread's earlier stores (remote ones included) before the arrival.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait for barriers that peers arrive on: acquire at cluster scope, so the
// peers' stores into this CTA's shared memory are visible afterwards. Bounded
// like mbar_wait (limit_ns), and returns at once if this CTA aborted.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (abort_flag != nullptr && *abort_flag) return false;
        if (global_ns() - t0 > limit_ns) {
            if (abort_flag != nullptr) *abort_flag = 1;
            atomicOr(&g_dotl_dev_error, kDevErrWaitTimeout);
            return false;
        }
    }
}

// Every thread of every CTA of the cluster, once, right after the barriers
// are initialised (before any peer may arrive on them). Nothing precedes it
// that could stall: all CTAs of a cluster are launched together.
__device__ __forceinline__ void cluster_sync_after_init() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------- programmatic dependent launch --
// Kernels are launched with programmatic stream serialization: the next kernel
// in the stream may start its prologue while this one drains. pdl_wait() blocks
// until every kernel this one depends on has completed and its writes are
// visible; it must precede the first read of a predecessor's output (and every
// TMEM allocation, so a waiting CTA never holds tensor memory).
// pdl_launch_dependents() lets the next kernel begin launching; its own
// pdl_wait() still waits for this kernel's completion.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Per-warpgroup register budget (all four warps of a warpgroup execute it).
template <int N>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }

// --------------------------------------------------------------------- TMA --

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

// Shared -> global tensor store (bulk-group completion); clips at the tensor
// bounds. The smem source must not be rewritten before bulk_wait_read().
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(src)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N committed bulk groups of this thread still reading shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every committed bulk group of this thread complete (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ----------------------------------------------------------------- tcgen05 --

__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// ------------------------------------------------ CTA pairs (cta_group::2) --
// Two CTAs of a cluster run one M=256 MMA: each holds 128 rows of A, half of
// B's rows and 128 rows of the accumulator in its own TMEM. The leader (rank
// 0) issues the MMAs and commits; every CTA loads its own operand halves.

// TMEM allocation for the pair (one warp of each CTA, the same warp index and
// the same destination offset in both).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// A tile into this CTA's shared memory whose completion (bytes) is counted on
// the mbarrier at shared::cluster address `bar_cluster` (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
        : "memory");
}

// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both], M = 256, issued
// by the leader alone.
__device__ __forceinline__ void mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the mbarrier at shared::cluster address `bar` (this CTA's
// or the peer's) when the pair MMAs this thread issued so far have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem], fp16 inputs, fp32 accumulate. One thread issues.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Instruction descriptor for kind::f16 with fp16 A/B and an fp32 accumulator.
// Bit layout (PTX ISA, "Instruction descriptor" for .kind::f16): c_format at
// [4,6) = 1 (F32), a/b format at [7,10)/[10,13) = 0 (F16), a/b major at bits
// 15/16 (0 = K-major, 1 = MN-major), N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Shared-memory matrix descriptor (PTX ISA "Shared memory descriptor"):
// start address >> 4 at [0,14), leading byte offset >> 4 at [16,30), stride
// byte offset >> 4 at [32,46), version 1 at [46,48), layout at [61,64).
enum SmemLayout : uint32_t { kSwizzleNone = 0, kSwizzle128 = 2, kSwizzle64 = 4, kSwizzle32 = 6 };

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
           (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (static_cast<uint64_t>(layout) << 61);
}

// 32 lanes x 32 consecutive 32-bit TMEM columns: thread t of the warp gets row
// (lane base + t), columns [col, col + 32). Warp-collective.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// D[tmem] (+)= A[tmem] * B[smem]: the A operand (M=128 rows in lanes, K fp16
// values packed two per 32-bit column, lower k in the low half) read from
// tensor memory. One thread issues.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit TMEM columns from registers (warp-collective).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns from registers (warp-collective).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Completes every outstanding tcgen05.st of this thread.
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns (warp-collective).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// Completes every outstanding tcgen05.ld of this thread. The registers are
// tied to the wait so the compiler cannot read them before it.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// -------------------------------------------------------------- arithmetic --

// Exact (erf) GELU, the form F.gelu(approximate="none") computes, using
// CUDA's erff.
__device__ __forceinline__ float gelu_erf(float v) {
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
}

// GELU(v) = 0.5 v (1 + erf(v / sqrt 2)) with erf from Abramowitz & Stegun,
// Handbook of Mathematical Functions, formula 7.1.28 (Hastings):
// erf(x) = 1 - R(x), R(x) = (1 + a1 x + ... + a6 x^6)^-16, |error| <= 3e-7.
// With u = |v| and Q = R(u / sqrt 2) / 2, both sign cases collapse to
//   GELU(v) = max(v, 0) - u Q
// (v >= 0: v - v R/2; v < 0: v R/2). Q comes from one polynomial whose
// coefficients absorb the 1/sqrt 2 argument scale (a_i 2^(-i/2)) and the 1/2
// (a factor 2^(1/16) on every coefficient, since Q = (2^(1/16) P)^-16): six
// FMAs, four squarings, one fast reciprocal, one max and one FMA. Agrees with
// the float64 erf GELU to 7.1e-7 absolute over [-12, 12] (the GPU test checks
// 1e-6 (1 + |v|)). For large u, P^16 overflows to +inf and Q to 0, giving
// max(v, 0).
__device__ __forceinline__ float gelu_fast(float v) {
    const float u = fabsf(v);
    float t = fmaf(u, 5.6212997e-06f, 5.1055209e-05f);
    t = fmaf(t, u, 3.9686137e-05f);
    t = fmaf(t, u, 3.4227392e-03f);
    t = fmaf(t, u, 2.2076998e-02f);
    t = fmaf(t, u, 5.2075163e-02f);
    t = fmaf(t, u, 1.0442738f);
    t = t * t;
    t = t * t;
    t = t * t;
    t = t * t;
    return fmaf(-u, __fdividef(1.0f, t), fmaxf(v, 0.0f));
}

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic: two IEEE fp32 lanes per
// instruction, each lane exactly what the scalar fmaf / fmul computes)
__device__ __forceinline__ unsigned long long f32x2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f32x2_split(unsigned long long r, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ unsigned long long fma_x2(unsigned long long a, unsigned long long b,
                                                      unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long mul_x2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// gelu_fast on two values at once: the polynomial, the squarings and the
// final FMA run as f32x2 instructions (half the issue slots of the scalar
// form, the same per-lane arithmetic); the reciprocal and the max stay scalar.
__device__ __forceinline__ void gelu_fast_pair(float& v0, float& v1) {
    const float u0 = fabsf(v0), u1 = fabsf(v1);
    const unsigned long long u = f32x2(u0, u1);
    unsigned long long t = fma_x2(u, f32x2(5.6212997e-06f, 5.6212997e-06f), f32x2(5.1055209e-05f, 5.1055209e-05f));
    t = fma_x2(t, u, f32x2(3.9686137e-05f, 3.9686137e-05f));
    t = fma_x2(t, u, f32x2(3.4227392e-03f, 3.4227392e-03f));
    t = fma_x2(t, u, f32x2(2.2076998e-02f, 2.2076998e-02f));
    t = fma_x2(t, u, f32x2(5.2075163e-02f, 5.2075163e-02f));
    t = fma_x2(t, u, f32x2(1.0442738f, 1.0442738f));
    t = mul_x2(t, t);
    t = mul_x2(t, t);
    t = mul_x2(t, t);
    t = mul_x2(t, t);
    float t0, t1;
    f32x2_split(t, t0, t1);
    const unsigned long long r =
        fma_x2(f32x2(-u0, -u1), f32x2(rcp_approx(t0), rcp_approx(t1)), f32x2(fmaxf(v0, 0.0f), fmaxf(v1, 0.0f)));
    f32x2_split(r, v0, v1);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// The fp16 pair of (a, b) for the three-product GEMM mode: hi = fp16(v) and
// lo = fp16(v - hi), both round to nearest even, so hi + lo carries v to about
// 22 bits (a product a w then splits into a_hi w_hi + a_lo w_hi + a_hi w_lo,
// dropping only a_lo w_lo).
__device__ __forceinline__ void split_half2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

}  // namespace dotl
