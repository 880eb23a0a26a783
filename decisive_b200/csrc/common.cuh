// Shared device helpers for the sm_100a kernels: PTX wrappers for mbarriers, TMA, tcgen05
// (tensor memory + UMMA), bounded waits, and the device-side layout constants.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define DB_GROUP 64

// Device error word bits (written with atomicOr; read back by the host after a launch).
#define DB_DEV_ERR_TIMEOUT_TMA 0x1
#define DB_DEV_ERR_TIMEOUT_MMA 0x2
#define DB_DEV_ERR_TIMEOUT_CVT 0x4
#define DB_DEV_ERR_TIMEOUT_EPI 0x8
#define DB_DEV_ERR_SHAPE 0x10

// A wait on an mbarrier gives up after this many nanoseconds; a legitimate wait in these
// kernels lasts microseconds.  On expiry the kernel records the error and winds down.
#define DB_WAIT_LIMIT_NS 2000000000ull

namespace db {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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
// Non-blocking test of the same condition (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait.  Returns false when the CTA was aborted (by this or another thread) or the
// limit expired; in the latter case the abort flag and the device error word are set.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        // plain try_wait: with a suspend-time hint the thread was observed to wake microseconds
        // after the phase completed
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// Tests two mbarrier phases with both tests in flight at once (one asm block: the second test does
// not wait for the first one's result); bit 0 / bit 1 of the return value: phase of a / b done.
__device__ __forceinline__ uint32_t mbar_test_wait2(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb) {
    uint32_t ra, rb;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%2], %3;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%4], %5;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "selp.u32 %1, 2, 0, q;\n\t}"
        : "=r"(ra), "=r"(rb)
        : "r"(smem_u32(a)), "r"(pa), "r"(smem_u32(b)), "r"(pb)
        : "memory");
    return ra | rb;
}
// Four phases tested with all four tests in flight; bits 0-3 of the return value.
__device__ __forceinline__ uint32_t mbar_test_wait4(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb, uint64_t* c,
                                                    uint32_t pc, uint64_t* d, uint32_t pd) {
    uint32_t ra, rb, rc, rd;
    asm volatile(
        "{\n\t.reg .pred p, q, r, s;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%4], %5;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 q, [%6], %7;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 r, [%8], %9;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 s, [%10], %11;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "selp.u32 %1, 2, 0, q;\n\t"
        "selp.u32 %2, 4, 0, r;\n\t"
        "selp.u32 %3, 8, 0, s;\n\t}"
        : "=r"(ra), "=r"(rb), "=r"(rc), "=r"(rd)
        : "r"(smem_u32(a)), "r"(pa), "r"(smem_u32(b)), "r"(pb), "r"(smem_u32(c)), "r"(pc), "r"(smem_u32(d)), "r"(pd)
        : "memory");
    return ra | rb | rc | rd;
}
// Bounded waits for two or four phases (as mbar_spin, for every barrier given); a phase seen
// complete stays counted.
__device__ __forceinline__ bool mbar_spin2(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb,
                                           volatile int* abort_flag, int* err, int code) {
    uint32_t done = mbar_test_wait2(a, pa, b, pb);
    if (done == 3u) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        done |= mbar_test_wait2(a, pa, b, pb);
        if (done == 3u) return true;
        if ((i & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}
__device__ __forceinline__ bool mbar_spin4(uint64_t* a, uint32_t pa, uint64_t* b, uint32_t pb, uint64_t* c,
                                           uint32_t pc, uint64_t* d, uint32_t pd, volatile int* abort_flag, int* err,
                                           int code) {
    uint32_t done = mbar_test_wait4(a, pa, b, pb, c, pc, d, pd);
    if (done == 15u) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        done |= mbar_test_wait4(a, pa, b, pb, c, pc, d, pd);
        if (done == 15u) return true;
        if ((i & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// Bounded wait that never suspends the thread (mbarrier.test_wait in a loop): for waits on the
// critical path, where a thread suspended in try_wait was measured to resume 0.3-1.4 us after the
// phase completed.  Poll from one lane per warp.
__device__ __forceinline__ bool mbar_spin(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// The same poll with a short sleep after every failed test: for waiters that share their SM
// sub-partition with a latency-critical warp (the MMA issuer), so that polling does not take its
// issue slots.
__device__ __forceinline__ bool mbar_spin_polite(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                                 int code) {
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(32);
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 15u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// Bounded wait that ignores the abort flag: used while winding down after an abort, to let this
// thread's own asynchronous copies or MMAs land before the CTA releases its memory.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t start = globaltimer();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer() - start > limit_ns) return false;
    return true;
}

// Programmatic dependent launch: a kernel launched with the programmatic-serialization attribute
// (db_launch_pdl) may be scheduled while the previous kernel in its stream is still finishing; it
// waits here, before touching anything, until that kernel has completed and its writes are
// visible.  Returns at once for a launch without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the stream (launched with programmatic dependent launch) start once every
// CTA of this grid has passed here; it still waits (pdl_wait) for this grid's completion before it
// reads anything this grid writes.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Hardware named barrier among `count` threads (a multiple of 32); barrier 0 is __syncthreads.
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ------------------------------------------------------------------ cp.async (per-thread, 16 B)
__device__ __forceinline__ void cp_async16(uint32_t dst_smem, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst_smem), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ------------------------------------------------------------------ shared-window loads
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(addr));
    return r;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// ------------------------------------------------------------------ packed f32x2 arithmetic
// Two independent IEEE binary32 operations, each rounded to nearest even: bit-identical to the
// scalar __fmul_rn / __fmaf_rn / __fadd_rn on each half, at half the instruction count.
__device__ __forceinline__ uint64_t f2_pack(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Bounded wait for roles that run ahead of the pipeline (producer, converters): after the first
// failed test the thread sleeps between polls, leaving issue slots and the barrier unit to the
// latency-critical roles (MMA issuer, epilogue) that share its SM sub-partition.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(128);
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer() - start > DB_WAIT_LIMIT_NS) {
                *abort_flag = 1;
                atomicOr(err, code);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------ fences
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ TMA (no multicast)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Tensor store / reduce-add shared -> global (bulk-group completion, issued by one thread).
// x is the innermost coordinate; x * element size must be a multiple of 16 bytes and both
// coordinates non-negative.  Elements outside the tensor are skipped.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src_smem, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(src_smem), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src_smem, int x, int y) {
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src_smem), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until all of this thread's bulk groups have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16), completion
// counted on an mbarrier's transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, one CTA.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier once every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Waits for prior tcgen05.ld and ties the loaded registers to the wait, so the compiler cannot
// move any use of them above it (the ld's outputs are only valid after tcgen05.wait::ld).
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
          "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
          "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
          "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
        :
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base lane + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[8]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7])
                 :
                 : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b(uint32_t taddr, uint32_t (&r)[8]) { tmem_ld_32x32b_x8(taddr, r); }
__device__ __forceinline__ void tmem_ld_32x32b(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld_32x32b_x16(taddr, r); }
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}

// ------------------------------------------------------------------ CTA pairs (cluster of 2)
// A pair of CTAs shares one MMA of M = 256: each CTA holds 128 rows of A and half of B in its own
// shared memory and its own 128 TMEM lanes of D; the even CTA (rank 0) issues the MMA.  Barriers
// of the other CTA are addressed through mapa (no multicast is used anywhere).
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
                 "r"(bytes)
                 : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on a barrier that may live in
// the peer CTA of the pair (cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A * B^T over the pair: M = 256 (128 rows per CTA), B split by N across the CTAs.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive (once) on the barrier at a cluster address when every pair MMA issued so far has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of 128 bytes,
// 8-row atoms 1024 bytes apart.  Start address must sit in a 1024-byte aligned atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;                    // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;          // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1u << 46;                    // descriptor version (tcgen05)
    d |= (uint64_t)2u << 61;                    // SWIZZLE_128B
    return d;
}

// Instruction descriptor for kind::f16: A,B f16 K-major, D f32, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
    return (1u << 4)                            // D format f32
           | (0u << 7) | (0u << 10)             // A, B f16
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ tcgen05 kind::i8
// Instruction descriptor for kind::i8: A and B signed 8-bit, K-major, D s32, shape M x N.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int M, int N) {
    return (2u << 4)                            // D format s32
           | (1u << 7) | (1u << 10)             // A, B signed 8-bit
           | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (K = 32 per instruction), one CTA.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The same over a CTA pair: M = 256 (128 rows per CTA), B split by N across the two CTAs.
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns, every one set to v (thread i writes lane base + i).
__device__ __forceinline__ void tmem_st_32x32b_x32_fill(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
            taddr),
        "r"(v)
        : "memory");
}
// 32 lanes x 64 consecutive 32-bit columns, every one set to v.
__device__ __forceinline__ void tmem_st_32x32b_x64_fill(uint32_t taddr, uint32_t v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], "
        "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
        "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(
            taddr),
        "r"(v)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace db
