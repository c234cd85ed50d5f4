// common.cuh -- device helpers for the sm_100a kernels of libugbsa.
//
// Inline-PTX wrappers for mbarriers, TMA tensor loads, the tcgen05 tensor-core
// path (TMEM alloc / MMA / commit / ld / st) and shared-memory matrix
// descriptors.  Every wait on an mbarrier is bounded in wall time (globaltimer):
// on expiry the waiting thread records UGBSA_DEV_ERR_TIMEOUT in the kernel's
// error word and returns false, and the kernel winds down (drains its own TMA
// copies, frees its TMEM) instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#define UGBSA_BLOCK 64

// Device-side error bits (OR-ed into the error word handed to each kernel).
#define UGBSA_DEV_ERR_TIMEOUT 0x1
#define UGBSA_DEV_ERR_BOUNDS 0x2

// Wall-time bound for one mbarrier wait: 2 s.  A healthy wait lasts
// nanoseconds to microseconds; this only ends a wait that can never finish.
#ifndef UGBSA_WAIT_LIMIT_NS
#define UGBSA_WAIT_LIMIT_NS 2000000000ull
#endif

namespace ugbsa {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous global -> shared copy (L2 only) and the wait for all of this thread's copies
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Error context of a CTA: `err` is the library's sticky device error word
// (read by the host), `abort` a CTA-local shared flag that tells the other
// threads of the CTA to stop waiting once one of them gave up.
struct WaitCtx {
    int *err;
    int *abort;
};

// Wait until the phase with the given parity has completed.  Returns false if
// it does not within the time limit (setting the timeout bit and the CTA's
// abort flag), or as soon as another thread of the CTA has given up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, WaitCtx c) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(a, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*(volatile int *)c.abort) return false;
            if (global_timer_ns() - t0 > UGBSA_WAIT_LIMIT_NS) {
                atomicOr(c.err, UGBSA_DEV_ERR_TIMEOUT);
                *(volatile int *)c.abort = 1;
                return false;
            }
        }
    }
}

// Bounded wait used while draining after an abort: ignores the abort flag.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity, int *err) {
    const uint32_t a = smem_u32(bar);
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if (mbar_try_wait(a, parity)) return true;
        if ((it & 63u) == 63u && global_timer_ns() - t0 > UGBSA_WAIT_LIMIT_NS) {
            atomicOr(err, UGBSA_DEV_ERR_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------- TMA
// 4-D tiled tensor load into shared memory, completion counted on `bar`.
// Coordinates are in elements, innermost first.  The innermost coordinate
// must be a multiple of 16 bytes' worth of elements (callers pass 0 or 64).
__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}

// TMA tile store shared -> global (bulk group); rows or columns outside the tensor are not written
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *smem_src, int c0, int c1, int c2,
                                             int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of this thread's committed bulk stores have been read
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads).
// Sequence tile of a call's local query tile t: the call covers pairs of
// consecutive tiles dealt with stride pair_stride from tile t_base (pair_stride
// 1: the contiguous tiles t_base, t_base + 1, ...).
__host__ __device__ __forceinline__ int seq_tile(int t, int t_base, int pair_stride) {
    return t_base + t + 2 * (t >> 1) * (pair_stride - 1);
}

// float -> uint32 whose unsigned order is the float order (-0 folded into +0,
// every NaN above +inf, as torch's sort places NaN first when descending).
__device__ __forceinline__ uint32_t ordered_key(float v) {
    v = __fadd_rn(v, 0.0f);
    if (v != v) return 0xffffffffu;
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t u) {
    const uint32_t b = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    return __uint_as_float(b);
}

// Three-input maximum (one instruction on sm_100; NaN inputs are dropped as by fmaxf)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// fp32 pairs in one 64-bit register (packed fma / add on sm_100)
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f32x2_split(uint64_t r, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma_x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd_x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fmul_x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Barrier over a subset of the CTA's warps (id 1..15; __syncthreads uses 0).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may become resident while its predecessor in the
// stream still runs; grid_dep_wait() returns once that predecessor has completed and
// its memory is visible (at once when there is no such dependency).
// grid_dep_launch() lets this grid's dependent start launching (it takes effect when
// every CTA of the grid has issued it or exited).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
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

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/fp16 in, fp32 acc).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Call right after tmem_wait_ld(): marks the loaded registers as (re)defined
// here, so the compiler cannot schedule their uses above the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 layout: version 1
// at bits 46-47, layout type 2 at bits 61-63).
//   K-major operand : rows of 128 B (64 bf16), 8-row groups `sbo` bytes apart;
//                     lbo unused (1).
//   MN-major operand: 64 contiguous elements per K row, 8 K rows per 1024 B;
//                     `sbo` = bytes between 8-row K groups, `lbo` = bytes between
//                     64-element MN groups.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   ab_bf16: 1 = bf16 operands, 0 = fp16.  a_mn / b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int ab_bf16, int a_mn, int b_mn) {
    return (1u << 4)                                   // D format f32
           | ((uint32_t)ab_bf16 << 7)                  // A format
           | ((uint32_t)ab_bf16 << 10)                 // B format
           | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

}  // namespace ugbsa
