// weaver_device.cuh — sm_100a device helpers shared by the Weaver kernels:
// TMA tensor loads into shared memory, mbarrier transaction barriers with
// bounded waits, f16 conversion and vector reductions.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "weaver_internal.hpp"

namespace weaver {

// Every spin on an mbarrier or a dependency counter gives up after
// kWaitNs of wall time (%globaltimer), or at once when another wait of the
// same launch has already given up (DEVERR_TIMEOUT in the status word).  The
// caller then skips the work that depended on the wait and winds down, so a
// lost arrival costs at most kWaitNs per CTA instead of hanging the GPU.
constexpr uint64_t kWaitNs = 500ull * 1000 * 1000;

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

__device__ __forceinline__ bool timed_out(const uint32_t* status) {
    return (*reinterpret_cast<const volatile uint32_t*>(status) & DEVERR_TIMEOUT) != 0;
}

// Records an expired wait: DEVERR_TIMEOUT in status[0] and, for the first
// one only, (1 << 31) | (CTA << 8) | site in status[1], so the host can say
// which wait expired.
__device__ __forceinline__ void note_timeout(uint32_t* status, uint32_t site) {
    atomicOr(status, DEVERR_TIMEOUT);
    atomicCAS(status + 1, 0u, 0x80000000u | (blockIdx.x << 8) | (site & 0xFFu));
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and records the
// timeout with `site`) if the phase did not complete in time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t site = 0,
                                          uint64_t limit_ns = kWaitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (timed_out(status)) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                note_timeout(status, site);
                return false;
            }
        }
    }
}

// Wait for the last phase of a barrier whose earlier waits may have been
// abandoned: used only to drain a CTA's own copies before it exits.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > kWaitNs) return;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread spins (bounded) until *cnt >= target; false if it gave up.
__device__ __forceinline__ bool spin_until(const uint32_t* cnt, uint32_t target, uint32_t* status, uint32_t site,
                                           uint64_t limit_ns = kWaitNs) {
    if (ld_acquire_gpu(cnt) >= target) return true;
    const uint64_t start = globaltimer_ns();
    uint32_t ns = 32;
    while (ld_acquire_gpu(cnt) < target) {
        if (timed_out(status)) return false;
        if (globaltimer_ns() - start > limit_ns) {
            note_timeout(status, site);
            return false;
        }
        __nanosleep(ns);
        if (ns < 256) ns <<= 1;
    }
    return true;
}

__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_sys_v2(uint2* p, uint32_t x, uint32_t y) {
    asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ uint2 ld_relaxed_sys_v2(const uint2* p) {
    uint2 v;
    asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}

// Waits (bounded, like every wait here) until three (value, tag) words all
// carry `tag`; false, with DEVERR_TIMEOUT recorded, if they did not in time.
static __device__ __forceinline__ bool ll_wait3(const uint2* a, const uint2* b, const uint2* c, uint32_t tag, uint2& wa,
                                         uint2& wb, uint2& wc, uint32_t* status, uint64_t limit_ns = kWaitNs) {
    wa = ld_relaxed_sys_v2(a);
    wb = ld_relaxed_sys_v2(b);
    wc = ld_relaxed_sys_v2(c);
    if (wa.y == tag && wb.y == tag && wc.y == tag) return true;
    const uint64_t start = globaltimer_ns();
    uint32_t ns = 32;
    for (;;) {
        if (wa.y != tag) wa = ld_relaxed_sys_v2(a);
        if (wb.y != tag) wb = ld_relaxed_sys_v2(b);
        if (wc.y != tag) wc = ld_relaxed_sys_v2(c);
        if (wa.y == tag && wb.y == tag && wc.y == tag) return true;
        if (timed_out(status)) return false;
        if (globaltimer_ns() - start > limit_ns) {
            note_timeout(status, 26);
            return false;
        }
        __nanosleep(ns);
        if (ns < 128) ns <<= 1;
    }
}


// 2-D tiled TMA load of box (c0 = innermost element, c1 = row) into shared
// memory, completing `bar`'s transaction count.  c0 * element size must be a
// multiple of 16 bytes (callers pass multiples of 64 f16 elements).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 1-D bulk copy (TMA engine, no tensor map) of `bytes` (multiple of 16, both
// addresses 16-byte aligned) into shared memory, completing `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Named barrier over `count` threads (a warp-aligned subset of the block).
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Counter updates with release (and acquire) semantics at gpu scope: the
// ordering of a fence and an atomic in one operation.
__device__ __forceinline__ void red_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Order-preserving float <-> int keys, so atomicMax on ints is a max on floats.
__device__ __forceinline__ int fkey(float f) {
    const int i = __float_as_int(f);
    return i >= 0 ? i : (i ^ 0x7FFFFFFF);
}
__device__ __forceinline__ float unkey(int k) { return __int_as_float(k >= 0 ? k : (k ^ 0x7FFFFFFF)); }

__device__ __forceinline__ void red_add_v2(float* addr, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(addr), "f"(a), "f"(b) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a TMA box
// written with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows): chunks are XOR-ed
// with the row index modulo 8.
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void h8_to_f8(const uint4 raw, float f[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

__device__ __forceinline__ void h4_to_f4(const uint2 raw, float f[4]) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
    const float2 a = __half22float2(h[0]);
    const float2 b = __half22float2(h[1]);
    f[0] = a.x;
    f[1] = a.y;
    f[2] = b.x;
    f[3] = b.y;
}

__device__ __forceinline__ float h2f(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

// Vector reduction into global memory (sm_90+): four independent fp32 adds.
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

// ---- tensor-core fragments (mma.sync m16n8k16, f16 inputs, fp32 accumulate) ----

// Four 8x8 b16 matrices from shared memory; lane L gives the row address of
// row L % 8 of matrix L / 8.
__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(row_addr)));
}

// Four 8x8 b16 matrices, each transposed on the way (lane T receives rows
// 2(T%4), 2(T%4)+1 of column T/4 of the stored matrix).
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t r[4], const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(row_addr)));
}

// c += a (16x16, row-major) * b (16x8, column-major); f16 inputs, fp32 c.
// a0..a3: (row gid, k 2tig..) (row gid+8, k 2tig..) (row gid, k 8+2tig..) (row gid+8, k 8+2tig..).
__device__ __forceinline__ void mma_16816(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    mma_16816(c, a[0], a[1], a[2], a[3], b0, b1);
}

// ---- proxy fences and bulk (TMA engine) reductions ----

// Orders this thread's generic-proxy accesses to global memory with later
// async-proxy (bulk copy / bulk reduce) accesses, and the reverse.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// 16-byte asynchronous copy global -> shared (L2 only), tracked per thread.
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the barrier's expected count must include this arrival).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 16-byte cp.async that writes zeros instead when !valid (no bytes read).
__device__ __forceinline__ void cp_async16_zfill(void* sdst, const void* gsrc, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sdst)), "l"(gsrc),
                 "r"(valid ? 16u : 0u)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Every group but the most recent one committed by this thread has landed.
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy / bulk reduce) reads of them.
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk (TMA engine) element-wise fp32 add of `bytes` (multiple of 16, both
// addresses 16-byte aligned) of shared memory into global memory, tracked by
// this thread's bulk group.
__device__ __forceinline__ void bulk_reduce_add_f32(void* gdst, const void* ssrc, uint32_t bytes) {
    asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst),
                 "r"(smem_u32(ssrc)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Every committed bulk operation of this thread has finished reading its source.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Every committed bulk operation of this thread has completed (writes performed).
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Bring `bytes` (multiple of 16, 16-byte aligned) of global memory into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gsrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// exp(x - m) that is 0 when m is -inf (an empty or fully masked run, where x
// is -inf too).  Written without a select on the result: m = -inf is replaced
// by +inf, so the exponent is -inf and the exponential 0; a conditional on the
// result made the compiler wrap every exponential in control flow, which made
// loops over it 2.3x slower (measured on a 1600-token softmax pass).
__device__ __forceinline__ float exp_shift(float x, float m) {
    return __expf(x - (m == -INFINITY ? INFINITY : m));
}

}  // namespace weaver
