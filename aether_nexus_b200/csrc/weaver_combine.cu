// weaver_combine.cu — split-KV combine across the GPUs of one node over
// NVLink peer memory, in one kernel: every rank writes its packed (m, l, o)
// partials straight into every peer's receive buffer, publishes an epoch
// flag in each peer's memory, waits (bounded) until every peer's flag for
// this epoch has arrived in its own memory, and merges by log-sum-exp.
//
// Memory per rank (one cudaMalloc, exported with cudaIpcGetMemHandle and
// opened by the peers with cudaIpcOpenMemHandle — plain peer mappings):
//   recv   [2][world][slot] fp32             double-buffered by epoch parity;
//                                            slot = rows * (D + 2) rounded up to 4
//   flags  [world] u32                       last epoch received from rank p
//   state  [2] u32                           epoch counter, status word
// Ordering: a rank writes its partials for epoch e into every peer's buffer
// e & 1, synchronises the CTA, and one thread issues a system-scope release
// fence and stores e into every peer's flags[rank]; the reader polls its own
// flags and issues a system-scope acquire fence before its CTA reads the
// buffer.  A rank can only start epoch e + 2 after every peer signalled
// epoch e + 1, which each peer does after finishing its epoch-e merge, so
// buffer e & 1 is never overwritten while it is being read.
// That argument needs every earlier wait to have succeeded: once a wait has
// timed out (status word set) a late peer may still write into a buffer, so
// from then on every run of this combiner writes zeros and touches no peer
// memory; the combiner must be destroyed and recreated by every rank.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kCombineThreads = 1024;
constexpr uint32_t kCombineMaxRows = 1024;   // rows whose statistics fit the shared tables
constexpr uint64_t kCombineWaitNs = 1000ull * 1000 * 1000;  // 1 s

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kCombineThreads) combine_kernel(CombineArgs c, const float* __restrict__ packed,
                                                                  __half* __restrict__ out) {
    __shared__ uint32_t s_epoch, s_ok;
    __shared__ float s_f[kCombineMaxRanks][kCombineMaxRows / 4];  // per-part factor of each row (chunked)
    __shared__ float s_l[kCombineMaxRows / 4];                      // merged l of each row (chunked)
    // a programmatic dependent launch: placed early, it starts work only once
    // the step kernel that wrote `packed` has completed; the next step may be
    // placed as soon as this kernel starts
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t tid = threadIdx.x;
    const uint32_t part = c.rows * (c.D + 2);  // floats of one rank's packed partials
    const uint32_t slot = (part + 3) & ~3u;    // 16-byte aligned slots
    if (tid == 0) {
        s_epoch = c.state[0] + 1;
        s_ok = *reinterpret_cast<volatile uint32_t*>(&c.state[1]) == 0u;
    }
    __syncthreads();
    if (!s_ok) {
        // an earlier wait expired: this combiner is unusable (see above)
        for (uint32_t i = tid; i < c.rows * c.D; i += kCombineThreads) out[i] = __float2half_rn(0.0f);
        return;
    }
    const uint32_t epoch = s_epoch, buf = epoch & 1u;
    // 1. this rank's partials into slot [rank] of every peer's buffer (self included)
    for (uint32_t p = 0; p < c.world; ++p) {
        float* dst = c.recv[p] + (static_cast<uint64_t>(buf) * c.world + c.rank) * slot;
        for (uint32_t j = tid; j < part / 4; j += kCombineThreads)
            reinterpret_cast<float4*>(dst)[j] = __ldcg(reinterpret_cast<const float4*>(packed) + j);
        for (uint32_t i = (part / 4) * 4 + tid; i < part; i += kCombineThreads) dst[i] = __ldcg(packed + i);
    }
    __syncthreads();
    if (tid == 0) {
        // 2. publish: flags[rank] = epoch in every peer's memory.  The barrier
        // puts every thread's writes above before this thread's release fence,
        // which is cumulative: one system-scope fence covers the whole CTA.
        fence_acq_rel_sys();
        for (uint32_t p = 0; p < c.world; ++p) st_relaxed_sys(c.flags[p] + c.rank, epoch);
        // 3. wait (bounded) until every rank's epoch has arrived here, then
        // one acquire fence before anyone reads the buffer
        const uint64_t t0 = globaltimer_ns();
        for (uint32_t p = 0; p < c.world; ++p) {
            const uint32_t* f = c.flags[c.rank] + p;
            while (static_cast<int32_t>(ld_relaxed_sys(f) - epoch) < 0) {
                if (globaltimer_ns() - t0 > kCombineWaitNs) {
                    atomicOr(&c.state[1], 1u);
                    s_ok = 0;
                    break;
                }
            }
        }
        fence_acq_rel_sys();
    }
    __syncthreads();
    if (tid == 0) c.state[0] = epoch;
    // 4. merge, in chunks of kCombineMaxRows / 4 rows: per-row factors and l
    // into shared memory, then every output with its parts' loads in flight
    const float* base = c.recv[c.rank] + static_cast<uint64_t>(buf) * c.world * slot;
    constexpr uint32_t kRowsPer = kCombineMaxRows / 4;
    for (uint32_t r0 = 0; r0 < c.rows; r0 += kRowsPer) {
        const uint32_t nr = min(kRowsPer, c.rows - r0);
        for (uint32_t r = tid; r < nr; r += kCombineThreads) {
            const uint32_t row = r0 + r;
            float mv[kCombineMaxRanks];
            float M = -INFINITY;
#pragma unroll
            for (uint32_t p = 0; p < kCombineMaxRanks; ++p) {
                mv[p] = p < c.world ? __ldcg(base + p * slot + row) : -INFINITY;
                M = fmaxf(M, mv[p]);
            }
            float L = 0.0f;
#pragma unroll
            for (uint32_t p = 0; p < kCombineMaxRanks; ++p) {
                const float f = p < c.world ? exp_shift(mv[p], M) : 0.0f;
                if (p < c.world) L += __ldcg(base + p * slot + c.rows + row) * f;
                s_f[p][r] = f;
            }
            s_l[r] = s_ok ? L : 0.0f;
        }
        __syncthreads();
        for (uint32_t idx = tid; idx < nr * c.D; idx += kCombineThreads) {
            const uint32_t r = idx / c.D, dim = idx % c.D, row = r0 + r;
            float v[kCombineMaxRanks];
#pragma unroll
            for (uint32_t p = 0; p < kCombineMaxRanks; ++p)
                v[p] = p < c.world ? __ldcg(base + p * slot + 2 * c.rows + static_cast<uint64_t>(row) * c.D + dim) : 0.0f;
            float O = 0.0f;
#pragma unroll
            for (uint32_t p = 0; p < kCombineMaxRanks; ++p) O = fmaf(s_f[p][r], v[p], O);
            const float L = s_l[r];
            out[static_cast<uint64_t>(row) * c.D + dim] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_combine(const CombineArgs& c, const float* packed, __half* out, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kCombineThreads);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, combine_kernel, c, packed, out);
}

}  // namespace weaver
