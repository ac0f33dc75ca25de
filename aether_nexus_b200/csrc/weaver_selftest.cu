// weaver_selftest.cu — a self-test of the bounded device-side waits that every
// kernel of this library uses (mbarrier phases, dependency counters, and the
// (value, step tag) words peers write in the fused split-KV merge).  Each wait
// is pointed at a condition that nothing will ever satisfy, with a short
// limit; the test passes when every wait gives up on its own, records
// DEVERR_TIMEOUT in its status word and lets the kernel finish, so the CUDA
// context stays usable.  No counterpart in the reference (its kernel has no
// waits and no error path).
#include <cuda_runtime.h>

#include "weaver_cuda.h"
#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

// st: 3 status pairs (one per wait, so one expired wait does not cut the next
// short), cnt: a zeroed counter, word: a zeroed (value, tag) word, out[0]: a
// bitmask of the waits that returned false, out[1..3]: their durations (ns).
__global__ void wait_selftest_kernel(uint32_t* st, const uint32_t* cnt, const uint2* word, uint64_t limit_ns,
                                     uint64_t* out) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_barrier_init();
    uint64_t mask = 0;
    uint64_t t0 = globaltimer_ns();
    if (!mbar_wait(&bar, 0, st + 0, 30, limit_ns)) mask |= 1;  // no arrival ever comes
    uint64_t t1 = globaltimer_ns();
    if (!spin_until(cnt, 1u, st + 2, 31, limit_ns)) mask |= 2;  // the counter stays 0
    uint64_t t2 = globaltimer_ns();
    uint2 a, b, c;
    if (!ll_wait3(word, word, word, 7u, a, b, c, st + 4, limit_ns)) mask |= 4;  // tag 7 never written
    uint64_t t3 = globaltimer_ns();
    mbar_arrive(&bar);  // complete the phase before the CTA exits
    out[0] = mask;
    out[1] = t1 - t0;
    out[2] = t2 - t1;
    out[3] = t3 - t2;
}

}  // namespace
}  // namespace weaver

using namespace weaver;

extern "C" int weaver_wait_selftest(uint32_t limit_us, uint32_t* expired_mask, uint64_t* waited_ns,
                                    uint32_t* status_words) {
    if (!expired_mask || limit_us == 0 || limit_us > 1000000) return WEAVER_ERR_INVALID_ARGUMENT;
    uint8_t* buf = nullptr;
    const size_t bytes = 256;
    if (cudaMalloc(&buf, bytes) != cudaSuccess) return WEAVER_ERR_CUDA;
    int rc = WEAVER_OK;
    uint64_t host[4] = {0, 0, 0, 0};
    uint32_t st[6] = {0, 0, 0, 0, 0, 0};
    uint32_t* d_st = reinterpret_cast<uint32_t*>(buf);
    const uint32_t* d_cnt = reinterpret_cast<const uint32_t*>(buf + 64);
    const uint2* d_word = reinterpret_cast<const uint2*>(buf + 128);
    uint64_t* d_out = reinterpret_cast<uint64_t*>(buf + 192);
    if (cudaMemset(buf, 0, bytes) != cudaSuccess) rc = WEAVER_ERR_CUDA;
    if (rc == WEAVER_OK) {
        wait_selftest_kernel<<<1, 32>>>(d_st, d_cnt, d_word, static_cast<uint64_t>(limit_us) * 1000, d_out);
        if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
            cudaMemcpy(host, d_out, sizeof(host), cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(st, d_st, sizeof(st), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = WEAVER_ERR_CUDA;
    }
    cudaFree(buf);
    *expired_mask = static_cast<uint32_t>(host[0]);
    if (waited_ns)
        for (int i = 0; i < 3; ++i) waited_ns[i] = host[1 + i];
    if (status_words)
        for (int i = 0; i < 6; ++i) status_words[i] = st[i];
    return rc;
}
