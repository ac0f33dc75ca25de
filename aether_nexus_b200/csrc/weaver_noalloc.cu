// weaver_noalloc.cu — exact hot-pool decode attention that allocates nothing.
//
// Some callers cannot allocate device memory while they run: a serving loop
// that reserves its whole device-memory budget at start-up and forbids any
// later cudaMalloc/cudaFree (allocation latency and fragmentation in the
// token loop), or a host process whose device memory is owned by another
// allocator and which therefore may not call the CUDA allocator itself.  The
// plan-based entry points allocate their scratch when a plan is created, which
// such callers cannot do.  weaver_hot_decode_noalloc() computes the same
// split-KV attention over the hot pool, keeping its per-chunk (m, l, o)
// partials in a fixed array compiled into this library (kScratchFloats fp32,
// 2 MiB) that every GPU loading the library holds until the process exits.
//
// The caller passes inputs and outputs only.  The first call on a device
// looks up the device address of the array (cudaGetSymbolAddress, with that
// device current); that first call should come before any stream capture.
// Every call shares the one array, so calls whose kernels overlap on the GPU
// (different streams, or different host threads on one device) race and must
// be ordered by the caller.  Nothing in the array has to start at zero: each
// call writes every partial it later reads.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/weaver_cuda.h"
#include "weaver_device.cuh"

namespace weaver {
namespace {

constexpr uint32_t kScratchFloats = 1u << 19;  // 2 MiB of partials
constexpr uint32_t kMaxDevices = 64;
constexpr uint32_t kMaxChunks = 296;           // two waves of 148 SMs
constexpr uint32_t kMaxBlocks = 1u << 24;

// The scratch: host code must use the address from cudaGetSymbolAddress.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

std::mutex g_setup_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// Partials layout: [chunk][Hkv][G][2 + D]  (m, l, o[0..D)).
template <int D, int G>
__global__ void __launch_bounds__(128) noalloc_partial_kernel(const __half* __restrict__ q,
                                                              const __half* __restrict__ hk,
                                                              const __half* __restrict__ hv, uint64_t pool_blocks,
                                                              const uint32_t* __restrict__ refs, uint32_t n_blocks,
                                                              uint32_t blocks_per_chunk, uint32_t Hkv, float scale,
                                                              float* __restrict__ part, uint32_t* __restrict__ bad) {
    constexpr int VPL = D / 32;
    __shared__ float qs[G][D];
    __shared__ float ps[4][G][16];
    __shared__ float cm[4][G], cl[4][G], co[4][G][D];
    const uint32_t chunk = blockIdx.x, g = blockIdx.y;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x)
        qs[i / D][i % D] = __half2float(q[(static_cast<uint64_t>(g) * G + i / D) * D + i % D]) * scale;
    __syncthreads();
    const uint32_t b0 = chunk * blocks_per_chunk;
    const uint32_t b1 = min(b0 + blocks_per_chunk, n_blocks);
    const uint32_t tok = lane & 15, hf = lane >> 4;
    float m[G], ls[G], o[G][VPL];
#pragma unroll
    for (int r = 0; r < G; ++r) {
        m[r] = -INFINITY;
        ls[r] = 0.0f;
#pragma unroll
        for (int e = 0; e < VPL; ++e) o[r][e] = 0.0f;
    }
    for (uint32_t blk = b0 + warp; blk < b1; blk += 4) {
        const uint32_t phys = refs[blk] & WEAVER_REF_MASK;
        const bool ok = phys < pool_blocks;
        if (!ok && lane == 0) atomicOr(bad, 1u);
        const uint64_t row = (static_cast<uint64_t>(ok ? phys : 0) * 16 + tok) * Hkv + g;
        // q.K: lanes t and t+16 each take half of token t's dims
        float acc[G];
#pragma unroll
        for (int r = 0; r < G; ++r) acc[r] = 0.0f;
        const uint4* kr = reinterpret_cast<const uint4*>(hk + row * D + hf * (D / 2));
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
            float kf[8];
            h8_to_f8(ok ? kr[c] : make_uint4(0, 0, 0, 0), kf);
#pragma unroll
            for (int r = 0; r < G; ++r)
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[r] = fmaf(qs[r][hf * (D / 2) + c * 8 + e], kf[e], acc[r]);
        }
        float alpha[G];
#pragma unroll
        for (int r = 0; r < G; ++r) {
            acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 16);
            const float s = ok ? acc[r] : -INFINITY;
            float mx = s;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[r], mx);
            alpha[r] = exp_shift(m[r], mn);
            const float p = exp_shift(s, mn);
            ls[r] = ls[r] * alpha[r] + (lane < 16 ? p : 0.0f);
            m[r] = mn;
            if (lane < 16) ps[warp][r][tok] = p;
        }
        __syncwarp();
        // p.V: lane owns VPL consecutive dims of every token row
        const uint64_t vbase = (static_cast<uint64_t>(ok ? phys : 0) * 16) * Hkv + g;
#pragma unroll
        for (int r = 0; r < G; ++r)
#pragma unroll
            for (int e = 0; e < VPL; ++e) o[r][e] *= alpha[r];
        for (int t = 0; t < 16; ++t) {
            const __half* vr = hv + (vbase + static_cast<uint64_t>(t) * Hkv) * D + lane * VPL;
            float vf[VPL];
#pragma unroll
            for (int e = 0; e < VPL; ++e) vf[e] = ok ? __half2float(vr[e]) : 0.0f;
#pragma unroll
            for (int r = 0; r < G; ++r) {
                const float pt = ps[warp][r][t];
#pragma unroll
                for (int e = 0; e < VPL; ++e) o[r][e] = fmaf(pt, vf[e], o[r][e]);
            }
        }
        __syncwarp();
    }
#pragma unroll
    for (int r = 0; r < G; ++r) {
        const float lw = warp_sum(ls[r]);
        if (lane == 0) {
            cm[warp][r] = m[r];
            cl[warp][r] = lw;
        }
#pragma unroll
        for (int e = 0; e < VPL; ++e) co[warp][r][lane * VPL + e] = o[r][e];
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < G * D; i += blockDim.x) {
        const uint32_t r = i / D, dim = i % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, cm[w][r]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float f = exp_shift(cm[w][r], M);
            L += cl[w][r] * f;
            O += co[w][r][dim] * f;
        }
        float* pp = part + ((static_cast<uint64_t>(chunk) * Hkv + g) * G + r) * (2 + D);
        if (dim == 0) {
            pp[0] = M;
            pp[1] = L;
        }
        pp[2 + dim] = O;
    }
}

__global__ void noalloc_merge_kernel(const float* __restrict__ part, uint32_t chunks, uint32_t Hq, uint32_t D,
                                     __half* __restrict__ out) {
    const uint32_t h = blockIdx.x, dim = threadIdx.x;
    const uint64_t stride = static_cast<uint64_t>(Hq) * (2 + D);  // one chunk: all (g, r) rows
    const float* p = part + static_cast<uint64_t>(h) * (2 + D);
    float M = -INFINITY;
    for (uint32_t c = 0; c < chunks; ++c) M = fmaxf(M, p[c * stride]);
    float L = 0.0f, O = 0.0f;
    for (uint32_t c = 0; c < chunks; ++c) {
        const float f = exp_shift(p[c * stride], M);
        L += p[c * stride + 1] * f;
        O += p[c * stride + 2 + dim] * f;
    }
    out[static_cast<uint64_t>(h) * D + dim] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
}

template <int D, int G>
void launch_partial(dim3 grid, cudaStream_t s, const __half* q, const __half* hk, const __half* hv, uint64_t pb,
                    const uint32_t* refs, uint32_t n, uint32_t bpc, uint32_t Hkv, float scale, float* part,
                    uint32_t* bad) {
    noalloc_partial_kernel<D, G><<<grid, 128, 0, s>>>(q, hk, hv, pb, refs, n, bpc, Hkv, scale, part, bad);
}

}  // namespace
}  // namespace weaver

using namespace weaver;

extern "C" int weaver_hot_decode_noalloc(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, float scale,
                                         const void* q, const void* hot_k, const void* hot_v,
                                         uint64_t hot_pool_blocks, const uint32_t* hot_refs, uint32_t n_blocks,
                                         void* out, uint32_t* bad_ref_flag, void* stream) {
    if (!q || !hot_k || !hot_v || !out || !bad_ref_flag || (n_blocks && !hot_refs)) return WEAVER_ERR_INVALID_ARGUMENT;
    if (kv_heads == 0 || q_heads % kv_heads) return WEAVER_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(hot_k) | reinterpret_cast<uintptr_t>(hot_v)) & 15u)
        return WEAVER_ERR_MISALIGNED;
    const uint32_t G = q_heads / kv_heads;
    if ((head_dim != 64 && head_dim != 128) || (G != 1 && G != 2 && G != 4 && G != 8)) return WEAVER_ERR_UNSUPPORTED;
    // the per-chunk partials of one call must fit the fixed scratch array
    const uint64_t per_chunk = static_cast<uint64_t>(q_heads) * (2 + head_dim);
    if (n_blocks > kMaxBlocks || per_chunk > kScratchFloats) return WEAVER_ERR_CAPACITY;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= static_cast<int>(kMaxDevices))
        return WEAVER_ERR_NO_DEVICE;
    float* scratch;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess) {
                return WEAVER_ERR_CUDA;
            }
            g_scratch_ptr[dev] = static_cast<float*>(p);
        }
        scratch = g_scratch_ptr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    __half* o = static_cast<__half*>(out);
    if (n_blocks == 0) {
        // nothing to attend to: the reference's l > 0 guard gives zeros
        return cudaMemsetAsync(out, 0, static_cast<size_t>(q_heads) * head_dim * 2, s) == cudaSuccess
                   ? WEAVER_OK : WEAVER_ERR_CUDA;
    }
    uint32_t chunks = (n_blocks + 3) / 4;
    const uint32_t cap = static_cast<uint32_t>(kScratchFloats / per_chunk);
    if (chunks > kMaxChunks) chunks = kMaxChunks;
    if (chunks > cap) chunks = cap;
    const uint32_t bpc = (n_blocks + chunks - 1) / chunks;
    chunks = (n_blocks + bpc - 1) / bpc;
    const dim3 grid(chunks, kv_heads);
    const __half* qh = static_cast<const __half*>(q);
    const __half* kh = static_cast<const __half*>(hot_k);
    const __half* vh = static_cast<const __half*>(hot_v);
#define WEAVER_NOALLOC_CASE(DD, GG) \
    if (head_dim == DD && G == GG)  \
        launch_partial<DD, GG>(grid, s, qh, kh, vh, hot_pool_blocks, hot_refs, n_blocks, bpc, kv_heads, scale, scratch, bad_ref_flag);
    WEAVER_NOALLOC_CASE(128, 1) WEAVER_NOALLOC_CASE(128, 2) WEAVER_NOALLOC_CASE(128, 4) WEAVER_NOALLOC_CASE(128, 8)
    WEAVER_NOALLOC_CASE(64, 1) WEAVER_NOALLOC_CASE(64, 2) WEAVER_NOALLOC_CASE(64, 4) WEAVER_NOALLOC_CASE(64, 8)
#undef WEAVER_NOALLOC_CASE
    if (cudaGetLastError() != cudaSuccess) return WEAVER_ERR_CUDA;
    noalloc_merge_kernel<<<q_heads, head_dim, 0, s>>>(scratch, chunks, q_heads, head_dim, o);
    return cudaGetLastError() == cudaSuccess ? WEAVER_OK : WEAVER_ERR_CUDA;
}
