// weaver_hot_mma.cu — the multi-kernel step's hot pass on mma.sync tensor
// cores, for plans with 8 or more query rows per kv head (the speculative
// verify of configuration c4: 8 drafts x 4 q heads, or 8 q heads per kv head
// of the 70B shape), where the hot blocks are a GEMM (weaver_kernel.metal:141-168
// with the causal rule of ops.metal:546-555); rows past R of a 16-row tile
// are zero queries that are never written.
//
// Same work split and outputs as hot_kernel: one CTA per (hot item = run of
// one sequence's hot blocks, kv head g, 16 query rows); its (m, l, o) per row
// goes to hm / hl / ho for merge_kernel.  Four warps take the item's blocks
// round-robin, each through a two-stage cp.async ring of K and V rows
// (128-byte-swizzled, the physical block from the page table, bit 31 masked,
// an out-of-range block flagged and skipped), and run the FlashAttention-2
// block step of weaver_fa.cuh.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_fa.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kHmThreads = 128;

template <int D>
struct HmLayout {
    static constexpr uint32_t kTile = FaTile<D>::kTile;
    static constexpr uint32_t kStage = 2 * kTile;
    static constexpr uint32_t kRing = 4 * 2 * kStage;       // 4 warps x 2 stages
    static constexpr uint32_t kRed = 4 * 16 * (D + 2) * 4;
    static constexpr uint32_t kQ = 16 * D * 2;
    static constexpr uint32_t kBytes = (kRing > kRed ? kRing : kRed) + kQ;
};

// Copies of hot block `phys` (kv head g) into stage `st`; zeros when !valid.
template <int D>
__device__ __forceinline__ void hm_issue(uint8_t* st, const __half* hk, const __half* hv, uint32_t phys, bool valid,
                                         uint32_t Hkv, uint32_t g, uint32_t lane) {
    using T = FaTile<D>;
#pragma unroll
    for (uint32_t i = lane; i < 16 * (D / 8); i += 32) {
        const uint32_t row = i / (D / 8), ch = i % (D / 8);
        const uint64_t off = ((static_cast<uint64_t>(valid ? phys : 0u) * kBlock + row) * Hkv + g) * D + ch * 8;
        const uint32_t so = (ch >> 3) * T::kBox + swz128(row, ch & 7);
        cp_async16_zfill(st + so, hk + off, valid);
        cp_async16_zfill(st + T::kTile + so, hv + off, valid);
    }
}

template <int D>
__global__ void __launch_bounds__(kHmThreads) hot_mma_kernel(const RunArgs a, const __half* __restrict__ hk,
                                                             const __half* __restrict__ hv) {
    using L = HmLayout<D>;
    constexpr int KS = D / 16, NT = D / 8;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __half* qs = reinterpret_cast<__half*>(smem + (L::kRing > L::kRed ? L::kRing : L::kRed));
    float* red = reinterpret_cast<float*>(smem);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2;
    const HotItem item = a.hot_items[blockIdx.x];
    const uint32_t g = blockIdx.y, rt = blockIdx.z, b = item.seq;
    const uint32_t npages = item.page_end - item.page_begin;
    const uint32_t Th = (a.hot_indptr[b + 1] - a.hot_indptr[b]) * kBlock;

    // query rows rt*16 .. +15 of kv head g (row r: draft r / G, q head g*G + r % G); zero past R
    for (uint32_t i = tid; i < 16 * (D / 8); i += kHmThreads) {
        const uint32_t r = i / (D / 8), ch = i % (D / 8), row = rt * 16 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row < a.R) {
            const uint32_t j = row / a.G, h = g * a.G + row % a.G;
            v = *reinterpret_cast<const uint4*>(a.q + ((static_cast<uint64_t>(b) * a.nq + j) * a.Hq + h) * D + ch * 8);
        }
        *reinterpret_cast<uint4*>(qs + r * D + ch * 8) = v;
    }
    __syncthreads();
    uint32_t qf[KS][4];
    fa_load_q<D>(qs, qf, lane);
    int32_t lim[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const uint32_t row = rt * 16 + gid + 8 * hh;
        int32_t l = row < a.R ? static_cast<int32_t>(Th) : 0;
        if ((a.flags & 1u) && row < a.R)  // WEAVER_FLAG_CAUSAL (ops.metal:549)
            l = static_cast<int32_t>(Th) - static_cast<int32_t>(a.nq) + 1 + static_cast<int32_t>(row / a.G);
        lim[hh] = l;
    }

    uint8_t* ring = smem + warp * 2 * L::kStage;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
    // this warp's blocks: i = warp, warp + 4, ...; the physical block and its validity per block
    const uint32_t nb = npages > warp ? (npages - warp + 3) / 4 : 0;
    bool ok_cur = false, ok_next = false;
    if (nb) {
        const uint32_t ph = a.hot_refs[item.page_begin + warp] & kRefMask;
        ok_cur = ph < a.hot_pool_blocks;
        if (!ok_cur && lane == 0) atomicOr(a.status, DEVERR_REF_RANGE);
        hm_issue<D>(ring, hk, hv, ph, ok_cur, a.Hkv, g, lane);
    }
    cp_async_commit();
    for (uint32_t k = 0; k < nb; ++k) {
        if (k + 1 < nb) {
            const uint32_t ph = a.hot_refs[item.page_begin + warp + 4 * (k + 1)] & kRefMask;
            ok_next = ph < a.hot_pool_blocks;
            if (!ok_next && lane == 0) atomicOr(a.status, DEVERR_REF_RANGE);
            hm_issue<D>(ring + ((k + 1) & 1) * L::kStage, hk, hv, ph, ok_next, a.Hkv, g, lane);
        }
        cp_async_commit();
        cp_async_wait1();  // block k has landed (this lane's copies)
        __syncwarp();      // ... and every lane's
        const uint8_t* Ks = ring + (k & 1) * L::kStage;
        fa_block<D>(Ks, Ks + L::kTile, qf, lim, static_cast<int32_t>(item.pos_base + (warp + 4 * k) * kBlock),
                    a.scale, ok_cur, m_run, l_run, o, lane);
        __syncwarp();  // every lane done with the stage before it is refilled
        ok_cur = ok_next;
    }
    cp_async_wait_all();
    __syncthreads();  // the rings are dead: reuse the space for the warps' partials
    fa_store_partial<D>(red + warp * 16 * (D + 2), m_run, l_run, o, lane);
    __syncthreads();
    for (uint32_t x = tid; x < 16 * D; x += kHmThreads) {
        const uint32_t r = x / D, d = x % D, row = rt * 16 + r;
        if (row >= a.R) continue;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, red[(w * 16 + r) * (D + 2)]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float* pw = red + (w * 16 + r) * (D + 2);
            const float f = exp_shift(pw[0], M);
            Ls += pw[1] * f;
            O += pw[2 + d] * f;
        }
        const uint64_t pidx = (static_cast<uint64_t>(blockIdx.x) * a.Hkv + g) * a.RP + row;
        if (d == 0) {
            a.hm[pidx] = M;
            a.hl[pidx] = Ls;
        }
        a.ho[pidx * D + d] = O;
    }
}

}  // namespace

bool hot_mma_supported(const RunArgs& a) { return (a.D == 64 || a.D == 128) && a.R >= 4; }

cudaError_t launch_hot_mma(const RunArgs& a, const __half* hot_k, const __half* hot_v, cudaStream_t s) {
    if (a.n_hot_items == 0) return cudaSuccess;
    const size_t smem = 1024 + (a.D == 128 ? HmLayout<128>::kBytes : HmLayout<64>::kBytes);
    dim3 grid(a.n_hot_items, a.Hkv, (a.R + 15) / 16);
    cudaError_t e;
    if (a.D == 128) {
        e = cudaFuncSetAttribute(hot_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        hot_mma_kernel<128><<<grid, kHmThreads, smem, s>>>(a, hot_k, hot_v);
    } else {
        e = cudaFuncSetAttribute(hot_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        hot_mma_kernel<64><<<grid, kHmThreads, smem, s>>>(a, hot_k, hot_v);
    }
    return cudaGetLastError();
}

}  // namespace weaver
