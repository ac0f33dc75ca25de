// weaver_mha.cu — the full loop's exact multi-query attention
// (nexus-core/src/ops.metal:528-616, called at inference.rs:552-562 for the
// prompt, plain decode and the speculative-verify batch): query token qi of
// nq attends to the cache positions < total_kv_len - nq + 1 + qi, scale
// 1/sqrt(d), GQA (q head h reads kv head h / (Hq / Hkv)).
//
// Split-KV on the tensor cores.  One CTA (4 warps) per (chunk of 64 * bpw
// positions, kv head g, tile of 16 query rows of g); row r of g is query
// token r / G, q head g * G + r % G.  Each warp streams its 16-position blocks
// of the chunk through a two-stage cp.async ring (K and V rows of head g into
// 128-byte-swizzled shared memory, zero-filled past the cache length) and
// runs FlashAttention-2 style mma.sync.m16n8k16: S = Q K^T with the query
// fragments held in registers, the causal mask per row, an online softmax per
// row, O += P V with P reused from the S registers.  The four warps' partials
// merge in shared memory into the chunk's (m, l, o) per row; a merge kernel
// over the chunks writes the f16 output (one chunk: written directly).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_fa.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kMhaThreads = 128;

template <int D>
struct MhaLayout {
    static constexpr uint32_t kBoxes = D / 64;
    static constexpr uint32_t kBox = 16 * 128;                 // 16 rows x 64 f16, 128-byte swizzle
    static constexpr uint32_t kTile = kBoxes * kBox;           // one 16-position block of K (or V)
    static constexpr uint32_t kStage = 2 * kTile;              // K and V
    static constexpr uint32_t kWarpRing = 2 * kStage;          // two stages per warp
    static constexpr uint32_t kRing = 4 * kWarpRing;
    static constexpr uint32_t kQ = 16 * D * 2;                 // the query tile, row-major
    static constexpr uint32_t kRed = 4 * 16 * (D + 2) * 4;     // four warps' (m, l, o) rows
    static constexpr uint32_t kBytes = (kRing > kRed ? kRing : kRed) + kQ;
};

// Issue the copies of block `blk` (positions 16 blk .. 16 blk + 15) of kv head
// g into ring stage `st`: 16 rows x D/8 chunks for K and for V, 2 * D/8 per lane.
template <int D>
__device__ __forceinline__ void issue_block(uint8_t* st, const __half* kc, const __half* vc, uint32_t blk,
                                            uint32_t T, uint32_t row_stride, uint32_t g, uint32_t lane) {
    using L = MhaLayout<D>;
#pragma unroll
    for (uint32_t i = lane; i < 16 * (D / 8); i += 32) {
        const uint32_t row = i / (D / 8), ch = i % (D / 8);
        const uint32_t pos = blk * 16 + row;
        const bool valid = pos < T;
        const uint64_t off = static_cast<uint64_t>(valid ? pos : 0u) * row_stride + g * D + ch * 8;
        const uint32_t so = (ch >> 3) * L::kBox + swz128(row, ch & 7);
        cp_async16_zfill(st + so, kc + off, valid);
        cp_async16_zfill(st + L::kTile + so, vc + off, valid);
    }
}

template <int D>
__global__ void __launch_bounds__(kMhaThreads) mha_kernel(const __half* __restrict__ q, const __half* __restrict__ kc,
                                                          const __half* __restrict__ vc, __half* __restrict__ out,
                                                          float* __restrict__ part, uint32_t T, uint32_t Hq,
                                                          uint32_t Hkv, uint32_t nq, uint32_t bpw) {
    using L = MhaLayout<D>;
    constexpr int KS = D / 16, NT = D / 8;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    __half* qs = reinterpret_cast<__half*>(smem + (L::kRing > L::kRed ? L::kRing : L::kRed));
    float* red = reinterpret_cast<float*>(smem);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t gid = lane >> 2, tig = lane & 3;
    const uint32_t chunk = blockIdx.x, g = blockIdx.y, rt = blockIdx.z;
    const uint32_t G = Hq / Hkv, R = nq * G, row_stride = Hkv * D;
    const uint32_t rows_total = nq * Hq;
    const uint32_t n_chunks = gridDim.x;

    // query tile: rows rt*16 .. +15 of kv head g (zero past R)
    for (uint32_t i = tid; i < 16 * (D / 8); i += kMhaThreads) {
        const uint32_t r = i / (D / 8), ch = i % (D / 8), rr = rt * 16 + r;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (rr < R) {
            const uint32_t j = rr / G, h = g * G + rr % G;
            v = *reinterpret_cast<const uint4*>(q + (static_cast<uint64_t>(j) * Hq + h) * D + ch * 8);
        }
        *reinterpret_cast<uint4*>(qs + r * D + ch * 8) = v;
    }
    __syncthreads();
    uint32_t qf[KS][4];
    fa_load_q<D>(qs, qf, lane);
    // causal limits of this lane's two rows (gid, gid + 8); rows past R see nothing
    int32_t lim[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const uint32_t rr = rt * 16 + gid + 8 * hh;
        lim[hh] = rr < R ? static_cast<int32_t>(T - nq + 1 + rr / G) : 0;
    }
    // the positions this warp visits: blocks chunk*4*bpw + warp + 4k, below the tile's largest limit
    const uint32_t r_hi = min(R, rt * 16 + 16) - 1;
    const uint32_t tile_lim = T - nq + 1 + r_hi / G;
    const uint32_t nblk_all = (tile_lim + 15) / 16;
    const uint32_t b0 = chunk * 4 * bpw + warp;
    uint32_t nb = 0;
    for (uint32_t k = 0; k < bpw; ++k)
        if (b0 + 4 * k < nblk_all) ++nb;

    uint8_t* ring = smem + warp * L::kWarpRing;
    const float scale = rsqrtf(static_cast<float>(D));
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;

    if (nb > 0) issue_block<D>(ring, kc, vc, b0, T, row_stride, g, lane);
    cp_async_commit();
    for (uint32_t k = 0; k < nb; ++k) {
        if (k + 1 < nb) issue_block<D>(ring + ((k + 1) & 1) * L::kStage, kc, vc, b0 + 4 * (k + 1), T, row_stride, g, lane);
        cp_async_commit();
        cp_async_wait1();  // block k has landed (this lane's copies)
        __syncwarp();      // ... and every lane's
        const uint8_t* Ks = ring + (k & 1) * L::kStage;
        fa_block<D>(Ks, Ks + L::kTile, qf, lim, static_cast<int32_t>((b0 + 4 * k) * 16), scale, true, m_run, l_run, o,
                    lane);
        __syncwarp();  // every lane done with the stage before it is refilled
    }
    cp_async_wait_all();
    __syncthreads();  // the rings are dead: reuse the space for the warps' partials
    // red: [warp][16 rows][D + 2]: m, l, o
    fa_store_partial<D>(red + warp * 16 * (D + 2), m_run, l_run, o, lane);
    __syncthreads();
    // merge the four warps: thread tid takes (row, dimensions tid % 8 + 8k)
    for (uint32_t x = tid; x < 16 * D; x += kMhaThreads) {
        const uint32_t r = x / D, d = x % D, rr = rt * 16 + r;
        if (rr >= R) continue;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, red[(w * 16 + r) * (D + 2)]);
        float Lsum = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float* pw = red + (w * 16 + r) * (D + 2);
            const float f = exp_shift(pw[0], M);
            Lsum += pw[1] * f;
            O += pw[2 + d] * f;
        }
        const uint32_t j = rr / G, h = g * G + rr % G;
        const uint64_t row = static_cast<uint64_t>(j) * Hq + h;
        if (n_chunks == 1) {
            out[row * D + d] = __float2half_rn(Lsum > 0.0f ? O / Lsum : 0.0f);
        } else {
            // partial of this chunk: [chunk][m rows | l rows | o rows * D]
            float* pc = part + static_cast<uint64_t>(chunk) * rows_total * (D + 2);
            if (d == 0) {
                pc[row] = M;
                pc[rows_total + row] = Lsum;
            }
            pc[2ull * rows_total + row * D + d] = O;
        }
    }
}

}  // namespace

size_t mha_smem_bytes(uint32_t D) {
    return 1024 + (D == 128 ? MhaLayout<128>::kBytes : MhaLayout<64>::kBytes);
}

// Positions per warp-block count: enough CTAs to fill the SMs twice over.
static uint32_t mha_bpw(uint32_t T, uint32_t Hkv, uint32_t row_tiles, uint32_t n_sm) {
    const uint64_t blocks = (static_cast<uint64_t>(T) + 15) / 16;
    const uint64_t ctas_per_chunk_column = static_cast<uint64_t>(Hkv) * row_tiles;
    uint32_t bpw = 1;
    while (bpw < 64 && ((blocks + 4 * bpw * 2 - 1) / (4 * bpw * 2)) * ctas_per_chunk_column >= 2ull * n_sm) bpw *= 2;
    return bpw;
}

uint64_t mha_scratch_floats(uint32_t T, uint32_t D, uint32_t Hq, uint32_t Hkv, uint32_t nq, uint32_t n_sm) {
    const uint32_t R = nq * (Hq / Hkv), row_tiles = (R + 15) / 16;
    const uint32_t bpw = mha_bpw(T, Hkv, row_tiles, n_sm);
    const uint64_t n_chunks = ((T + 15) / 16 + 4 * bpw - 1) / (4 * bpw);
    return n_chunks > 1 ? n_chunks * static_cast<uint64_t>(nq) * Hq * (D + 2) : 0;
}

cudaError_t launch_mha(const __half* q, const __half* kc, const __half* vc, __half* out, float* scratch, uint32_t T,
                       uint32_t D, uint32_t Hq, uint32_t Hkv, uint32_t nq, uint32_t n_sm, cudaStream_t s) {
    const uint32_t R = nq * (Hq / Hkv), row_tiles = (R + 15) / 16;
    const uint32_t bpw = mha_bpw(T, Hkv, row_tiles, n_sm);
    const uint32_t n_chunks = ((T + 15) / 16 + 4 * bpw - 1) / (4 * bpw);
    const size_t smem = mha_smem_bytes(D);
    dim3 grid(n_chunks, Hkv, row_tiles);
    cudaError_t e;
    if (D == 128) {
        e = cudaFuncSetAttribute(mha_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        mha_kernel<128><<<grid, kMhaThreads, smem, s>>>(q, kc, vc, out, scratch, T, Hq, Hkv, nq, bpw);
    } else {
        e = cudaFuncSetAttribute(mha_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        mha_kernel<64><<<grid, kMhaThreads, smem, s>>>(q, kc, vc, out, scratch, T, Hq, Hkv, nq, bpw);
    }
    if ((e = cudaGetLastError()) != cudaSuccess || n_chunks == 1) return e;
    const uint32_t rows = nq * Hq;
    return launch_merge_partials_strided(n_chunks, rows, D, scratch, scratch + rows, scratch + 2ull * rows,
                                         static_cast<uint64_t>(rows) * (D + 2), out, s);
}

}  // namespace weaver
