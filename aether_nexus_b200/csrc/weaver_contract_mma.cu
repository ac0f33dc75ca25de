// weaver_contract_mma.cu — the multi-kernel step's cold contraction
// o_cold = w . V_dict (the values of weaver_kernel.metal:192-221 without
// reconstructing V) on mma.sync tensor cores.
//
// One CTA (4 warps) per (kv head g, 16 of the head's B x R query rows (row
// q = sequence q / R, row q % R: a tile spans sequences when R < 16, so a
// dictionary tile read serves 16 rows), 64 of the D value dimensions, atom
// split): the warps take the split's 64-atom slices of g's dictionary
// round-robin through a per-warp two-stage cp.async ring (128-byte-swizzled
// rows, zero past A), load the slice's weights (fp32, [b][g][atom][RP] in L2)
// straight into A-operand fragments, and accumulate O (16 rows x 64 dims)
// with m16n8k16 MMAs, V via transposed ldmatrix.  The weights enter the MMA
// as two f16 parts, hi = f16(w) and lo = f16(w - hi) (about 22 bits of the
// fp32 weight), after scaling each slice by a power of two that keeps its
// largest weight below 2^15 (unscaled exactly in fp32 afterwards), so no
// weight overflows or loses more than fp32 rounding.  The four warps' sums
// meet in shared memory and the CTA adds its sums into the one cold partial
// per (b, g) with vector reductions (the merge reads one partial instead of
// A / 128).  The atom splits S exist for small grids (a few kv heads and
// sequences: c5's 8 x 1 x 2 CTAs would stream 2 MB of dictionary per head
// through 2 SMs).
#include <algorithm>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kCmThreads = 128;
constexpr uint32_t kCmAtoms = 64;  // atoms per slice (4 k-steps of 16)

struct CmLayout {
    static constexpr uint32_t kSlice = kCmAtoms * 128;          // 64 atoms x 64 f16 (one half of D = 128)
    static constexpr uint32_t kRing = 4 * 2 * kSlice;           // 4 warps x 2 stages
    static constexpr uint32_t kRed = 4 * 16 * 64 * 4;
    static constexpr uint32_t kBytes = kRing > kRed ? kRing : kRed;
};

// Rows a0 .. a0 + 63 of the dictionary, dims d0 .. d0 + 63, into a stage.
template <int D>
__device__ __forceinline__ void cm_issue(uint8_t* st, const __half* vd, uint32_t a0, uint32_t d0, uint32_t A,
                                         uint32_t lane) {
#pragma unroll
    for (uint32_t i = lane; i < kCmAtoms * 8; i += 32) {
        const uint32_t row = i / 8, ch = i % 8;
        const bool valid = a0 + row < A;
        cp_async16_zfill(st + swz128(row, ch), vd + static_cast<uint64_t>(valid ? a0 + row : 0u) * D + d0 + ch * 8,
                         valid);
    }
}

template <int D>
__global__ void __launch_bounds__(kCmThreads) cold_contract_mma_kernel(const RunArgs a, uint32_t S) {
    using L = CmLayout;
    constexpr int NT = 8;  // 64 dims
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    const uint32_t split = blockIdx.z % S, zz = blockIdx.z / S;
    const uint32_t g = blockIdx.x, rt = blockIdx.y, d0 = (zz % (D / 64)) * 64;
    const uint32_t A = a.A, RP = a.RP, R = a.R, nrows = a.B * a.R;
    const __half* vd = a.v_dict + static_cast<uint64_t>(g) * a.dict_row_stride * D;
    // this lane's two fragment rows q0 = rt*16 + gid and q1 = q0 + 8: their weight rows
    const uint32_t q0 = rt * 16 + gid, q1 = q0 + 8;
    const bool ok0 = q0 < nrows, ok1 = q1 < nrows;
    const float* w0 = a.w + ((static_cast<uint64_t>(ok0 ? q0 / R : 0) * a.Hkv + g) * A) * RP + (ok0 ? q0 % R : 0);
    const float* w1 = a.w + ((static_cast<uint64_t>(ok1 ? q1 / R : 0) * a.Hkv + g) * A) * RP + (ok1 ? q1 % R : 0);
    uint8_t* ring = smem + warp * 2 * L::kSlice;
    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;

    // this split's slices sl0 .. sl1 - 1; warp w takes sl0 + w, sl0 + w + 4, ...
    const uint32_t n_slices = (A + kCmAtoms - 1) / kCmAtoms;
    const uint32_t sl0 = static_cast<uint32_t>(static_cast<uint64_t>(n_slices) * split / S);
    const uint32_t sl1 = static_cast<uint32_t>(static_cast<uint64_t>(n_slices) * (split + 1) / S);
    const uint32_t mine = sl1 - sl0;
    const uint32_t nb = mine > warp ? (mine - warp + 3) / 4 : 0;
    if (nb) cm_issue<D>(ring, vd, (sl0 + warp) * kCmAtoms, d0, A, lane);
    cp_async_commit();
#pragma unroll 1
    for (uint32_t k = 0; k < nb; ++k) {
        const uint32_t a0 = (sl0 + warp + 4 * k) * kCmAtoms;
        if (k + 1 < nb) cm_issue<D>(ring + ((k + 1) & 1) * L::kSlice, vd, a0 + 4 * kCmAtoms, d0, A, lane);
        cp_async_commit();
        // this slice's weights: rows r0 / r1, atoms a0 + 16 ks + 2 tig (+1, +8, +9)
        float wv[4][8];
        float mx = 0.0f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t at = a0 + ks * 16 + 2 * tig + (e & 1) + ((e >> 2) & 1) * 8;
                const bool hi = (e >> 1) & 1;
                const bool ok = at < A && (hi ? ok1 : ok0);
                const float v = ok ? __ldcg((hi ? w1 : w0) + static_cast<uint64_t>(at) * RP) : 0.0f;
                wv[ks][e] = v;
                mx = fmaxf(mx, fabsf(v));
            }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        // a power of two that brings the slice's largest weight below 2^15 (1 if it already is)
        int ex = 0;
        if (mx >= 32768.0f) frexpf(mx, &ex);
        const float down = ex ? ldexpf(1.0f, 15 - ex) : 1.0f, up = ex ? ldexpf(1.0f, ex - 15) : 1.0f;
        uint32_t wa[4][4], wl[4][4];
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                // fragment q: (row r0 | r1) x (atoms 2tig.. | 8 + 2tig..); hi and lo parts
                const float x0 = wv[ks][2 * q] * down, x1 = wv[ks][2 * q + 1] * down;
                const __half2 h = __floats2half2_rn(x0, x1);
                const float2 hf = __half22float2(h);
                const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
                wa[ks][q] = *reinterpret_cast<const uint32_t*>(&h);
                wl[ks][q] = *reinterpret_cast<const uint32_t*>(&l);
            }
        cp_async_wait1();  // slice k has landed (this lane's copies)
        __syncwarp();      // ... and every lane's
        const uint8_t* Vs = ring + (k & 1) * L::kSlice;
        float t[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) t[j][e] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int j = 0; j < NT; j += 2) {
                const uint32_t arow = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const uint32_t dch = j + (lane >> 4);
                uint32_t vb[4];
                ldmatrix_x4_trans(vb, Vs + swz128(arow, dch));
                mma_16816(t[j], wa[ks], vb[0], vb[1]);
                mma_16816(t[j + 1], wa[ks], vb[2], vb[3]);
                mma_16816(t[j], wl[ks], vb[0], vb[1]);
                mma_16816(t[j + 1], wl[ks], vb[2], vb[3]);
            }
        }
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[j][e] = fmaf(t[j][e], up, o[j][e]);
        __syncwarp();  // every lane done with the stage before it is refilled
    }
    cp_async_wait_all();
    __syncthreads();  // the rings are dead: the warps' sums go to shared memory
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        *reinterpret_cast<float2*>(&red[(warp * 16 + gid) * 64 + j * 8 + 2 * tig]) = make_float2(o[j][0], o[j][1]);
        *reinterpret_cast<float2*>(&red[(warp * 16 + gid + 8) * 64 + j * 8 + 2 * tig]) = make_float2(o[j][2], o[j][3]);
    }
    __syncthreads();
    // the CTA's sum of 16 rows x 64 dims into the one cold partial (zeroed
    // before the launch), four dims per vector reduction
    for (uint32_t x = threadIdx.x; x < 16 * 16; x += kCmThreads) {
        const uint32_t r = x / 16, d = (x % 16) * 4, q = rt * 16 + r;
        if (q >= nrows) continue;
        const uint32_t b = q / R, row = q % R;
        float sm[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            sm[i] = (red[r * 64 + d + i] + red[(16 + r) * 64 + d + i]) + (red[(32 + r) * 64 + d + i] + red[(48 + r) * 64 + d + i]);
        red_add_v4(a.ocold + ((static_cast<uint64_t>(b) * a.Hkv + g) * RP + row) * D + d0 + d, sm[0], sm[1], sm[2], sm[3]);
    }
}

}  // namespace

bool contract_mma_supported(const RunArgs& a) { return a.D == 64 || a.D == 128; }

uint32_t contract_mma_splits(const RunArgs& a, uint32_t sms) {
    const uint32_t base = a.Hkv * ((a.B * a.R + 15) / 16) * (a.D / 64);
    const uint32_t n_slices = (a.A + kCmAtoms - 1) / kCmAtoms;
    uint32_t sp = (4 * sms + base - 1) / base;      // about four CTAs per SM (latency: 4 warps each)
    sp = std::min(sp, std::max(1u, n_slices / 4));  // a slice per warp at least
    sp = std::min(sp, a.n_atom_tiles);              // no more splits than 128-atom tiles
    return std::max(sp, 1u);
}

cudaError_t launch_cold_contract_mma(const RunArgs& a, uint32_t S, cudaStream_t s) {
    if (a.n_cold_items == 0) return cudaSuccess;
    const size_t smem = 1024 + CmLayout::kBytes;
    dim3 grid(a.Hkv, (a.B * a.R + 15) / 16, (a.D / 64) * S);
    cudaError_t e = cudaMemsetAsync(a.ocold, 0, sizeof(float) * a.B * a.Hkv * static_cast<size_t>(a.RP) * a.D, s);
    if (e != cudaSuccess) return e;
    if (a.D == 128) {
        e = cudaFuncSetAttribute(cold_contract_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        cold_contract_mma_kernel<128><<<grid, kCmThreads, smem, s>>>(a, S);
    } else {
        e = cudaFuncSetAttribute(cold_contract_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        cold_contract_mma_kernel<64><<<grid, kCmThreads, smem, s>>>(a, S);
    }
    return cudaGetLastError();
}

}  // namespace weaver
