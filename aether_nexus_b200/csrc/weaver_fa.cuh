// weaver_fa.cuh — one 16-position block of exact attention for 16 query rows
// on mma.sync tensor cores (FlashAttention-2 register layout), shared by the
// full loop's multi-query attention (weaver_mha.cu) and the multi-kernel
// step's hot pass at many query rows (weaver_hot_mma.cu).
//
// K and V blocks sit in shared memory as [D/64 boxes][16 rows][128 B] with the
// 128-byte swizzle (swz128).  Query fragments (A operand of S = Q K^T, rows
// gid and gid + 8 of the 16-row tile) stay in registers; the scores of the
// block come out in the C layout (row gid: positions 8n + 2tig, +1; row gid+8
// the same), which is exactly the A layout of P for O += P V.
#pragma once

#include <cuda_fp16.h>

#include "weaver_device.cuh"

namespace weaver {

template <int D>
struct FaTile {
    static constexpr uint32_t kBoxes = D / 64;
    static constexpr uint32_t kBox = 16 * 128;       // 16 rows x 64 f16
    static constexpr uint32_t kTile = kBoxes * kBox;  // one block of K (or V)
};

// Query fragments from a row-major [16][D] f16 tile in shared memory.
template <int D>
__device__ __forceinline__ void fa_load_q(const __half* qs, uint32_t qf[D / 16][4], uint32_t lane) {
    const uint32_t gid = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
        qf[ks][0] = *reinterpret_cast<const uint32_t*>(qs + gid * D + ks * 16 + 2 * tig);
        qf[ks][1] = *reinterpret_cast<const uint32_t*>(qs + (gid + 8) * D + ks * 16 + 2 * tig);
        qf[ks][2] = *reinterpret_cast<const uint32_t*>(qs + gid * D + ks * 16 + 8 + 2 * tig);
        qf[ks][3] = *reinterpret_cast<const uint32_t*>(qs + (gid + 8) * D + ks * 16 + 8 + 2 * tig);
    }
}

// One block: scores (times `scale`), positions pos0 + t masked at or past the
// row's limit lim[hh] (and all of them when !valid), online softmax update of
// (m_run, l_run) per row, O += P V.  l_run is this lane's partial sum (the
// caller adds the quad's lanes at the end).
template <int D>
__device__ __forceinline__ void fa_block(const uint8_t* Ks, const uint8_t* Vs, const uint32_t qf[D / 16][4],
                                         const int32_t lim[2], int32_t pos0, float scale, bool valid,
                                         float m_run[2], float l_run[2], float o[D / 8][4], uint32_t lane) {
    using T = FaTile<D>;
    constexpr int KS = D / 16, NT = D / 8;
    const uint32_t tig = lane & 3;
    float c[2][4];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 4; ++e) c[h][e] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const uint32_t trow = (lane & 7) + (lane >> 4) * 8;
        const uint32_t dch = ks * 2 + ((lane >> 3) & 1);
        uint32_t kb[4];
        ldmatrix_x4(kb, Ks + (dch >> 3) * T::kBox + swz128(trow, dch & 7));
        mma_16816(c[0], qf[ks], kb[0], kb[1]);
        mma_16816(c[1], qf[ks], kb[2], kb[3]);
    }
    float pv[2][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        float sv[4];
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int32_t pos = pos0 + n * 8 + 2 * static_cast<int32_t>(tig) + e;
                sv[n * 2 + e] = (valid && pos < lim[hh]) ? c[n][2 * hh + e] * scale : -INFINITY;
            }
        float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[hh], mx);
        const float alpha = exp_shift(m_run[hh], m_new);
#pragma unroll
        for (int e = 0; e < 4; ++e) pv[hh][e] = exp_shift(sv[e], m_new);
        l_run[hh] = l_run[hh] * alpha + (pv[hh][0] + pv[hh][1]) + (pv[hh][2] + pv[hh][3]);
        m_run[hh] = m_new;
#pragma unroll
        for (int j = 0; j < NT; ++j) {
            o[j][2 * hh] *= alpha;
            o[j][2 * hh + 1] *= alpha;
        }
    }
    // P as the A operand: a0 row gid positions 2tig.., a1 row gid+8, a2 / a3 positions 8+2tig..
    const __half2 p0 = __floats2half2_rn(pv[0][0], pv[0][1]);
    const __half2 p1 = __floats2half2_rn(pv[1][0], pv[1][1]);
    const __half2 p2 = __floats2half2_rn(pv[0][2], pv[0][3]);
    const __half2 p3 = __floats2half2_rn(pv[1][2], pv[1][3]);
    const uint32_t pa[4] = {*reinterpret_cast<const uint32_t*>(&p0), *reinterpret_cast<const uint32_t*>(&p1),
                            *reinterpret_cast<const uint32_t*>(&p2), *reinterpret_cast<const uint32_t*>(&p3)};
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
        const uint32_t trow = (lane & 7) + ((lane >> 3) & 1) * 8;
        const uint32_t dch = j + (lane >> 4);
        uint32_t vb[4];
        ldmatrix_x4_trans(vb, Vs + (dch >> 3) * T::kBox + swz128(trow, dch & 7));
        mma_16816(o[j], pa, vb[0], vb[1]);
        mma_16816(o[j + 1], pa, vb[2], vb[3]);
    }
}

// This warp's (m, l, o) of its 16 rows into red[16][D + 2] (l summed over the
// quad's lanes first).
template <int D>
__device__ __forceinline__ void fa_store_partial(float* red, float m_run[2], float l_run[2], const float o[D / 8][4],
                                                 uint32_t lane) {
    const uint32_t gid = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 1);
        l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 2);
        const uint32_t r = gid + 8 * hh;
        if (tig == 0) {
            red[r * (D + 2)] = m_run[hh];
            red[r * (D + 2) + 1] = l_run[hh];
        }
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
            red[r * (D + 2) + 2 + j * 8 + 2 * tig] = o[j][2 * hh];
            red[r * (D + 2) + 2 + j * 8 + 2 * tig + 1] = o[j][2 * hh + 1];
        }
    }
}

}  // namespace weaver
