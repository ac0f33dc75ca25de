// weaver_kernels.cu — sm_100a kernels of the Weaver decode step.
//
// One decode step (nexus-core/src/weaver_kernel.metal:118-240, generalised):
//   hot  : split-KV exact attention over 16-token blocks, K/V staged by TMA
//          (128B-swizzled boxes) through an mbarrier ring, one lane per token
//          for q.K, one lane per 4 (or 2) dims for p.V, fp32 online softmax.
//   cold : q_latent = scale * q . K_dict            (qlat_kernel)
//          s = sum_k cK_k q_latent[iK_k] per code   (cold_score_kernel)
//          w[iV_k] += exp(s - M) cV_k (global max M) (cold_scatter_kernel)
//          o_cold = w . V_dict                      (cold_contract_kernel)
//   merge: log-sum-exp of all hot partials and the cold partial (merge_kernel).
// Cold K and V are never reconstructed: the score is a 4-term gather of the
// projected query and the value is a contraction of the per-atom weights.
#include <cstdlib>

#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {

namespace {

__device__ __forceinline__ uint8_t* align_1024(uint8_t* p) {
    const uint32_t off = (1024u - (smem_u32(p) & 1023u)) & 1023u;
    return p + off;
}

__device__ __forceinline__ float dot8(const float* q, const float k[8]) {
    const float4 a = *reinterpret_cast<const float4*>(q);
    const float4 b = *reinterpret_cast<const float4*>(q + 4);
    float s = a.x * k[0];
    s = fmaf(a.y, k[1], s);
    s = fmaf(a.z, k[2], s);
    s = fmaf(a.w, k[3], s);
    s = fmaf(b.x, k[4], s);
    s = fmaf(b.y, k[5], s);
    s = fmaf(b.z, k[6], s);
    s = fmaf(b.w, k[7], s);
    return s;
}

// Query row `row` (0 <= row < R) of kv head g -> pointer to q[b][j][h][:].
__device__ __forceinline__ const __half* q_row_ptr(const RunArgs& a, uint32_t b, uint32_t g,
                                                   uint32_t row) {
    const uint32_t j = row / a.G, hh = row % a.G;
    const uint32_t h = g * a.G + hh;
    return a.q + ((static_cast<uint64_t>(b) * a.nq + j) * a.Hq + h) * a.D;
}

}  // namespace

// ---------------------------------------------------------------------------
// Hot pass: split-KV exact attention.
// grid (hot item, kv head g, row group z); 4 consumer warps + 1 TMA warp.
// ---------------------------------------------------------------------------
template <int D, int RM>
__global__ void __launch_bounds__(160) hot_kernel(const __grid_constant__ CUtensorMap tm_k,
                                                  const __grid_constant__ CUtensorMap tm_v,
                                                  const RunArgs a) {
    constexpr int kCons = 4;
    constexpr int kStages = 8;
    constexpr int kBoxes = D / 64;
    constexpr uint32_t kBoxBytes = kBlock * 128;      // one 16-row x 64-col f16 box
    constexpr uint32_t kPage = kBoxes * kBoxBytes;    // one head's block of K (or V)
    constexpr uint32_t kStage = 2 * kPage;
    constexpr int VPL = D / 32;                       // value dims per lane

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint8_t* stages = smem;
    float* q_s = reinterpret_cast<float*>(smem + kStages * kStage);   // [RM][D]
    float* p_s = q_s + RM * D;                                         // [kCons][RM][16]
    float* comb_m = p_s + kCons * RM * 16;                             // [kCons][RM]
    float* comb_l = comb_m + kCons * RM;                               // [kCons][RM]
    float* comb_o = comb_l + kCons * RM;                               // [kCons][RM][D]
    int* valid_s = reinterpret_cast<int*>(comb_o + kCons * RM * D);    // [kStages]
    uint64_t* full = reinterpret_cast<uint64_t*>(valid_s + kStages);   // [kStages]
    uint64_t* empty = full + kStages;                                  // [kStages]

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const HotItem item = a.hot_items[blockIdx.x];
    const uint32_t g = blockIdx.y, z = blockIdx.z, b = item.seq;
    const uint32_t npages = item.page_end - item.page_begin;
    const uint32_t Th = (a.hot_indptr[b + 1] - a.hot_indptr[b]) * kBlock;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_barrier_init();
    }
    for (uint32_t idx = tid; idx < RM * D; idx += blockDim.x) {
        const uint32_t r = idx / D, dim = idx % D, row = z * RM + r;
        float v = 0.0f;
        if (row < a.R) v = __half2float(q_row_ptr(a, b, g, row)[dim]) * a.scale;
        q_s[idx] = v;
    }
    __syncthreads();

    if (warp == kCons) {
        // TMA producer: one elected lane streams K and V blocks into the ring.
        if (lane == 0) {
            prefetch_tensormap(&tm_k);
            prefetch_tensormap(&tm_v);
            for (uint32_t i = 0; i < npages; ++i) {
                const uint32_t s = i % kStages;
                if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1, a.status)) break;
                const uint32_t phys = a.hot_refs[item.page_begin + i] & kRefMask;
                if (phys >= a.hot_pool_blocks) {
                    atomicOr(a.status, DEVERR_REF_RANGE);
                    valid_s[s] = 0;
                    mbar_arrive(&full[s]);
                    continue;
                }
                valid_s[s] = 1;
                uint8_t* dst = stages + s * kStage;
                mbar_arrive_expect_tx(&full[s], kStage);
#pragma unroll
                for (int bx = 0; bx < kBoxes; ++bx) {
                    const int32_t x = static_cast<int32_t>(g * D + bx * 64);
                    const int32_t y = static_cast<int32_t>(phys * kBlock);
                    tma_load_2d(dst + bx * kBoxBytes, &tm_k, &full[s], x, y);
                    tma_load_2d(dst + kPage + bx * kBoxBytes, &tm_v, &full[s], x, y);
                }
            }
        }
    } else {
        float m[RM], lsum[RM], o[RM][VPL];
        int32_t limit[RM];
#pragma unroll
        for (int r = 0; r < RM; ++r) {
            m[r] = -INFINITY;
            lsum[r] = 0.0f;
#pragma unroll
            for (int e = 0; e < VPL; ++e) o[r][e] = 0.0f;
            const uint32_t row = z * RM + r;
            int32_t lim = static_cast<int32_t>(Th);
            if ((a.flags & 1u) && row < a.R)  // WEAVER_FLAG_CAUSAL (ops.metal:549)
                lim = static_cast<int32_t>(Th) - static_cast<int32_t>(a.nq) + 1 +
                      static_cast<int32_t>(row / a.G);
            limit[r] = lim;
        }
        const uint32_t tok = lane & 15, hf = lane >> 4;
        for (uint32_t i = warp; i < npages; i += kCons) {
            const uint32_t s = i % kStages;
            if (!mbar_wait(&full[s], (i / kStages) & 1, a.status)) break;
            const bool pvalid = valid_s[s] != 0;
            const uint8_t* Ks = stages + s * kStage;
            const uint8_t* Vs = Ks + kPage;

            // scores: lanes t and t+16 each cover half of token t's dims
            float acc[RM];
#pragma unroll
            for (int r = 0; r < RM; ++r) acc[r] = 0.0f;
            if (D == 128) {
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint4 raw = *reinterpret_cast<const uint4*>(Ks + hf * kBoxBytes + swz128(tok, c));
                    float kf[8];
                    h8_to_f8(raw, kf);
#pragma unroll
                    for (int r = 0; r < RM; ++r) acc[r] += dot8(q_s + r * D + hf * 64 + c * 8, kf);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int cc = hf * 4 + c;
                    const uint4 raw = *reinterpret_cast<const uint4*>(Ks + swz128(tok, cc));
                    float kf[8];
                    h8_to_f8(raw, kf);
#pragma unroll
                    for (int r = 0; r < RM; ++r) acc[r] += dot8(q_s + r * D + cc * 8, kf);
                }
            }
            const int32_t pos = static_cast<int32_t>(item.pos_base + i * kBlock + tok);
            float alpha[RM];
#pragma unroll
            for (int r = 0; r < RM; ++r) {
                acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 16);
                const float sc = (pvalid && pos < limit[r]) ? acc[r] : -INFINITY;
                float mx = sc;
#pragma unroll
                for (int off = 8; off > 0; off >>= 1)
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
                const float m_new = fmaxf(m[r], mx);
                alpha[r] = exp_shift(m[r], m_new);
                const float p = exp_shift(sc, m_new);
                lsum[r] = lsum[r] * alpha[r] + (lane < 16 ? p : 0.0f);
                m[r] = m_new;
                if (lane < 16) p_s[(warp * RM + r) * 16 + tok] = p;
            }
            __syncwarp();
#pragma unroll
            for (int r = 0; r < RM; ++r)
#pragma unroll
                for (int e = 0; e < VPL; ++e) o[r][e] *= alpha[r];
            // p.V: lane owns VPL consecutive dims
#pragma unroll 4
            for (int t = 0; t < 16; ++t) {
                float vf[VPL];
                if (D == 128) {
                    const uint32_t bx = lane >> 4, chunk = (lane & 15) >> 1;
                    const uint2 raw = *reinterpret_cast<const uint2*>(
                        Vs + bx * kBoxBytes + swz128(t, chunk) + (lane & 1) * 8);
                    h4_to_f4(raw, vf);
                } else {
                    const uint32_t chunk = lane >> 2;
                    const uint32_t raw = *reinterpret_cast<const uint32_t*>(
                        Vs + swz128(t, chunk) + (lane & 3) * 4);
                    const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&raw));
                    vf[0] = v2.x;
                    vf[VPL - 1] = v2.y;
                }
#pragma unroll
                for (int r = 0; r < RM; ++r) {
                    const float pt = p_s[(warp * RM + r) * 16 + t];
#pragma unroll
                    for (int e = 0; e < VPL; ++e) o[r][e] = fmaf(pt, vf[e], o[r][e]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
#pragma unroll
        for (int r = 0; r < RM; ++r) {
            const float lw = warp_sum(lsum[r]);
            if (lane == 0) {
                comb_m[warp * RM + r] = m[r];
                comb_l[warp * RM + r] = lw;
            }
#pragma unroll
            for (int e = 0; e < VPL; ++e) comb_o[(warp * RM + r) * D + lane * VPL + e] = o[r][e];
        }
    }
    __syncthreads();

    for (uint32_t idx = tid; idx < RM * D; idx += blockDim.x) {
        const uint32_t r = idx / D, dim = idx % D, row = z * RM + r;
        if (row >= a.R) continue;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kCons; ++w) M = fmaxf(M, comb_m[w * RM + r]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < kCons; ++w) {
            const float f = exp_shift(comb_m[w * RM + r], M);
            L += comb_l[w * RM + r] * f;
            O += comb_o[(w * RM + r) * D + dim] * f;
        }
        const uint64_t pidx = (static_cast<uint64_t>(blockIdx.x) * a.Hkv + g) * a.RP + row;
        if (dim == 0) {
            a.hm[pidx] = M;
            a.hl[pidx] = L;
        }
        a.ho[pidx * D + dim] = O;
    }
}

// ---------------------------------------------------------------------------
// q_latent = scale * q . K_dict for one 128-atom tile; also clears w.
// grid (atom tile, kv head, sequence); 4 warps, one lane per atom.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) qlat_kernel(const __grid_constant__ CUtensorMap tm_kdict,
                                                   const RunArgs a) {
    constexpr int kBoxes = D / 64;
    constexpr uint32_t kBoxBytes = kAtomTile * 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint8_t* tile = smem;                                             // [kBoxes][128][128 B]
    float* q_s = reinterpret_cast<float*>(smem + kBoxes * kBoxBytes); // [RPad8][D]
    uint64_t* bar = reinterpret_cast<uint64_t*>(q_s + ((a.RP + 7) / 8) * 8 * D);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t t = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, kBoxes * kBoxBytes);
        const int32_t y = static_cast<int32_t>(g * a.dict_row_stride + t * kAtomTile);
#pragma unroll
        for (int bx = 0; bx < kBoxes; ++bx) tma_load_2d(tile + bx * kBoxBytes, &tm_kdict, bar, bx * 64, y);
    }
    const uint32_t rpad = ((a.RP + 7) / 8) * 8;
    for (uint32_t idx = tid; idx < rpad * D; idx += blockDim.x) {
        const uint32_t r = idx / D, dim = idx % D;
        float v = 0.0f;
        if (r < a.R) v = __half2float(q_row_ptr(a, b, g, r)[dim]) * a.scale;
        q_s[idx] = v;
    }
    __syncthreads();
    const bool ok = mbar_wait(bar, 0, a.status);

    const uint32_t row = warp * 32 + lane;
    const uint32_t atom = t * kAtomTile + row;
    const uint64_t base = ((static_cast<uint64_t>(b) * a.Hkv + g) * a.A + atom) * a.RP;
    for (uint32_t rg = 0; rg < rpad; rg += 8) {
        float acc[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) acc[r] = 0.0f;
        if (ok) {
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4*>(tile + (c >> 3) * kBoxBytes + swz128(row, c & 7));
                float kf[8];
                h8_to_f8(raw, kf);
#pragma unroll
                for (int r = 0; r < 8; ++r) acc[r] += dot8(q_s + (rg + r) * D + c * 8, kf);
            }
        }
        if (atom < a.A) {
#pragma unroll
            for (int r = 0; r < 8; ++r)
                if (rg + r < a.RP) {
                    a.qlat[base + rg + r] = acc[r];
                    a.w[base + rg + r] = 0.0f;
                }
        }
    }
}

// Caller-supplied f16 q_latent [B][nq][Hq][A] -> internal fp32 layout; clears w.
__global__ void qlat_import_kernel(const RunArgs a) {
    const uint64_t total = static_cast<uint64_t>(a.B) * a.Hkv * a.A * a.RP;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t r = i % a.RP;
        const uint64_t rest = i / a.RP;
        const uint32_t atom = rest % a.A;
        const uint64_t bg = rest / a.A;
        const uint32_t g = bg % a.Hkv, b = static_cast<uint32_t>(bg / a.Hkv);
        float v = 0.0f;
        if (r < a.R) {
            const uint32_t j = r / a.G, h = g * a.G + r % a.G;
            v = __half2float(a.q_latent[((static_cast<uint64_t>(b) * a.nq + j) * a.Hq + h) * a.A + atom]);
        }
        a.qlat[i] = v;
        a.w[i] = 0.0f;
    }
}

// ---------------------------------------------------------------------------
// Cold scores: one thread per cold token of a <=16-block item.
// ---------------------------------------------------------------------------
template <int RP>
__device__ __forceinline__ void load_rows(const float* p, float v[RP]) {
    if constexpr (RP >= 4) {
#pragma unroll
        for (int r = 0; r < RP; r += 4) {
            const float4 x = __ldg(reinterpret_cast<const float4*>(p + r));
            v[r] = x.x;
            v[r + 1] = x.y;
            v[r + 2] = x.z;
            v[r + 3] = x.w;
        }
    } else if constexpr (RP == 2) {
        const float2 x = __ldg(reinterpret_cast<const float2*>(p));
        v[0] = x.x;
        v[1] = x.y;
    } else {
        v[0] = __ldg(p);
    }
}

template <int RP>
__global__ void __launch_bounds__(256) cold_score_kernel(const RunArgs a) {
    __shared__ float red[8][RP];
    // kv heads fastest in launch order (one item's head CTAs share its code lines)
    const uint32_t ci = blockIdx.y + blockIdx.z * gridDim.y, g = blockIdx.x;
    if (ci >= a.n_cold_items) return;
    const ColdItem item = a.cold_items[ci];
    const uint32_t b = item.seq;
    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t page = item.page_begin + t / kBlock, tt = t % kBlock;
    float s[RP];
#pragma unroll
    for (int r = 0; r < RP; ++r) s[r] = -INFINITY;
    if (page < item.page_end) {
        const uint32_t phys = a.cold_refs[page] & kRefMask;
        if (phys < a.cold_pool_blocks) {
            const uint4 code = __ldg(&a.cold_k[(static_cast<uint64_t>(phys) * kBlock + tt) * a.Hkv + g]);
            const uint16_t* idx = reinterpret_cast<const uint16_t*>(&code.x);
            const uint16_t* cf = reinterpret_cast<const uint16_t*>(&code.z);
            const float* base = a.qlat + (static_cast<uint64_t>(b) * a.Hkv + g) * a.A * RP;
#pragma unroll
            for (int r = 0; r < RP; ++r) s[r] = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (idx[k] >= a.A) {
                    atomicOr(a.status, DEVERR_ATOM_RANGE);
                    continue;
                }
                const float c = h2f(cf[k]);
                float v[RP];
                load_rows<RP>(base + static_cast<uint64_t>(idx[k]) * RP, v);
#pragma unroll
                for (int r = 0; r < RP; ++r) s[r] = fmaf(c, v[r], s[r]);
            }
        } else {
            atomicOr(a.status, DEVERR_REF_RANGE);
        }
        float* dst = a.scores + (static_cast<uint64_t>(g) * a.cold_tokens + static_cast<uint64_t>(page) * kBlock + tt) * RP;
#pragma unroll
        for (int r = 0; r < RP; ++r) dst[r] = s[r];
    }
#pragma unroll
    for (int r = 0; r < RP; ++r) {
        const float mx = warp_max(s[r]);
        if (lane == 0) red[warp][r] = mx;
    }
    __syncthreads();
    if (t < RP) {
        float mx = red[0][t];
#pragma unroll
        for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w][t]);
        a.cmax[(static_cast<uint64_t>(ci) * a.Hkv + g) * RP + t] = mx;
    }
}

// ---------------------------------------------------------------------------
// Cold values: w[iV_k] += exp(s - M) * cV_k with the sequence-wide max M.
// ---------------------------------------------------------------------------
template <int RP>
__global__ void __launch_bounds__(256) cold_scatter_kernel(const RunArgs a) {
    __shared__ float Ms[RP];
    __shared__ float red[8][RP];
    // kv heads fastest in launch order (one item's head CTAs share its code lines)
    const uint32_t ci = blockIdx.y + blockIdx.z * gridDim.y, g = blockIdx.x;
    if (ci >= a.n_cold_items) return;
    const ColdItem item = a.cold_items[ci];
    const uint32_t b = item.seq;
    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    if (warp == 0) {
        const uint32_t i0 = a.cold_item_ptr[b], i1 = a.cold_item_ptr[b + 1];
#pragma unroll
        for (int r = 0; r < RP; ++r) {
            float mx = -INFINITY;
            for (uint32_t it = i0 + lane; it < i1; it += 32)
                mx = fmaxf(mx, a.cmax[(static_cast<uint64_t>(it) * a.Hkv + g) * RP + r]);
            mx = warp_max(mx);
            if (lane == 0) Ms[r] = mx;
        }
    }
    __syncthreads();
    const uint32_t page = item.page_begin + t / kBlock, tt = t % kBlock;
    float p[RP];
#pragma unroll
    for (int r = 0; r < RP; ++r) p[r] = 0.0f;
    if (page < item.page_end) {
        const uint32_t phys = a.cold_refs[page] & kRefMask;
        if (phys < a.cold_pool_blocks) {
            const float* src = a.scores + (static_cast<uint64_t>(g) * a.cold_tokens + static_cast<uint64_t>(page) * kBlock + tt) * RP;
            float sv[RP];
            load_rows<RP>(src, sv);
#pragma unroll
            for (int r = 0; r < RP; ++r) p[r] = exp_shift(sv[r], Ms[r]);
            const uint4 code = __ldg(&a.cold_v[(static_cast<uint64_t>(phys) * kBlock + tt) * a.Hkv + g]);
            const uint16_t* idx = reinterpret_cast<const uint16_t*>(&code.x);
            const uint16_t* cf = reinterpret_cast<const uint16_t*>(&code.z);
            float* wb = a.w + (static_cast<uint64_t>(b) * a.Hkv + g) * a.A * RP;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (idx[k] >= a.A) {
                    atomicOr(a.status, DEVERR_ATOM_RANGE);
                    continue;
                }
                const float c = h2f(cf[k]);
                float* dst = wb + static_cast<uint64_t>(idx[k]) * RP;
                if constexpr (RP >= 4) {
#pragma unroll
                    for (int r = 0; r < RP; r += 4)
                        red_add_v4(dst + r, c * p[r], c * p[r + 1], c * p[r + 2], c * p[r + 3]);
                } else {
#pragma unroll
                    for (int r = 0; r < RP; ++r) atomicAdd(dst + r, c * p[r]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RP; ++r) {
        const float sm = warp_sum(p[r]);
        if (lane == 0) red[warp][r] = sm;
    }
    __syncthreads();
    if (t < RP) {
        float sm = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sm += red[w][t];
        a.csum[(static_cast<uint64_t>(ci) * a.Hkv + g) * RP + t] = sm;
    }
}

// ---------------------------------------------------------------------------
// The same two passes for 32+ query rows per kv head (speculative verify):
// lane = query row (RP / 32 rows per lane), so every q_latent gather, score
// store and weight update of a (token, atom) is one coalesced 128-byte access
// per 32 rows instead of a thread's RP / 4 16-byte ones.  Warp w owns the
// item's tokens 32w .. 32w + 31 (an item is at most 16 blocks = 256 tokens):
// its lanes first load those 32 tokens' codes (and block references) at
// once, then walk the tokens, taking each code from its lane by shuffles.
// ---------------------------------------------------------------------------
static_assert(kColdItemPages * kBlock == 256, "row-lane cold passes: 8 warps x 32 tokens per item");

// Code of this lane's token (32w + lane) of the item, and whether its block is valid.
__device__ __forceinline__ uint4 row_lane_code(const RunArgs& a, const ColdItem& item, const uint4* pool, uint32_t g,
                                               uint32_t warp, uint32_t lane, uint32_t ntok, bool& valid) {
    const uint32_t tok = warp * 32 + lane;
    valid = false;
    if (tok >= ntok) return make_uint4(0, 0, 0, 0);
    const uint32_t phys = a.cold_refs[item.page_begin + tok / kBlock] & kRefMask;
    valid = phys < a.cold_pool_blocks;
    return valid ? __ldg(&pool[(static_cast<uint64_t>(phys) * kBlock + tok % kBlock) * a.Hkv + g]) : make_uint4(0, 0, 0, 0);
}

template <int RP>
__global__ void __launch_bounds__(256) cold_score_rows_kernel(const RunArgs a) {
    constexpr int RPL = RP / 32;
    __shared__ float red[8][RP];
    // kv heads fastest in launch order (one item's head CTAs share its code lines)
    const uint32_t ci = blockIdx.y + blockIdx.z * gridDim.y, g = blockIdx.x;
    if (ci >= a.n_cold_items) return;
    const ColdItem item = a.cold_items[ci];
    const uint32_t b = item.seq;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ntok = (item.page_end - item.page_begin) * kBlock;
    const float* base = a.qlat + (static_cast<uint64_t>(b) * a.Hkv + g) * a.A * RP + lane;
    bool valid;
    const uint4 mine = row_lane_code(a, item, a.cold_k, g, warp, lane, ntok, valid);
    if (warp * 32 + lane < ntok && !valid) atomicOr(a.status, DEVERR_REF_RANGE);
    const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
    const uint32_t nt = ntok > warp * 32 ? min(32u, ntok - warp * 32) : 0u;
    float mx[RPL];
#pragma unroll
    for (int j = 0; j < RPL; ++j) mx[j] = -INFINITY;
    bool bad_atom = false;
#pragma unroll 4
    for (uint32_t t = 0; t < nt; ++t) {
        const uint32_t cx = __shfl_sync(0xffffffffu, mine.x, t), cy = __shfl_sync(0xffffffffu, mine.y, t);
        const uint32_t cz = __shfl_sync(0xffffffffu, mine.z, t), cw = __shfl_sync(0xffffffffu, mine.w, t);
        const uint32_t iw[2] = {cx, cy}, fw[2] = {cz, cw};
        float s[RPL];
#pragma unroll
        for (int j = 0; j < RPL; ++j) s[j] = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t idx = (iw[k >> 1] >> (16 * (k & 1))) & 0xFFFFu;
            const float c = h2f(static_cast<uint16_t>(fw[k >> 1] >> (16 * (k & 1))));
            const bool ok = idx < a.A;
            bad_atom |= !ok;
#pragma unroll
            for (int j = 0; j < RPL; ++j)
                s[j] = fmaf(c, ok ? __ldcg(base + static_cast<uint64_t>(idx) * RP + 32 * j) : 0.0f, s[j]);
        }
        const bool vt = (vmask >> t) & 1u;
        const uint32_t tok = warp * 32 + t;
        float* dst = a.scores + (static_cast<uint64_t>(g) * a.cold_tokens +
                                 static_cast<uint64_t>(item.page_begin) * kBlock + tok) * RP + lane;
#pragma unroll
        for (int j = 0; j < RPL; ++j) {
            const float sv = vt ? s[j] : -INFINITY;
            dst[32 * j] = sv;
            mx[j] = fmaxf(mx[j], sv);
        }
    }
    if (bad_atom && (vmask != 0)) atomicOr(a.status, DEVERR_ATOM_RANGE);
#pragma unroll
    for (int j = 0; j < RPL; ++j) red[warp][lane + 32 * j] = mx[j];
    __syncthreads();
    for (uint32_t r = threadIdx.x; r < RP; r += 256) {
        float m = red[0][r];
#pragma unroll
        for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w][r]);
        a.cmax[(static_cast<uint64_t>(ci) * a.Hkv + g) * RP + r] = m;
    }
}

template <int RP>
__global__ void __launch_bounds__(256) cold_scatter_rows_kernel(const RunArgs a) {
    constexpr int RPL = RP / 32;
    __shared__ float red[8][RP];
    // kv heads fastest in launch order (one item's head CTAs share its code lines)
    const uint32_t ci = blockIdx.y + blockIdx.z * gridDim.y, g = blockIdx.x;
    if (ci >= a.n_cold_items) return;
    const ColdItem item = a.cold_items[ci];
    const uint32_t b = item.seq;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ntok = (item.page_end - item.page_begin) * kBlock;
    bool valid;
    const uint4 mine = row_lane_code(a, item, a.cold_v, g, warp, lane, ntok, valid);
    const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
    const uint32_t nt = ntok > warp * 32 ? min(32u, ntok - warp * 32) : 0u;
    // the sequence-wide maximum of each of this lane's rows
    float M[RPL];
    {
        const uint32_t i0 = a.cold_item_ptr[b], i1 = a.cold_item_ptr[b + 1];
#pragma unroll
        for (int j = 0; j < RPL; ++j) {
            float m = -INFINITY;
            for (uint32_t it = i0; it < i1; ++it)
                m = fmaxf(m, __ldcg(&a.cmax[(static_cast<uint64_t>(it) * a.Hkv + g) * RP + lane + 32 * j]));
            M[j] = m;
        }
    }
    float* wb = a.w + (static_cast<uint64_t>(b) * a.Hkv + g) * a.A * RP + lane;
    const float* sb = a.scores + (static_cast<uint64_t>(g) * a.cold_tokens + static_cast<uint64_t>(item.page_begin) * kBlock +
                                  warp * 32) * RP + lane;
    float ls[RPL];
#pragma unroll
    for (int j = 0; j < RPL; ++j) ls[j] = 0.0f;
#pragma unroll 4
    for (uint32_t t = 0; t < nt; ++t) {
        const uint32_t cx = __shfl_sync(0xffffffffu, mine.x, t), cy = __shfl_sync(0xffffffffu, mine.y, t);
        const uint32_t cz = __shfl_sync(0xffffffffu, mine.z, t), cw = __shfl_sync(0xffffffffu, mine.w, t);
        if (!((vmask >> t) & 1u)) continue;  // flagged by the score pass
        const uint32_t iw[2] = {cx, cy}, fw[2] = {cz, cw};
        float p[RPL];
#pragma unroll
        for (int j = 0; j < RPL; ++j) {
            p[j] = exp_shift(__ldcg(sb + static_cast<uint64_t>(t) * RP + 32 * j), M[j]);
            ls[j] += p[j];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t idx = (iw[k >> 1] >> (16 * (k & 1))) & 0xFFFFu;
            if (idx >= a.A) continue;  // flagged by the score pass when the K code shares it; V codes checked here
            const float c = h2f(static_cast<uint16_t>(fw[k >> 1] >> (16 * (k & 1))));
#pragma unroll
            for (int j = 0; j < RPL; ++j) atomicAdd(wb + static_cast<uint64_t>(idx) * RP + 32 * j, c * p[j]);
        }
    }
    // V-code atom indices out of range
    {
        bool bad = false;
        if (valid)
            for (int k = 0; k < 4; ++k)
                bad |= ((((k < 2) ? mine.x : mine.y) >> (16 * (k & 1))) & 0xFFFFu) >= a.A;
        if (bad) atomicOr(a.status, DEVERR_ATOM_RANGE);
    }
#pragma unroll
    for (int j = 0; j < RPL; ++j) red[warp][lane + 32 * j] = ls[j];
    __syncthreads();
    for (uint32_t r = threadIdx.x; r < RP; r += 256) {
        float sm = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) sm += red[w][r];
        a.csum[(static_cast<uint64_t>(ci) * a.Hkv + g) * RP + r] = sm;
    }
}

// ---------------------------------------------------------------------------
// o_cold partial = w[tile] . V_dict[tile] for one 128-atom tile.
// grid (atom tile, kv head, sequence); 4 warps x 32 atoms, lane owns dims.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) cold_contract_kernel(const __grid_constant__ CUtensorMap tm_vdict,
                                                            const RunArgs a) {
    constexpr int kBoxes = D / 64;
    constexpr uint32_t kBoxBytes = kAtomTile * 128;
    constexpr int VPL = D / 32;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align_1024(smem_raw);
    uint8_t* tile = smem;
    const uint32_t rpad = ((a.RP + 7) / 8) * 8;
    float* w_s = reinterpret_cast<float*>(smem + kBoxes * kBoxBytes);   // [128][rpad]
    float* comb = w_s + kAtomTile * rpad;                               // [4][8][D]
    uint64_t* bar = reinterpret_cast<uint64_t*>(comb + 4 * 8 * D);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t t = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, kBoxes * kBoxBytes);
        const int32_t y = static_cast<int32_t>(g * a.dict_row_stride + t * kAtomTile);
#pragma unroll
        for (int bx = 0; bx < kBoxes; ++bx) tma_load_2d(tile + bx * kBoxBytes, &tm_vdict, bar, bx * 64, y);
    }
    const uint64_t wbase = ((static_cast<uint64_t>(b) * a.Hkv + g) * a.A + static_cast<uint64_t>(t) * kAtomTile) * a.RP;
    for (uint32_t idx = tid; idx < kAtomTile * rpad; idx += blockDim.x) {
        const uint32_t row = idx / rpad, r = idx % rpad;
        float v = 0.0f;
        if (t * kAtomTile + row < a.A && r < a.RP) v = a.w[wbase + static_cast<uint64_t>(row) * a.RP + r];
        w_s[idx] = v;
    }
    __syncthreads();
    const bool ok = mbar_wait(bar, 0, a.status);

    for (uint32_t rg = 0; rg < rpad; rg += 8) {
        float o[8][VPL];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int e = 0; e < VPL; ++e) o[r][e] = 0.0f;
        if (ok) {
#pragma unroll 4
            for (int i = 0; i < 32; ++i) {
                const uint32_t row = warp * 32 + i;
                float vf[VPL];
                if (D == 128) {
                    const uint32_t bx = lane >> 4, chunk = (lane & 15) >> 1;
                    const uint2 raw = *reinterpret_cast<const uint2*>(
                        tile + bx * kBoxBytes + swz128(row, chunk) + (lane & 1) * 8);
                    h4_to_f4(raw, vf);
                } else {
                    const uint32_t chunk = lane >> 2;
                    const uint32_t raw = *reinterpret_cast<const uint32_t*>(tile + swz128(row, chunk) + (lane & 3) * 4);
                    const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&raw));
                    vf[0] = v2.x;
                    vf[VPL - 1] = v2.y;
                }
                const float* wr = w_s + row * rpad + rg;
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const float wv = wr[r];
#pragma unroll
                    for (int e = 0; e < VPL; ++e) o[r][e] = fmaf(wv, vf[e], o[r][e]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int e = 0; e < VPL; ++e) comb[(warp * 8 + r) * D + lane * VPL + e] = o[r][e];
        __syncthreads();
        for (uint32_t idx = tid; idx < 8 * D; idx += blockDim.x) {
            const uint32_t r = idx / D, dim = idx % D;
            if (rg + r >= a.RP) continue;
            const float sm = comb[(0 * 8 + r) * D + dim] + comb[(1 * 8 + r) * D + dim] +
                             comb[(2 * 8 + r) * D + dim] + comb[(3 * 8 + r) * D + dim];
            a.ocold[((((static_cast<uint64_t>(b) * a.Hkv + g) * a.n_atom_tiles + t) * a.RP) + rg + r) * D + dim] = sm;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Log-sum-exp merge of hot chunk partials and the cold partial; one CTA per
// query row (b, j, h), kMergeGroups threads per dim.
// ---------------------------------------------------------------------------
constexpr uint32_t kMergeGroups = 4;

__global__ void merge_kernel(const RunArgs a) {
    // kMergeGroups groups of D threads (one per dimension); the maxima and the
    // cold sum are reduced over all threads, the hot partials and the cold
    // contraction partials are split over the groups (a long context has
    // hundreds of cold items and tens of hot partials per row: few loads per
    // thread in flight, one pass over shared memory to combine)
    __shared__ float red[3][32];
    __shared__ float og[kMergeGroups][129];  // D <= 128
    __shared__ float lg[kMergeGroups];
    const uint32_t row = blockIdx.x, tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t D = a.D, dim = tid % D, grp = tid / D;
    const uint32_t h = row % a.Hq, j = (row / a.Hq) % a.nq, b = row / (a.Hq * a.nq);
    const uint32_t g = h / a.G, r = j * a.G + h % a.G;
    const uint32_t h0 = a.hot_item_ptr[b], h1 = a.hot_item_ptr[b + 1];
    const uint32_t c0 = a.cold_item_ptr[b], c1 = a.cold_item_ptr[b + 1];
    float mh = -INFINITY, mc = -INFINITY, lcs = 0.0f;
    for (uint32_t it = h0 + tid; it < h1; it += nt) mh = fmaxf(mh, a.hm[(static_cast<uint64_t>(it) * a.Hkv + g) * a.RP + r]);
    for (uint32_t it = c0 + tid; it < c1; it += nt) {
        const uint64_t ci = (static_cast<uint64_t>(it) * a.Hkv + g) * a.RP + r;
        mc = fmaxf(mc, a.cmax[ci]);
        lcs += a.csum[ci];
    }
    mh = warp_max(mh);
    mc = warp_max(mc);
    lcs = warp_sum(lcs);
    if (lane == 0) {
        red[0][warp] = mh;
        red[1][warp] = mc;
        red[2][warp] = lcs;
    }
    __syncthreads();
    float M = -INFINITY, Mc = -INFINITY, lc = 0.0f;
    for (uint32_t w = 0; w < nt / 32; ++w) {
        M = fmaxf(M, red[0][w]);
        Mc = fmaxf(Mc, red[1][w]);
        lc += red[2][w];
    }
    M = fmaxf(M, Mc);
    float L = 0.0f, O = 0.0f;
    for (uint32_t it = h0 + grp; it < h1; it += kMergeGroups) {
        const uint64_t pi = (static_cast<uint64_t>(it) * a.Hkv + g) * a.RP + r;
        const float f = exp_shift(a.hm[pi], M);
        L += a.hl[pi] * f;
        O += a.ho[pi * D + dim] * f;
    }
    if (c1 > c0) {
        const float f = exp_shift(Mc, M);
        const uint64_t ob = ((static_cast<uint64_t>(b) * a.Hkv + g) * a.n_atom_tiles) * a.RP;
        float oc = 0.0f;
        for (uint32_t t = grp; t < a.n_atom_tiles; t += kMergeGroups)
            oc += a.ocold[(ob + static_cast<uint64_t>(t) * a.RP + r) * D + dim];
        if (grp == 0) L += lc * f;
        O += oc * f;
    }
    og[grp][dim] = O;
    if (dim == 0) lg[grp] = L;
    __syncthreads();
    if (grp) return;
    O = 0.0f;
    L = 0.0f;
#pragma unroll
    for (uint32_t q = 0; q < kMergeGroups; ++q) {
        O += og[q][dim];
        L += lg[q];
    }
    if (a.flags & 4u) {  // WEAVER_FLAG_PARTIALS
        if (dim == 0) {
            a.part_m[row] = M;
            a.part_l[row] = L;
        }
        a.part_o[static_cast<uint64_t>(row) * D + dim] = O;
    } else {
        a.out[static_cast<uint64_t>(row) * D + dim] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
    }
}

// Part p's statistics at m/l + p * ml_stride, its outputs at o + p * o_stride.
__global__ void merge_partials_kernel(uint32_t n_parts, uint32_t rows, uint32_t D, const float* m,
                                      const float* l, const float* o, uint64_t ml_stride, uint64_t o_stride,
                                      __half* out) {
    const uint32_t row = blockIdx.x, dim = threadIdx.x;
    float M = -INFINITY;
    for (uint32_t p = 0; p < n_parts; ++p) M = fmaxf(M, m[p * ml_stride + row]);
    float L = 0.0f, O = 0.0f;
    for (uint32_t p = 0; p < n_parts; ++p) {
        const float f = exp_shift(m[p * ml_stride + row], M);
        L += l[p * ml_stride + row] * f;
        O += o[p * o_stride + static_cast<uint64_t>(row) * D + dim] * f;
    }
    out[static_cast<uint64_t>(row) * D + dim] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
}

// ---------------------------------------------------------------------------
// Atom selection (distiller.rs:185-234): 8 rows of one kv head per CTA, one
// warp per row; dictionary tiles staged in shared memory and shared by the 8
// rows.  Dots are summed in dimension order from -0.0 (each f16*f16 product
// is exact in fp32, so the fused multiply-add rounds like a separate add).
// ---------------------------------------------------------------------------
namespace {
__device__ __forceinline__ bool ranks_before(float sa, uint32_t ia, float sb, uint32_t ib) {
    const bool na = isnan(sa), nb = isnan(sb);
    if (na != nb) return nb;
    if (!na && sa != sb) return sa > sb;
    return ia < ib;
}
}  // namespace

template <int D>
__global__ void __launch_bounds__(256) distill_kernel(const __half* rows, uint32_t n_rows,
                                                      uint32_t kv_heads, const __half* dict,
                                                      uint32_t A, uint64_t dict_head_stride,
                                                      uint4* out, const uint32_t* src_blocks,
                                                      const uint32_t* dst_blocks, uint64_t src_limit,
                                                      uint64_t dst_limit, uint32_t* bad) {
    constexpr int kTile = 64;
    constexpr int kPitch = D + 8;  // halves; breaks bank alignment of rows
    // block-list mode (migration): grid row y distills hot block src_blocks[y]
    // (n_rows rows) into cold block dst_blocks[y]; out-of-range blocks are
    // skipped and reported
    if (src_blocks) {
        const uint32_t sb = src_blocks[blockIdx.y], db = dst_blocks[blockIdx.y];
        if (sb >= src_limit || db >= dst_limit) {
            if (threadIdx.x == 0) atomicOr(bad, 1u);
            return;
        }
        rows += static_cast<uint64_t>(sb) * n_rows * D;
        out += static_cast<uint64_t>(db) * n_rows;
    }
    __shared__ __align__(16) __half dsm[kTile * kPitch];
    __shared__ __align__(16) float xs[8][D];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // CTA c covers rows {g + kv_heads * (8*k + warp)} of head g = c % kv_heads
    const uint32_t g = blockIdx.x % kv_heads;
    const uint32_t group = blockIdx.x / kv_heads;
    const uint32_t ridx = g + kv_heads * (group * 8 + warp);
    const bool has_row = ridx < n_rows;
    for (uint32_t i = lane; i < D; i += 32)
        xs[warp][i] = has_row ? __half2float(rows[static_cast<uint64_t>(ridx) * D + i]) : 0.0f;
    const __half* dg = dict + static_cast<uint64_t>(g) * dict_head_stride;
    float bs[4];
    uint32_t bi[4];
    int nb = 0;
    for (uint32_t a0 = 0; a0 < A; a0 += kTile) {
        __syncthreads();
        for (uint32_t i = threadIdx.x; i < kTile * (D / 8); i += blockDim.x) {
            const uint32_t r = i / (D / 8), c = i % (D / 8);
            uint4 v = make_uint4(0, 0, 0, 0);
            if (a0 + r < A) v = *reinterpret_cast<const uint4*>(dg + static_cast<uint64_t>(a0 + r) * D + c * 8);
            *reinterpret_cast<uint4*>(&dsm[r * kPitch + c * 8]) = v;
        }
        __syncthreads();
        for (uint32_t rr = lane; rr < kTile; rr += 32) {
            const uint32_t atom = a0 + rr;
            if (atom >= A) break;
            float s = -0.0f;
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
                const uint4 raw = *reinterpret_cast<const uint4*>(&dsm[rr * kPitch + c * 8]);
                float kf[8];
                h8_to_f8(raw, kf);
#pragma unroll
                for (int e = 0; e < 8; ++e) s = __fmaf_rn(xs[warp][c * 8 + e], kf[e], s);
            }
            int pos = nb;
            while (pos > 0 && ranks_before(s, atom, bs[pos - 1], bi[pos - 1])) --pos;
            if (pos < 4) {
                for (int q = (nb < 4 ? nb : 3); q > pos; --q) {
                    bs[q] = bs[q - 1];
                    bi[q] = bi[q - 1];
                }
                bs[pos] = s;
                bi[pos] = atom;
                if (nb < 4) ++nb;
            }
        }
    }
    // merge the 32 per-lane top-4 lists: 4 rounds of a warp arg-best
    uint16_t oi[4] = {0, 0, 0, 0};
    uint16_t oc[4] = {0, 0, 0, 0};
    int head = 0;
    for (int k = 0; k < 4; ++k) {
        const bool have = head < nb;
        float cs = have ? bs[head] : 0.0f;
        uint32_t ci = have ? bi[head] : 0xFFFFFFFFu;
        uint32_t cl = have ? lane : 0xFFFFFFFFu;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float os = __shfl_xor_sync(0xffffffffu, cs, off);
            const uint32_t oi_ = __shfl_xor_sync(0xffffffffu, ci, off);
            const uint32_t ol = __shfl_xor_sync(0xffffffffu, cl, off);
            bool take;
            if (ol == 0xFFFFFFFFu) take = false;
            else if (cl == 0xFFFFFFFFu) take = true;
            else take = ranks_before(os, oi_, cs, ci);
            if (take) {
                cs = os;
                ci = oi_;
                cl = ol;
            }
        }
        if (cl == 0xFFFFFFFFu) break;  // fewer than 4 atoms in the dictionary
        oi[k] = static_cast<uint16_t>(ci);
        oc[k] = __half_as_ushort(__float2half_rn(cs));
        if (lane == cl) ++head;
    }
    if (has_row && lane == 0) {
        uint4 code;
        code.x = oi[0] | (static_cast<uint32_t>(oi[1]) << 16);
        code.y = oi[2] | (static_cast<uint32_t>(oi[3]) << 16);
        code.z = oc[0] | (static_cast<uint32_t>(oc[1]) << 16);
        code.w = oc[2] | (static_cast<uint32_t>(oc[3]) << 16);
        out[ridx] = code;
    }
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
namespace {
// Raise a kernel's dynamic shared memory limit once (not inside graph captures).
template <auto Kernel>
cudaError_t smem_once(size_t bytes) {
    static size_t done = 0;  // one counter per kernel instantiation
    if (bytes <= done) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess) done = bytes;
    return e;
}

template <int D, int RM>
cudaError_t launch_hot_t(const RunArgs& a, const CUtensorMap& tk, const CUtensorMap& tv, uint32_t rgroups,
                         cudaStream_t s) {
    constexpr int kStages = 8, kCons = 4;
    constexpr size_t stage = 2 * (D / 64) * kBlock * 128;
    const size_t smem = 1024 + kStages * stage + sizeof(float) * (RM * D + kCons * RM * 16 + 2 * kCons * RM + kCons * RM * D) +
                        sizeof(int) * kStages + 2 * kStages * sizeof(uint64_t) + 16;
    auto k = hot_kernel<D, RM>;
    cudaError_t e = smem_once<hot_kernel<D, RM>>(smem);
    if (e != cudaSuccess) return e;
    dim3 grid(a.n_hot_items, a.Hkv, rgroups);
    k<<<grid, 160, smem, s>>>(tk, tv, a);
    return cudaGetLastError();
}

template <int RP>
cudaError_t launch_cold_t(const RunArgs& a, cudaStream_t s, bool scatter) {
    const uint32_t gy = a.n_cold_items < 65535u ? a.n_cold_items : 65535u;
    dim3 grid(a.Hkv, gy, (a.n_cold_items + gy - 1) / gy);
    if constexpr (RP >= 32) {
        // WEAVER_COLD_PER_THREAD=1 keeps the thread-per-token kernels
        const char* env = getenv("WEAVER_COLD_PER_THREAD");
        if (!(env && env[0] == '1')) {
            if (scatter) cold_scatter_rows_kernel<RP><<<grid, 256, 0, s>>>(a);
            else cold_score_rows_kernel<RP><<<grid, 256, 0, s>>>(a);
            return cudaGetLastError();
        }
    }
    if (scatter) cold_scatter_kernel<RP><<<grid, 256, 0, s>>>(a);
    else cold_score_kernel<RP><<<grid, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_cold_any(const RunArgs& a, cudaStream_t s, bool scatter) {
    switch (a.RP) {
        case 1: return launch_cold_t<1>(a, s, scatter);
        case 2: return launch_cold_t<2>(a, s, scatter);
        case 4: return launch_cold_t<4>(a, s, scatter);
        case 8: return launch_cold_t<8>(a, s, scatter);
        case 16: return launch_cold_t<16>(a, s, scatter);
        case 32: return launch_cold_t<32>(a, s, scatter);
        case 64: return launch_cold_t<64>(a, s, scatter);
        default: return cudaErrorInvalidValue;
    }
}
}  // namespace

cudaError_t launch_hot(const RunArgs& a, const CUtensorMap& tk, const CUtensorMap& tv, uint32_t rgroups,
                       cudaStream_t s) {
    if (a.n_hot_items == 0) return cudaSuccess;
    const uint32_t rm = a.R >= kHotRows ? kHotRows : a.RP;
    if (a.D == 128) {
        switch (rm) {
            case 1: return launch_hot_t<128, 1>(a, tk, tv, rgroups, s);
            case 2: return launch_hot_t<128, 2>(a, tk, tv, rgroups, s);
            case 4: return launch_hot_t<128, 4>(a, tk, tv, rgroups, s);
            default: return launch_hot_t<128, 8>(a, tk, tv, rgroups, s);
        }
    }
    switch (rm) {
        case 1: return launch_hot_t<64, 1>(a, tk, tv, rgroups, s);
        case 2: return launch_hot_t<64, 2>(a, tk, tv, rgroups, s);
        case 4: return launch_hot_t<64, 4>(a, tk, tv, rgroups, s);
        default: return launch_hot_t<64, 8>(a, tk, tv, rgroups, s);
    }
}

cudaError_t launch_qlat(const RunArgs& a, const CUtensorMap& tm, cudaStream_t s) {
    const uint32_t rpad = ((a.RP + 7) / 8) * 8;
    const size_t smem = 1024 + (a.D / 64) * kAtomTile * 128 + sizeof(float) * rpad * a.D + 16;
    dim3 grid(a.n_atom_tiles, a.Hkv, a.B);
    cudaError_t e;
    if (a.D == 128) {
        e = smem_once<qlat_kernel<128>>(smem);
        if (e != cudaSuccess) return e;
        qlat_kernel<128><<<grid, 128, smem, s>>>(tm, a);
    } else {
        e = smem_once<qlat_kernel<64>>(smem);
        if (e != cudaSuccess) return e;
        qlat_kernel<64><<<grid, 128, smem, s>>>(tm, a);
    }
    return cudaGetLastError();
}

cudaError_t launch_qlat_import(const RunArgs& a, cudaStream_t s) {
    const uint64_t total = static_cast<uint64_t>(a.B) * a.Hkv * a.A * a.RP;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks == 0) blocks = 1;
    qlat_import_kernel<<<static_cast<uint32_t>(blocks), 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_cold_score(const RunArgs& a, cudaStream_t s) {
    if (a.n_cold_items == 0) return cudaSuccess;
    return launch_cold_any(a, s, false);
}

cudaError_t launch_cold_scatter(const RunArgs& a, cudaStream_t s) {
    if (a.n_cold_items == 0) return cudaSuccess;
    return launch_cold_any(a, s, true);
}

cudaError_t launch_cold_contract(const RunArgs& a, const CUtensorMap& tm, cudaStream_t s) {
    if (a.n_cold_items == 0) return cudaSuccess;
    const uint32_t rpad = ((a.RP + 7) / 8) * 8;
    const size_t smem = 1024 + (a.D / 64) * kAtomTile * 128 + sizeof(float) * (kAtomTile * rpad + 4 * 8 * a.D) + 16;
    dim3 grid(a.n_atom_tiles, a.Hkv, a.B);
    cudaError_t e;
    if (a.D == 128) {
        e = smem_once<cold_contract_kernel<128>>(smem);
        if (e != cudaSuccess) return e;
        cold_contract_kernel<128><<<grid, 128, smem, s>>>(tm, a);
    } else {
        e = smem_once<cold_contract_kernel<64>>(smem);
        if (e != cudaSuccess) return e;
        cold_contract_kernel<64><<<grid, 128, smem, s>>>(tm, a);
    }
    return cudaGetLastError();
}

cudaError_t launch_merge(const RunArgs& a, cudaStream_t s) {
    const uint32_t rows = a.B * a.nq * a.Hq;
    merge_kernel<<<rows, a.D * kMergeGroups, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_merge_partials(uint32_t n_parts, uint32_t rows, uint32_t D, const float* m, const float* l,
                                  const float* o, __half* out, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    merge_partials_kernel<<<rows, D, 0, s>>>(n_parts, rows, D, m, l, o, rows, static_cast<uint64_t>(rows) * D, out);
    return cudaGetLastError();
}

cudaError_t launch_merge_partials_strided(uint32_t n_parts, uint32_t rows, uint32_t D, const float* m,
                                          const float* l, const float* o, uint64_t part_stride, __half* out,
                                          cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    merge_partials_kernel<<<rows, D, 0, s>>>(n_parts, rows, D, m, l, o, part_stride, part_stride, out);
    return cudaGetLastError();
}

cudaError_t launch_distill(const __half* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t D, const __half* dict,
                           uint32_t A, uint64_t dict_head_stride, uint4* out, cudaStream_t s) {
    if (n_rows == 0) return cudaSuccess;
    const uint32_t per_head = (n_rows + kv_heads - 1) / kv_heads;
    const uint32_t groups = (per_head + 7) / 8;
    dim3 grid(groups * kv_heads);
    if (D == 128)
        distill_kernel<128><<<grid, 256, 0, s>>>(rows, n_rows, kv_heads, dict, A, dict_head_stride, out, nullptr, nullptr,
                                                 0, 0, nullptr);
    else
        distill_kernel<64><<<grid, 256, 0, s>>>(rows, n_rows, kv_heads, dict, A, dict_head_stride, out, nullptr, nullptr,
                                                0, 0, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_distill_blocks(const __half* pool, uint64_t pool_blocks, const uint32_t* src_blocks,
                                  const uint32_t* dst_blocks, uint32_t n_blocks, uint32_t kv_heads, uint32_t D,
                                  const __half* dict, uint32_t A, uint64_t dict_head_stride, uint4* cold,
                                  uint64_t cold_blocks, uint32_t* bad, cudaStream_t s) {
    if (n_blocks == 0) return cudaSuccess;
    const uint32_t rows = kBlock * kv_heads;  // one block: [16 tokens][kv_heads] rows of D
    const uint32_t groups = (kBlock + 7) / 8;
    dim3 grid(groups * kv_heads, n_blocks);
    if (D == 128)
        distill_kernel<128><<<grid, 256, 0, s>>>(pool, rows, kv_heads, dict, A, dict_head_stride, cold, src_blocks,
                                                 dst_blocks, pool_blocks, cold_blocks, bad);
    else
        distill_kernel<64><<<grid, 256, 0, s>>>(pool, rows, kv_heads, dict, A, dict_head_stride, cold, src_blocks,
                                                dst_blocks, pool_blocks, cold_blocks, bad);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Distiller::evaluate_entropy's proxy (nexus-core/src/distiller.rs:97-159):
// the variance of a hot block's f16 values (every token and kv head), the
// sum and the squared deviations accumulated in fp64, 0 for an all-zero
// block.  One warp per block; lanes take 8 values at a time, fixed
// reduction order (deterministic).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) block_entropy_kernel(const __half* pool, uint64_t n_blocks,
                                                            uint32_t vals_per_block, float* out) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t blk = static_cast<uint64_t>(blockIdx.x) * 8 + warp;
    if (blk >= n_blocks) return;
    const uint4* p = reinterpret_cast<const uint4*>(pool + blk * vals_per_block);
    const uint32_t n8 = vals_per_block / 8;
    double sum = 0.0;
    bool nz = false;
    for (uint32_t i = lane; i < n8; i += 32) {
        float f[8];
        h8_to_f8(__ldg(p + i), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            sum += static_cast<double>(f[e]);
            nz |= f[e] != 0.0f;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    nz = __any_sync(0xffffffffu, nz);
    const double mean = sum / static_cast<double>(vals_per_block);
    double var = 0.0;
    for (uint32_t i = lane; i < n8; i += 32) {
        float f[8];
        h8_to_f8(__ldg(p + i), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const double d = static_cast<double>(f[e]) - mean;
            var += d * d;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    if (lane == 0) out[blk] = nz ? static_cast<float>(var / static_cast<double>(vals_per_block)) : 0.0f;
}

cudaError_t launch_block_entropy(const __half* pool, uint64_t n_blocks, uint32_t vals_per_block, float* out,
                                 cudaStream_t s) {
    if (n_blocks == 0) return cudaSuccess;
    block_entropy_kernel<<<static_cast<uint32_t>((n_blocks + 7) / 8), 256, 0, s>>>(pool, n_blocks, vals_per_block, out);
    return cudaGetLastError();
}

}  // namespace weaver
