// weaver_cold_smem.cu — the multi-kernel step's two cold passes with one kv
// head's q_latent (scoring) or per-atom weights (scatter) held in a CTA's
// shared memory instead of gathered from / reduced into L2 (the scores and
// values of weaver_kernel.metal:170-221).
//
// Work split: a CTA takes one chunk (a run of consecutive cold items of one
// sequence b, plan-built so that the chunks of all (kv head, row slice) pairs
// fill the GPU about once), one kv head g and one slice of RS query rows
// (rows r0 .. r0 + RS - 1 of the RP padded rows; RS is the largest power of
// two <= RP whose A x RS fp32 table fits shared memory).
//
//   * score pass: the (b, g) q_latent rows (written as fp32 by the q_latent
//     kernel) are copied into shared memory once as f16 (the precision of the
//     reference's q_latent input, weaver.rs:139-237), so one 16-byte gather
//     serves 8 query rows: a score CTA takes RSS = min(RP, 8) rows of a part
//     of the chunk (the same grid as the scatter: RP / RS slices of RS rows
//     become RSS / RS parts of the chunk's items).  Each thread takes tokens,
//     reads the token's K code (16 B), gathers its four atoms' RSS values,
//     writes the RSS scores and keeps a running maximum, an exponential sum
//     and the largest sum of a token's |K coefficients|.  The part's maximum
//     goes to its first item in cmax (its other items get -inf), so every
//     reader that takes the maximum over a sequence's items sees the same
//     value; its exponential sum times that coefficient sum goes to cbound,
//     the scatter's guess of each row's sum of |coeff * p| terms.
//   * scatter pass: the sequence-wide maximum M (over cmax of b's items, made
//     complete by the kernel boundary) shifts the exponentials; each token's
//     coeff * exp(s - M) is added into an RS x A weight table in shared
//     memory (fixed-point int32 atomics with a per-row scale, checked, else
//     fp32 atomics; no L2 round trip per token), and the CTA
//     writes the table once: a plain store when the chunk is the whole
//     sequence, else vector reductions into the zeroed global weights.  The
//     chunk's exponential sum goes to csum as cmax's value did.
// A bad block reference or atom index sets its status bit and is skipped, as
// in the other cold passes.
#include <cstdlib>

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr uint32_t kCsThreads = 512;
constexpr uint32_t kCsWarps = kCsThreads / 32;
constexpr uint32_t kCsRefBytes = kCsMaxPages * 4;    // the chunk's block references
constexpr uint32_t kCsTableMax = 216 * 1024;         // bytes of the A x RS table

// RS f16 values at p (shared memory, 2*RS-byte aligned) as fp32.
template <int RS>
__device__ __forceinline__ void lds_h_rows(const __half* p, float v[RS]) {
    if constexpr (RS == 8) {
        h8_to_f8(*reinterpret_cast<const uint4*>(p), v);
    } else if constexpr (RS == 4) {
        h4_to_f4(*reinterpret_cast<const uint2*>(p), v);
    } else if constexpr (RS == 2) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(p));
        v[0] = x.x;
        v[1] = x.y;
    } else {
        v[0] = __half2float(*p);
    }
}

// RS fp32 values from / to global memory (L2 only: written and read once).
template <int RS>
__device__ __forceinline__ void ldcg_rs(const float* p, float v[RS]) {
    if constexpr (RS >= 4) {
#pragma unroll
        for (int r = 0; r < RS; r += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(p + r));
            v[r] = x.x;
            v[r + 1] = x.y;
            v[r + 2] = x.z;
            v[r + 3] = x.w;
        }
    } else if constexpr (RS == 2) {
        const float2 x = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = x.x;
        v[1] = x.y;
    } else {
        v[0] = __ldcg(p);
    }
}

template <int RS>
__device__ __forceinline__ void stcg_rs(float* p, const float v[RS]) {
    if constexpr (RS >= 4) {
#pragma unroll
        for (int r = 0; r < RS; r += 4)
            __stcg(reinterpret_cast<float4*>(p + r), make_float4(v[r], v[r + 1], v[r + 2], v[r + 3]));
    } else if constexpr (RS == 2) {
        __stcg(reinterpret_cast<float2*>(p), make_float2(v[0], v[1]));
    } else {
        __stcg(p, v[0]);
    }
}

// The chunk's pages p0 .. p0 + ntok / 16 - 1 (indices into cold_refs).
struct ChunkSpan {
    uint32_t p0, ntok;
};

__device__ __forceinline__ ChunkSpan chunk_span(const RunArgs& a, const ColdChunk& ch) {
    const uint32_t p0 = a.cold_items[ch.item_begin].page_begin;
    const uint32_t p1 = a.cold_items[ch.item_end - 1].page_end;
    return ChunkSpan{p0, (p1 - p0) * kBlock};
}

// The chunk's physical blocks into shared memory (bit 31 masked; 0xFFFFFFFF
// for a reference beyond the pool, flagged when `flag`), so a token's code
// load depends on no other global load.  The plan keeps chunks within
// kCsMaxPages pages.
__device__ __forceinline__ void load_chunk_refs(uint32_t* refs, const RunArgs& a, const ChunkSpan& sp, bool flag) {
    for (uint32_t i = threadIdx.x; i < sp.ntok / kBlock; i += kCsThreads) {
        const uint32_t phys = a.cold_refs[sp.p0 + i] & kRefMask;
        const bool ok = phys < a.cold_pool_blocks;
        if (!ok && flag) atomicOr(a.status, DEVERR_REF_RANGE);
        refs[i] = ok ? phys : 0xFFFFFFFFu;
    }
}

// Writes the chunk's per-row value v[r] (rows r0..r0+RS-1) to its first item
// and `rest` to its other items; threads 0 .. RS-1 of the CTA.
template <int RS>
__device__ __forceinline__ void put_chunk_rows(float* dst, const RunArgs& a, const ColdChunk& ch, uint32_t g,
                                               uint32_t r0, float v, float rest, uint32_t r) {
    for (uint32_t it = ch.item_begin; it < ch.item_end; ++it)
        dst[(static_cast<uint64_t>(it) * a.Hkv + g) * a.RP + r0 + r] = it == ch.item_begin ? v : rest;
}

// TOK: tokens per thread in flight (4 where two CTAs share an SM: the
// register budget of two 512-thread CTAs)
template <int RS, int TOK>
__global__ void __launch_bounds__(kCsThreads, TOK == 4 ? 2 : 1) cold_score_smem_kernel(const RunArgs a) {
    extern __shared__ float4 cs_smem[];
    uint32_t* refs = reinterpret_cast<uint32_t*>(cs_smem);                 // [kCsMaxPages]
    __half* ql = reinterpret_cast<__half*>(cs_smem) + kCsRefBytes / 2;      // [A][RS] f16
    __shared__ float red[kCsWarps][RS];
    // blockIdx.z: row slice zs of RS rows and part zp of the chunk's items
    const uint32_t n_slices = a.RP / RS, parts = gridDim.z / n_slices;
    const uint32_t zs = blockIdx.z % n_slices, zp = blockIdx.z / n_slices;
    ColdChunk ch = a.cold_chunks[blockIdx.y];
    {
        const uint32_t n = ch.item_end - ch.item_begin;
        const uint32_t i0 = ch.item_begin + n * zp / parts, i1 = ch.item_begin + n * (zp + 1) / parts;
        if (i0 == i1) return;  // an empty part (the whole CTA)
        ch.item_begin = i0;
        ch.item_end = i1;
    }
    const uint32_t g = blockIdx.x, r0 = zs * RS, b = ch.seq;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t A = a.A, RP = a.RP, Hkv = a.Hkv;
    const ChunkSpan sp = chunk_span(a, ch);

    // the (b, g) q_latent rows r0 .. r0 + RS - 1 of every atom, as f16
    const float* src = a.qlat + (static_cast<uint64_t>(b) * Hkv + g) * A * RP + r0;
    for (uint32_t i = tid; i < A; i += kCsThreads) {
        float v[RS];
        ldcg_rs<RS>(src + static_cast<uint64_t>(i) * RP, v);
        __half h[RS];
#pragma unroll
        for (int r = 0; r < RS; ++r) h[r] = __float2half_rn(v[r]);
        if constexpr (RS == 8) {
            *reinterpret_cast<uint4*>(ql + i * RS) = *reinterpret_cast<const uint4*>(h);
        } else if constexpr (RS == 4) {
            *reinterpret_cast<uint2*>(ql + i * RS) = *reinterpret_cast<const uint2*>(h);
        } else {
#pragma unroll
            for (int r = 0; r < RS; ++r) ql[i * RS + r] = h[r];
        }
    }
    load_chunk_refs(refs, a, sp, true);
    __syncthreads();

    // mx: running maximum of each row's scores; bs: sum over the thread's
    // tokens of exp(s - mx), rescaled as mx grows; kc: the largest sum of a
    // token's |K coefficients|.  bs * kc guesses the scatter's sum of
    // |V coefficient * p| terms (the scatter checks it and falls back).
    float mx[RS], bs[RS], kc = 0.0f;
#pragma unroll
    for (int r = 0; r < RS; ++r) {
        mx[r] = -INFINITY;
        bs[r] = 0.0f;
    }
    for (uint32_t x0 = 0; x0 < sp.ntok; x0 += kCsThreads * TOK) {
        uint4 code[TOK];
        uint32_t tokg[TOK];
        bool live[TOK], in[TOK];
#pragma unroll
        for (uint32_t u = 0; u < TOK; ++u) {
            const uint32_t x = x0 + tid + u * kCsThreads;
            in[u] = x < sp.ntok;
            live[u] = false;
            code[u] = make_uint4(0, 0, 0, 0);
            const uint32_t pi = in[u] ? x / kBlock : 0u, tt = x % kBlock;
            tokg[u] = (sp.p0 + pi) * kBlock + tt;
            if (in[u]) {
                const uint32_t phys = refs[pi];
                if (phys != 0xFFFFFFFFu) {
                    live[u] = true;
                    code[u] = __ldg(&a.cold_k[(static_cast<uint64_t>(phys) * kBlock + tt) * Hkv + g]);
                }
            }
        }
#pragma unroll
        for (uint32_t u = 0; u < TOK; ++u) {
            if (!in[u]) continue;

            float s[RS];
#pragma unroll
            for (int r = 0; r < RS; ++r) s[r] = live[u] ? 0.0f : -INFINITY;
            if (live[u]) {
                const uint16_t* idx = reinterpret_cast<const uint16_t*>(&code[u].x);
                const uint16_t* cf = reinterpret_cast<const uint16_t*>(&code[u].z);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (idx[k] >= A) {
                        atomicOr(a.status, DEVERR_ATOM_RANGE);
                        continue;
                    }
                    const float c = h2f(cf[k]);
                    float v[RS];
                    lds_h_rows<RS>(ql + static_cast<uint32_t>(idx[k]) * RS, v);
#pragma unroll
                    for (int r = 0; r < RS; ++r) s[r] = fmaf(c, v[r], s[r]);
                }
            }
            stcg_rs<RS>(a.scores + (static_cast<uint64_t>(g) * a.cold_tokens + tokg[u]) * RP + r0, s);
            if (live[u]) {
                const uint16_t* cf = reinterpret_cast<const uint16_t*>(&code[u].z);
                kc = fmaxf(kc, (fabsf(h2f(cf[0])) + fabsf(h2f(cf[1]))) + (fabsf(h2f(cf[2])) + fabsf(h2f(cf[3]))));
#pragma unroll
                for (int r = 0; r < RS; ++r) {  // one exponential: exp(-|s - mx|) serves both cases
                    const float e = __expf(-fabsf(s[r] - mx[r]));
                    const bool up = s[r] > mx[r];
                    bs[r] = up ? fmaf(bs[r], e, 1.0f) : bs[r] + e;
                    mx[r] = up ? s[r] : mx[r];
                }
            }
        }
    }
    __shared__ float cm[RS];
#pragma unroll
    for (int r = 0; r < RS; ++r) {
        const float m = warp_max(mx[r]);
        if (lane == 0) red[warp][r] = m;
    }
    __syncthreads();
    if (tid < RS) {
        float m = red[0][tid];
#pragma unroll
        for (uint32_t w = 1; w < kCsWarps; ++w) m = fmaxf(m, red[w][tid]);
        cm[tid] = m;
        put_chunk_rows<RS>(a.cmax, a, ch, g, r0, m, -INFINITY, tid);
    }
    __shared__ float kcw[kCsWarps];
    __syncthreads();
    kc = warp_max(kc);
    if (lane == 0) kcw[warp] = kc;
#pragma unroll
    for (int r = 0; r < RS; ++r) {
        const float b2 = warp_sum(bs[r] * exp_shift(mx[r], cm[r]));
        if (lane == 0) red[warp][r] = b2;
    }
    __syncthreads();
    if (tid < RS) {
        float b2 = 0.0f, k2 = 0.0f;
#pragma unroll
        for (uint32_t w = 0; w < kCsWarps; ++w) {
            b2 += red[w][tid];
            k2 = fmaxf(k2, kcw[w]);
        }
        put_chunk_rows<RS>(a.cbound, a, ch, g, r0, b2 * k2, 0.0f, tid);
    }
}

template <int RS, int TOK>
__global__ void __launch_bounds__(kCsThreads, TOK == 4 ? 2 : 1) cold_scatter_smem_kernel(const RunArgs a) {
    extern __shared__ float4 cs_smem[];
    // [RS][A]: row-major by query row, so a warp's 32 updates of one row
    // spread over all 32 banks (atom-major [A][RS] with RS = 4 would put them
    // on 8)
    uint32_t* refs = reinterpret_cast<uint32_t*>(cs_smem);            // [kCsMaxPages]
    float* ws = reinterpret_cast<float*>(cs_smem) + kCsRefBytes / 4;   // [RS][A]
    __shared__ float Ms[RS];
    __shared__ float red[kCsWarps][RS];
    const ColdChunk ch = a.cold_chunks[blockIdx.y];
    const uint32_t g = blockIdx.x, r0 = blockIdx.z * RS, b = ch.seq;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t A = a.A, RP = a.RP, Hkv = a.Hkv;
    const uint32_t i0 = a.cold_item_ptr[b], i1 = a.cold_item_ptr[b + 1];
    const ChunkSpan sp = chunk_span(a, ch);
    load_chunk_refs(refs, a, sp, false);  // (the score pass flagged a bad one)

    // Fixed-point table: integer shared-memory atomics are native (about 3x
    // the rate of the float ones), exact and order-independent.  Row r's
    // scale 2^F comes from the score pass's guess of the row's sum of |coeff
    // * p| terms (its exponential sum times its largest K coefficient sum);
    // the pass adds up the true sum S_r and the result is kept only if
    // 2^26 <= S_r * 2^F < 2^30: no int32 overflow even with every term's
    // rounding, and an average entry of A = 8192 atoms still spans 2^13
    // units, so its terms' roundings (half a unit each) stay near 1e-4 of it.
    // Otherwise — a guess far off, a non-finite score or coefficient — the
    // CTA zeroes the table and runs the pass again with fp32 atomics.
    __shared__ float Sc[RS];
    __shared__ uint32_t int_mode;
    if (warp == 0) {  // the sequence-wide maximum of rows r0 .. r0 + RS - 1
        bool fin = true;
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            float m = -INFINITY;
            for (uint32_t it = i0 + lane; it < i1; it += 32)
                m = fmaxf(m, __ldcg(&a.cmax[(static_cast<uint64_t>(it) * Hkv + g) * RP + r0 + r]));
            m = warp_max(m);
            float bnd = 0.0f;  // the guess, shifted to the sequence maximum
            for (uint32_t it = ch.item_begin + lane; it < ch.item_end; it += 32) {
                const uint64_t ci = (static_cast<uint64_t>(it) * Hkv + g) * RP + r0 + r;
                bnd += __ldcg(&a.cbound[ci]) * exp_shift(__ldcg(&a.cmax[ci]), m);
            }
            bnd = warp_sum(bnd);
            fin = fin && isfinite(bnd);
            int e = 0;
            if (bnd > 0.0f) frexpf(bnd, &e);
            const int F = min(126, max(-126, 29 - e));  // bnd * 2^F < 2^29
            if (lane == 0) {
                Ms[r] = m;
                Sc[r] = ldexpf(1.0f, F);
            }
        }
        if (lane == 0) int_mode = fin ? 1u : 0u;
    }
    float4* ws4 = reinterpret_cast<float4*>(ws);
    float M[RS], sc[RS], lsum[RS];
    bool use_int = false;
    for (int attempt = 0; attempt < 2; ++attempt) {
        for (uint32_t i = tid; i < A * RS / 4; i += kCsThreads) ws4[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if ((A * RS) % 4) {
            if (tid < (A * RS) % 4) ws[(A * RS / 4) * 4 + tid] = 0.0f;
        }
        __syncthreads();
        use_int = attempt == 0 && int_mode != 0;
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            M[r] = Ms[r];
            sc[r] = Sc[r];
            lsum[r] = 0.0f;
        }
        float tsum[RS];  // sum of |coeff * p| of this thread's terms (integer attempt)
#pragma unroll
        for (int r = 0; r < RS; ++r) tsum[r] = 0.0f;
        for (uint32_t x0 = 0; x0 < sp.ntok; x0 += kCsThreads * TOK) {
            uint4 code[TOK];
            float sv[TOK][RS];
            bool live[TOK];
#pragma unroll
            for (uint32_t u = 0; u < TOK; ++u) {
                const uint32_t x = x0 + tid + u * kCsThreads;
                live[u] = false;
                code[u] = make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int r = 0; r < RS; ++r) sv[u][r] = -INFINITY;
                if (x < sp.ntok) {
                    const uint32_t pi = x / kBlock, tt = x % kBlock;
                    const uint32_t phys = refs[pi];
                    if (phys != 0xFFFFFFFFu) {
                        live[u] = true;
                        code[u] = __ldg(&a.cold_v[(static_cast<uint64_t>(phys) * kBlock + tt) * Hkv + g]);
                        ldcg_rs<RS>(a.scores + (static_cast<uint64_t>(g) * a.cold_tokens + (sp.p0 + pi) * kBlock + tt) * RP + r0,
                                    sv[u]);
                    }
                }
            }
#pragma unroll
            for (uint32_t u = 0; u < TOK; ++u) {
                if (!live[u]) continue;
                float p[RS];
#pragma unroll
                for (int r = 0; r < RS; ++r) {
                    p[r] = exp_shift(sv[u][r], M[r]);
                    lsum[r] += p[r];
                }
                const uint16_t* idx = reinterpret_cast<const uint16_t*>(&code[u].x);
                const uint16_t* cf = reinterpret_cast<const uint16_t*>(&code[u].z);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (idx[k] >= A) {
                        atomicOr(a.status, DEVERR_ATOM_RANGE);
                        continue;
                    }
                    const float c = h2f(cf[k]);
                    float* dst = ws + idx[k];
                    if (use_int) {
#pragma unroll
                        for (int r = 0; r < RS; ++r) {
                            const float t = c * p[r];
                            tsum[r] += fabsf(t);
                            atomicAdd(reinterpret_cast<int*>(dst + r * A), __float2int_rn(t * sc[r]));
                        }
                    } else {
#pragma unroll
                        for (int r = 0; r < RS; ++r) atomicAdd(dst + r * A, c * p[r]);
                    }
                }
            }
        }
        if (!use_int) break;
        // keep the integer table only if every row's true sum fits the scale
#pragma unroll
        for (int r = 0; r < RS; ++r) {
            const float t = warp_sum(tsum[r]);
            if (lane == 0) red[warp][r] = t;
        }
        __syncthreads();
        if (tid == 0) {
            bool ok = true;
#pragma unroll
            for (int r = 0; r < RS; ++r) {
                float t = 0.0f;
                for (uint32_t w = 0; w < kCsWarps; ++w) t += red[w][r];
                const float scaled = t * sc[r];
                ok = ok && (t == 0.0f || (scaled >= 67108864.0f && scaled < 1073741824.0f));  // [2^26, 2^30)
            }
            int_mode = ok ? 2u : 0u;
        }
        __syncthreads();
        if (int_mode == 2u) break;  // (CTA-uniform) kept; else a second, fp32 pass
    }
#pragma unroll
    for (int r = 0; r < RS; ++r) {
        const float sm = warp_sum(lsum[r]);
        if (lane == 0) red[warp][r] = sm;
    }
    __syncthreads();  // the weight table and the partial sums are complete
    if (tid < RS) {
        float sm = 0.0f;
#pragma unroll
        for (uint32_t w = 0; w < kCsWarps; ++w) sm += red[w][tid];
        put_chunk_rows<RS>(a.csum, a, ch, g, r0, sm, 0.0f, tid);
    }
    // the table into w[b][g][atom][r0 .. r0 + RS - 1]
    float* wb = a.w + (static_cast<uint64_t>(b) * Hkv + g) * A * RP + r0;
    const bool whole = ch.item_begin == i0 && ch.item_end == i1;
    for (uint32_t atom = tid; atom < A; atom += kCsThreads) {
        float v[RS];
#pragma unroll
        for (int r = 0; r < RS; ++r)
            v[r] = use_int ? static_cast<float>(reinterpret_cast<const int*>(ws)[r * A + atom]) / sc[r] : ws[r * A + atom];
        float* dst = wb + static_cast<uint64_t>(atom) * RP;
        if (whole) {
            stcg_rs<RS>(dst, v);
        } else if constexpr (RS >= 4) {
#pragma unroll
            for (int r = 0; r < RS; r += 4) red_add_v4(dst + r, v[r], v[r + 1], v[r + 2], v[r + 3]);
        } else {
#pragma unroll
            for (int r = 0; r < RS; ++r) atomicAdd(dst + r, v[r]);
        }
    }
}

template <int RS, int TOK, bool kScatter>
cudaError_t launch_cs(const RunArgs& a, cudaStream_t s) {
    // both passes: RP / cold_slice_rows CTAs per (chunk, kv head)
    const size_t smem = kCsRefBytes + static_cast<size_t>(a.A) * RS * (kScatter ? sizeof(float) : sizeof(__half));
    // kv heads fastest in launch order: the CTAs of one chunk's heads run
    // together and share the 128-byte lines that hold a token's codes (and
    // scores), which are fetched from HBM once instead of once per head
    dim3 grid(a.Hkv, a.n_cold_chunks, a.RP / a.cold_slice_rows);
    cudaError_t e;
    if constexpr (kScatter) {
        e = cudaFuncSetAttribute(cold_scatter_smem_kernel<RS, TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        cold_scatter_smem_kernel<RS, TOK><<<grid, kCsThreads, smem, s>>>(a);
    } else {
        e = cudaFuncSetAttribute(cold_score_smem_kernel<RS, TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        cold_score_smem_kernel<RS, TOK><<<grid, kCsThreads, smem, s>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_cs_any(const RunArgs& a, cudaStream_t s, bool scatter) {
    if (!scatter) {
        // two CTAs per SM (4 tokens in flight each) when two f16 tables fit
        const bool two = 2 * (kCsRefBytes + static_cast<uint64_t>(a.A) * a.cold_score_rows * sizeof(__half) + 2048) <=
                         228ull * 1024;
        switch (a.cold_score_rows) {
            case 1: return launch_cs<1, 8, false>(a, s);
            case 2: return launch_cs<2, 8, false>(a, s);
            case 4: return two ? launch_cs<4, 4, false>(a, s) : launch_cs<4, 8, false>(a, s);
            case 8: return two ? launch_cs<8, 4, false>(a, s) : launch_cs<8, 8, false>(a, s);
            default: return cudaErrorInvalidValue;
        }
    }
    switch (a.cold_slice_rows) {
        case 1: return launch_cs<1, 8, true>(a, s);
        case 2: return launch_cs<2, 8, true>(a, s);
        case 4:
            if (cold_smem_ctas_per_sm(a.A, 4) >= 2) return launch_cs<4, 4, true>(a, s);
            return launch_cs<4, 8, true>(a, s);
        case 8: return launch_cs<8, 8, true>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

uint32_t cold_smem_slice_rows(uint32_t A, uint32_t RP) {
    if (RP > 16) return 0;  // 32+ rows: the row-lane L2 passes read each code once, coalesced
    uint32_t rs = RP < 8 ? RP : 8;
    while (rs > 1 && static_cast<uint64_t>(A) * rs * sizeof(float) > kCsTableMax) rs >>= 1;
    if (static_cast<uint64_t>(A) * rs * sizeof(float) > kCsTableMax) return 0;
    return rs;
}

uint32_t cold_smem_score_rows(uint32_t A, uint32_t RP, uint32_t rs) {
    // all the scatter slice's rows and up to 8 (one 16-byte gather), as many
    // as an f16 table of A atoms fits; a multiple of the scatter's slice
    uint32_t rss = RP < 8 ? RP : 8;
    while (rss > rs && static_cast<uint64_t>(A) * rss * sizeof(__half) > kCsTableMax) rss >>= 1;
    return rss < rs ? rs : rss;
}

uint32_t cold_smem_ctas_per_sm(uint32_t A, uint32_t rs) {
    const uint64_t bytes = kCsRefBytes + static_cast<uint64_t>(A) * rs * sizeof(float) + 1024 + 2 * kCsWarps * 8 * sizeof(float);
    uint64_t n = (228ull * 1024) / bytes;
    const uint64_t by_threads = 2048 / kCsThreads;
    if (n > by_threads) n = by_threads;
    return n ? static_cast<uint32_t>(n) : 1u;
}

bool cold_smem_enabled(const RunArgs& a) {
    const char* env = getenv("WEAVER_COLD_L2");  // 1: the L2 gather / reduction passes
    return a.cold_chunks && a.n_cold_chunks && a.n_cold_chunks <= 65535 && a.cold_slice_rows && a.cold_score_rows &&
           !(env && env[0] == '1');
}

cudaError_t launch_cold_score_smem(const RunArgs& a, cudaStream_t s) {
    if (a.n_cold_chunks == 0) return cudaSuccess;
    return launch_cs_any(a, s, false);
}

cudaError_t launch_cold_scatter_smem(const RunArgs& a, cudaStream_t s) {
    if (a.n_cold_chunks == 0) return cudaSuccess;
    return launch_cs_any(a, s, true);
}

}  // namespace weaver
