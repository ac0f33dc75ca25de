// weaver_headpart.cu — the decode step as one persistent kernel when one kv
// head's q_latent (A x RP f16) and per-atom weights (A x RP fp32) fit in a
// CTA's shared memory (RP <= 4, A * RP <= 16384: the 8B shape and smaller).
//
// Work split (one CTA per SM, cooperative launch so every CTA is resident):
//   * q_latent tiles: 128 atoms of one (sequence, kv head) each, spread
//     round-robin; scale * q . K_dict on tensor cores (mma.sync m16n8k16), the
//     result stored as f16 (the precision the reference's q_latent has).
//   * cold chunks: each CTA owns at most one run of <= 128 cold blocks of one
//     (sequence, kv head).  Its K and V codes (16 B per token) are copied in
//     at kernel start (cp.async) and stay in shared memory; the head's
//     q_latent is copied in once it is complete; scores overwrite the K codes
//     in place.  Once every chunk of the head has published its score maximum
//     M, the chunk adds coeff * exp(s - M) into the head's per-atom weights
//     with vector reductions at L2 (red.global.add.v4: one per (token, atom),
//     the four query rows packed), fire-and-forget.
//   * contraction tiles: 128 atoms of one (sequence, kv head), on tensor
//     cores: O += W . V_dict, V_dict tiles prefetched into L2 early and staged
//     by TMA.
//   * hot groups: exact split-KV attention over runs of hot blocks of one
//     (sequence, kv head), from a TMA ring of 8 or 16 blocks: 4 stages of
//     their own, the rest in the q_latent region once the chunk is scored
//     (and in the code buffers of a CTA without a chunk).
//   * merges: every hot group and contraction tile of a (sequence, kv head)
//     counts into one finish counter; the last one merges the head's hot
//     partials and its cold partial and writes the output rows.  Nobody waits
//     for a merge.
// Warp roles (11 warps): 0 dictionary producer, 1 hot producer, 2 code
// producer, 3-6 cold consumers, 7-10 hot consumers.
// Cross-CTA dependencies are counters per (sequence, kv head) (release: one
// thread's red.release / atom.acq_rel after the CTA barrier; acquire:
// ld.acquire polled by one thread).  The kernel is launched as a programmatic
// dependent: it waits for the previous kernel of the stream before touching
// memory, and the next step's CTAs take SMs as this step's leave them.  A CTA's cold work
// runs in phase order (q_latent tiles, chunk scores, chunk scatter,
// contraction tiles) and every wait is on an earlier phase, so with all CTAs
// resident no wait can deadlock.  Every wait is bounded (DEVERR_TIMEOUT).
#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr int kThreads = 352;
constexpr uint32_t kColdBar = 1, kHotBar = 2, kScoreBar = 3;
constexpr uint32_t kSmemBudget = 227 * 1024;                      // opt-in maximum per CTA
constexpr uint32_t kQlgBytes = 32768;                             // q_latent of one kv head (f16)
constexpr uint32_t kCodeBytes = kHpMaxChunkPages * kBlock * 16;   // 32 KB of codes per K / V
constexpr uint32_t kBulkPiece = 8192;
constexpr uint32_t kMergeScratch = 2 * (kHpMaxSlots + 1) * 4 + 12;  // floats per merging group
constexpr uint32_t kCtBatch = 4;                                    // contraction tiles per weight load
constexpr uint32_t kMaxHotStages = 16;

template <int D, int RP>
struct HpLayout {
    static constexpr uint32_t kBoxes = D / 64;
    static constexpr uint32_t kDictBox = kAtomTile * 128;        // 128 rows x 64 f16
    static constexpr uint32_t kDictSlot = kBoxes * kDictBox;
    static constexpr uint32_t kHotBox = kBlock * 128;            // 16 rows x 64 f16
    static constexpr uint32_t kHotPage = kBoxes * kHotBox;
    static constexpr uint32_t kHotStage = 2 * kHotPage;          // K then V
    static constexpr uint32_t dict = 0;                           // 2 slots: K_dict / V_dict tiles
    static constexpr uint32_t qlg = dict + 2 * kDictSlot;         // [A][RP] f16
    static constexpr uint32_t kbuf = qlg + kQlgBytes;             // K codes, then scores, then p
    static constexpr uint32_t vbuf = kbuf + kCodeBytes;           // V codes
    static constexpr uint32_t qb = vbuf + kCodeBytes;             // [2][8][D] f16 q for q_latent tiles
    static constexpr uint32_t qhb = qb + 2 * 8 * D * 2;           // [2][RP][D] f16 q of hot groups
    static constexpr uint32_t hcm = qhb + 2 * RP * D * 2;         // [4][RP]
    static constexpr uint32_t hcl = hcm + 4 * RP * 4;             // [4][RP]
    static constexpr uint32_t hco = hcl + 4 * RP * 4;             // [4][RP][D]
    static constexpr uint32_t cred = hco + 4 * RP * D * 4;        // [8][RP] score maxima
    static constexpr uint32_t ws = cred + 128 * 4;                // [kCtBatch][128][RP] contraction weights
    static constexpr uint32_t cphys = ws + kCtBatch * 128 * RP * 4;   // [128] chunk block refs
    static constexpr uint32_t misc = cphys + kHpMaxChunkPages * 4;    // 32 words, see below
    static constexpr uint32_t mscr = misc + 32 * 4;               // [2][kMergeScratch] merge scratch
    static constexpr uint32_t bars = mscr + 2 * kMergeScratch * 4;
    // full_d[2] empty_d[2] full_q[2] empty_q[2] kbar vbar qbar firstqt qfree full_h[16] empty_h[16]
    static constexpr uint32_t kFixedBars = 13;
    static constexpr uint32_t hot = (bars + (kFixedBars + 2 * kMaxHotStages) * 8 + 1023) / 1024 * 1024;
    static constexpr uint32_t kRoom = (kSmemBudget - 1024 - hot) / kHotStage;
    // hot ring stages: a multiple of the 4 consumer warps, so that block p
    // (consumed by warp p % 4) always reuses a stage its own warp emptied; a
    // parity wait can only tell apart phases one ring cycle apart
    static constexpr uint32_t kHS = (kRoom < kMaxHotStages ? kRoom : kMaxHotStages) / 4 * 4;
    static_assert(kHS >= 4, "hot ring needs at least one stage per consumer warp");
    static constexpr uint32_t total = hot + kHS * kHotStage;
    // The ring grows into the q_latent region (free once a chunk is scored) and,
    // in a CTA without a chunk, into the code buffers too: stages kHS.. live
    // there.  Counts stay multiples of 4.
    static constexpr uint32_t kExtQ = kQlgBytes / kHotStage;
    static constexpr uint32_t kExtAll = (kQlgBytes + 2 * kCodeBytes) / kHotStage;
    static constexpr uint32_t kStagesChunk = (kHS + kExtQ < kMaxHotStages ? kHS + kExtQ : kMaxHotStages) / 4 * 4;
    static constexpr uint32_t kStagesFree = (kHS + kExtAll < kMaxHotStages ? kHS + kExtAll : kMaxHotStages) / 4 * 4;
};
// misc words: [0, 4) invalid-page bits of the chunk, [4] cold-group
// broadcast, [5] hot-group broadcast, [8, 12) the head's cold score maximum,
// [16, 32) hot stage flags.

__device__ __forceinline__ void stamp(const HpArgs& ha, uint32_t slot) {
    if (ha.trace) ha.trace[blockIdx.x * kTraceSlots + slot] = globaltimer_ns();
}

__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t slots, uint32_t issued) {
    for (uint32_t s = 0; s < slots && s < issued; ++s) {
        const uint32_t last = s + ((issued - 1 - s) / slots) * slots;
        mbar_drain(&full[s], (last / slots) & 1);
    }
}

// Finishers of (b, g): its contraction tiles and its hot groups; the last one merges.
__device__ __forceinline__ uint32_t fin_target(const HpArgs& ha, uint32_t bg) {
    return (ha.n_chunks[bg] ? ha.r.n_atom_tiles : 0u) + ha.hot_groups[bg];
}

template <int RP>
__device__ __forceinline__ void load_rows(const float* p, float v[RP]) {
    if constexpr (RP == 4) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(p));
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (RP == 2) {
        const float2 x = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = x.x; v[1] = x.y;
    } else {
        v[0] = __ldcg(p);
    }
}

template <int RP>
__device__ __forceinline__ void load_rows_smem(const float* p, float v[RP]) {
    if constexpr (RP == 4) {
        const float4 x = *reinterpret_cast<const float4*>(p);
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (RP == 2) {
        const float2 x = *reinterpret_cast<const float2*>(p);
        v[0] = x.x; v[1] = x.y;
    } else {
        v[0] = *p;
    }
}

template <int RP>
__device__ __forceinline__ void store_rows(float* p, const float v[RP]) {
    if constexpr (RP == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    else if constexpr (RP == 2) *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    else *p = v[0];
}

template <int N>
__device__ __forceinline__ void load_cg(const float* p, float v[N]) {
    if constexpr (N == 4) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(p));
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (N == 2) {
        const float2 x = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = x.x; v[1] = x.y;
    } else {
        v[0] = __ldcg(p);
    }
}

// Cold scores of this CTA's chunk for the tokens t256, t256 + 256, ...:
// s[r] = sum_k coeff_k * q_latent[idx_k][r], written over the token's K code
// in place (blocks with an invalid reference get -inf); the running maximum
// per query row goes to mx.  Four tokens per thread in flight.
// Raw f16 q_latent rows of one atom (RP values) from shared memory, and
// their conversion: the gathers of a batch of tokens are all issued before
// any of them is used.
template <int RP>
__device__ __forceinline__ uint2 qlat_raw(const __half* q) {
    if constexpr (RP == 4) return *reinterpret_cast<const uint2*>(q);
    else if constexpr (RP == 2) return make_uint2(*reinterpret_cast<const uint32_t*>(q), 0u);
    else return make_uint2(*reinterpret_cast<const uint16_t*>(q), 0u);
}

template <int RP>
__device__ __forceinline__ void qlat_cvt(uint2 raw, float v[RP]) {
    if constexpr (RP == 4) {
        h4_to_f4(raw, v);
    } else if constexpr (RP == 2) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        v[0] = x.x; v[1] = x.y;
    } else {
        v[0] = h2f(static_cast<uint16_t>(raw.x));
    }
}

// Cold scores of tokens t256, t256 + 256, ... of the chunk: s[r] = sum_k
// coeff_k * q_latent[idx_k][r], written over the token's K code in kbuf; the
// running row maxima in mx.  Tokens of invalid pages score -inf; an atom
// index >= A raises DEVERR_ATOM_RANGE and its term is skipped.
template <int RP, int NBT = 1>
__device__ __forceinline__ void score_tokens(uint32_t t256, uint32_t ntok, uint32_t A, const uint32_t* cinv,
                                             uint8_t* kbuf, const __half* qlg, uint32_t* status, float mx[RP]) {
    for (uint32_t t0 = t256; t0 < ntok; t0 += 256 * NBT) {
        uint4 code[NBT];
        bool live[NBT];
#pragma unroll
        for (int u = 0; u < NBT; ++u) {
            const uint32_t tok = t0 + 256u * u, page = tok >> 4;
            live[u] = tok < ntok && !((cinv[(page >> 5) & 3] >> (page & 31)) & 1u);
            code[u] = live[u] ? *reinterpret_cast<const uint4*>(kbuf + tok * 16) : make_uint4(0, 0, 0, 0);
        }
        uint2 raw[NBT][4];
        bool bad = false;
#pragma unroll
        for (int u = 0; u < NBT; ++u)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t idx = ((k < 2 ? code[u].x : code[u].y) >> (16 * (k & 1))) & 0xFFFFu;
                bad |= idx >= A;
                raw[u][k] = qlat_raw<RP>(qlg + (idx < A ? idx : 0u) * RP);
            }
        if (bad) atomicOr(status, DEVERR_ATOM_RANGE);
#pragma unroll
        for (int u = 0; u < NBT; ++u) {
            float sc[RP];
#pragma unroll
            for (int r = 0; r < RP; ++r) sc[r] = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t idx = ((k < 2 ? code[u].x : code[u].y) >> (16 * (k & 1))) & 0xFFFFu;
                const float c = h2f(static_cast<uint16_t>((k < 2 ? code[u].z : code[u].w) >> (16 * (k & 1))));
                float qv[RP];
                qlat_cvt<RP>(raw[u][k], qv);
#pragma unroll
                for (int r = 0; r < RP; ++r) sc[r] = idx < A ? fmaf(c, qv[r], sc[r]) : sc[r];
            }
            const uint32_t tok = t0 + 256u * u;
            if (tok >= ntok) continue;
#pragma unroll
            for (int r = 0; r < RP; ++r) {
                sc[r] = live[u] ? sc[r] : -INFINITY;
                mx[r] = fmaxf(mx[r], sc[r]);
            }
            store_rows<RP>(reinterpret_cast<float*>(kbuf + tok * 16), sc);
        }
    }
}

// Split-KV across ranks, fused into the step: push this rank's (m, l, o)
// rows of (b, g) (row maxima fl, sums tot, the four warps' output sums in red)
// to every rank, then merge every rank's rows once their words carry this
// step's tag, and write the output.  A word is 8 bytes (value bits, tag),
// stored and loaded whole at system scope, so no fence or flag orders the
// data.  Rolled loops: it runs once per (sequence, kv head) per step and only
// on plans with an attached combiner.  Inline: an out-of-line call taking the
// kernel parameters by reference would move them all to local memory.
template <int D, int RP>
__device__ __forceinline__ void ll_merge(const HpArgs& ha, uint32_t ti, const float* fl, const float* tot,
                                      const uint32_t* rowx, const float* red) {
    const RunArgs& a = ha.r;
    constexpr uint32_t kOut = (RP * D + 127) / 128;
    const uint32_t W = ha.ll_world, tag = ld_relaxed_sys_u32(ha.ll_state) + 1u, par = tag & 1u;
    const uint64_t stride = D + 2;
#pragma unroll 1
    for (uint32_t k = 0; k < kOut; ++k) {
        const uint32_t idx = ti + 128 * k, r = idx / D, dim = idx % D;
        if (idx >= RP * D || r >= a.R) continue;
        const float O = (red[r * D + dim] + red[(RP + r) * D + dim]) + (red[(2 * RP + r) * D + dim] + red[(3 * RP + r) * D + dim]);
        const uint64_t off = ((static_cast<uint64_t>(par) * W + ha.ll_rank) * ha.ll_rows + rowx[r]) * stride;
#pragma unroll 1
        for (uint32_t p = 0; p < W; ++p) {
            uint2* dst = ha.ll_recv[p] + off;
            st_relaxed_sys_v2(dst + 2 + dim, __float_as_uint(O), tag);
            if (dim == 0) {
                st_relaxed_sys_v2(dst, __float_as_uint(fl[r]), tag);
                st_relaxed_sys_v2(dst + 1, __float_as_uint(tot[r]), tag);
            }
        }
    }
    const uint2* own = ha.ll_recv[ha.ll_rank];
#pragma unroll 1
    for (uint32_t k = 0; k < kOut; ++k) {
        const uint32_t idx = ti + 128 * k, r = idx / D, dim = idx % D;
        if (idx >= RP * D || r >= a.R) continue;
        float M = -INFINITY, L = 0.0f, O = 0.0f;  // online merge over the ranks
#pragma unroll 1
        for (uint32_t s = 0; s < W; ++s) {
            const uint2* src = own + ((static_cast<uint64_t>(par) * W + s) * ha.ll_rows + rowx[r]) * stride;
            uint2 wm, wl, wo;
            if (!ll_wait3(src, src + 1, src + 2 + dim, tag, wm, wl, wo, a.status)) continue;
            const float ms = __uint_as_float(wm.x), Mn = fmaxf(M, ms);
            const float fa = exp_shift(M, Mn), fb = exp_shift(ms, Mn);
            L = L * fa + __uint_as_float(wl.x) * fb;
            O = O * fa + __uint_as_float(wo.x) * fb;
            M = Mn;
        }
        a.out[static_cast<uint64_t>(rowx[r]) * D + dim] = __float2half_rn(L > 0.0f ? O / L : 0.0f);
    }
}

// Merge every hot slot of (b, g) with its cold partial and write the rows (out
// or the (m, l, o) partial outputs).  Run by one 128-thread group (named
// barrier `bar`) with `st` shared scratch of kMergeScratch floats and `red`
// of 4 x RP x D floats.  The caller passes the pair's hot slots [s0, s0 + ns)
// and whether it has a cold partial, read long before (plan tables are cold in
// L2 at this point).  What other CTAs published before their counter
// increments is read in one L2 round trip: the first 16 slots' outputs (split
// over the four warps, each lane D/32 dimensions) and the cold partial into
// registers, the slot statistics into shared memory.  Then per-row factors,
// the weighted sums and the four warps' sums added in shared memory.
template <int D, int RP>
__device__ void final_merge(const HpArgs& ha, uint32_t bg, uint32_t s0, uint32_t ns, bool cold, uint32_t ti,
                            uint32_t bar, float* st, float* red) {
    constexpr int VPL = D / 32;
    const RunArgs& a = ha.r;
    const uint32_t w = ti >> 5, lane = ti & 31, d0 = lane * VPL;
    float* fm = st;                                             // [ns + 1][RP]: m, then the partial's factor
    float* fl = st + (kHpMaxSlots + 1) * RP;                    // [ns + 1][RP]: l; fl[0..RP) then the row maxima
    float* tot = fl + (kHpMaxSlots + 1) * RP;                   // [RP] merged l, [RP] its reciprocal
    uint32_t* rowx = reinterpret_cast<uint32_t*>(tot + 2 * RP);  // [RP] output row of each query row
    float v[4][RP][VPL];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t j = w + 4 * q;
#pragma unroll
        for (int r = 0; r < RP; ++r) {
            if (j < ns) {
                load_cg<VPL>(ha.so + (static_cast<uint64_t>(s0 + j) * RP + r) * D + d0, v[q][r]);
            } else {
#pragma unroll
                for (int e = 0; e < VPL; ++e) v[q][r][e] = 0.0f;
            }
        }
    }
    float vc[RP][VPL];
#pragma unroll
    for (int r = 0; r < RP; ++r) {
        if (w == 0 && cold) {
            load_cg<VPL>(ha.ocold + (static_cast<uint64_t>(bg) * RP + r) * D + d0, vc[r]);
        } else {
#pragma unroll
            for (int e = 0; e < VPL; ++e) vc[r][e] = 0.0f;
        }
    }
    for (uint32_t t = ti; t < ns * RP; t += 128) {
        fm[t] = __ldcg(&ha.sm[s0 * RP + t]);
        fl[t] = __ldcg(&ha.sl[s0 * RP + t]);
    }
    if (ti < static_cast<uint32_t>(RP)) {
        fm[ns * RP + ti] = cold ? unkey(__ldcg(&ha.mkey[bg * RP + ti])) : -INFINITY;
        fl[ns * RP + ti] = cold ? __ldcg(&ha.wsum[static_cast<uint64_t>(bg) * (a.A * RP + 4) + a.A * RP + ti]) : 0.0f;
    }
    named_bar(bar, 128);
    if (w < static_cast<uint32_t>(RP)) {
        // warp r: row r's maximum, every partial's factor, the merged l
        const uint32_t r = w;
        float M = -INFINITY;
        for (uint32_t j = lane; j <= ns; j += 32) M = fmaxf(M, fm[j * RP + r]);
        M = warp_max(M);
        float L = 0.0f;
        for (uint32_t j = lane; j <= ns; j += 32) {
            const float f = exp_shift(fm[j * RP + r], M);
            L += fl[j * RP + r] * f;
            fm[j * RP + r] = f;
        }
        L = warp_sum(L);
        __syncwarp();
        if (lane == 0) {
            tot[r] = L;
            tot[RP + r] = L > 0.0f ? 1.0f / L : 0.0f;
            fl[r] = M;  // row maximum (fl[0..RP) is no longer needed)
            const uint32_t b = bg / a.Hkv, g = bg % a.Hkv;
            rowx[r] = (b * a.nq + r / a.G) * a.Hq + g * a.G + r % a.G;
        }
    }
    named_bar(bar, 128);
    {
        float acc[RP][VPL];
#pragma unroll
        for (int r = 0; r < RP; ++r) {
            const float f = fm[ns * RP + r];
#pragma unroll
            for (int e = 0; e < VPL; ++e) acc[r][e] = (w == 0 && cold) ? f * vc[r][e] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t j = w + 4 * q;
            if (j < ns) {
#pragma unroll
                for (int r = 0; r < RP; ++r) {
                    const float f = fm[j * RP + r];
#pragma unroll
                    for (int e = 0; e < VPL; ++e) acc[r][e] = fmaf(f, v[q][r][e], acc[r][e]);
                }
            }
        }
        for (uint32_t j0 = w + 16; j0 < ns; j0 += 16) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t j = j0 + 4 * q;
#pragma unroll
                for (int r = 0; r < RP; ++r) {
                    if (j < ns) {
                        load_cg<VPL>(ha.so + (static_cast<uint64_t>(s0 + j) * RP + r) * D + d0, v[q][r]);
                    } else {
#pragma unroll
                        for (int e = 0; e < VPL; ++e) v[q][r][e] = 0.0f;
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t j = j0 + 4 * q;
                if (j >= ns) break;
#pragma unroll
                for (int r = 0; r < RP; ++r) {
                    const float f = fm[j * RP + r];
#pragma unroll
                    for (int e = 0; e < VPL; ++e) acc[r][e] = fmaf(f, v[q][r][e], acc[r][e]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RP; ++r)
#pragma unroll
            for (int e = 0; e < VPL; ++e) red[(w * RP + r) * D + d0 + e] = acc[r][e];
    }
    named_bar(bar, 128);
    if (ha.ll_world) {  // merged over the ranks inside this step
        ll_merge<D, RP>(ha, ti, fl, tot, rowx, red);
        named_bar(bar, 128);  // scratch reusable
        return;
    }
    constexpr uint32_t kOut = (RP * D + 127) / 128;  // outputs per thread
#pragma unroll
    for (uint32_t k = 0; k < kOut; ++k) {
        const uint32_t idx = ti + 128 * k, r = idx / D, dim = idx % D;
        if (idx < RP * D && r < a.R) {
            const float O = (red[r * D + dim] + red[(RP + r) * D + dim]) + (red[(2 * RP + r) * D + dim] + red[(3 * RP + r) * D + dim]);
            const uint64_t row = rowx[r];
            if (a.flags & 4u) {  // WEAVER_FLAG_PARTIALS
                if (dim == 0) {
                    a.part_m[row] = fl[r];
                    a.part_l[row] = tot[r];
                }
                a.part_o[row * D + dim] = O;
            } else {
                a.out[row * D + dim] = __float2half_rn(O * tot[RP + r]);
            }
        }
    }
    named_bar(bar, 128);  // scratch reusable
}

}  // namespace

template <int D, int RP>
__global__ void __launch_bounds__(kThreads, 1)
    hp_step_kernel(const __grid_constant__ CUtensorMap tm_hk, const __grid_constant__ CUtensorMap tm_hv,
                   const __grid_constant__ CUtensorMap tm_kd, const __grid_constant__ CUtensorMap tm_vd,
                   const __grid_constant__ CUtensorMap tm_kc, const __grid_constant__ CUtensorMap tm_vc,
                   const HpArgs ha) {
    using L = HpLayout<D, RP>;
    constexpr uint32_t kHS = L::kHS;
    const RunArgs& a = ha.r;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* dict = smem + L::dict;
    __half* qlg = reinterpret_cast<__half*>(smem + L::qlg);
    uint8_t* kbuf = smem + L::kbuf;
    uint8_t* vbuf = smem + L::vbuf;
    __half* qb = reinterpret_cast<__half*>(smem + L::qb);
    __half* qhb = reinterpret_cast<__half*>(smem + L::qhb);
    float* hcm = reinterpret_cast<float*>(smem + L::hcm);
    float* hcl = reinterpret_cast<float*>(smem + L::hcl);
    float* hco = reinterpret_cast<float*>(smem + L::hco);
    float* cred = reinterpret_cast<float*>(smem + L::cred);
    float* ws = reinterpret_cast<float*>(smem + L::ws);
    uint32_t* cphys = reinterpret_cast<uint32_t*>(smem + L::cphys);
    uint32_t* misc = reinterpret_cast<uint32_t*>(smem + L::misc);
    uint32_t* cinv = misc;
    uint32_t* hflags = misc + 16;
    volatile uint32_t* cflag = misc + 4;
    volatile uint32_t* hflag = misc + 5;
    float* cscr = reinterpret_cast<float*>(misc + 8);
    float* cmrg = reinterpret_cast<float*>(smem + L::mscr);
    float* hmrg = cmrg + kMergeScratch;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bars);
    uint64_t* full_d = bars;
    uint64_t* empty_d = full_d + 2;
    uint64_t* full_q = empty_d + 2;
    uint64_t* empty_q = full_q + 2;
    uint64_t* kbar = empty_q + 2;
    uint64_t* vbar = kbar + 1;
    uint64_t* qbar = vbar + 1;
    uint64_t* firstqt = qbar + 1;
    uint64_t* qfree = firstqt + 1;
    uint64_t* full_h = qfree + 1;
    uint64_t* empty_h = full_h + kMaxHotStages;

    // launched as a programmatic dependent: wait until the previous kernel in
    // the stream has completed (its writes visible), and let the next one be
    // placed on SMs as soon as this step's CTAs leave them
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t cta = blockIdx.x;
    const uint32_t Hkv = a.Hkv, A = a.A, R = a.R, G = a.G, nq = a.nq, Hq = a.Hq;
    const uint32_t NB = a.B * Hkv;
    const uint32_t wstride = A * RP + 4;
    uint32_t* cnt = ha.counters;
    const uint32_t i0 = ha.item_ptr[cta], i1 = ha.item_ptr[cta + 1];
    const uint32_t g0 = ha.group_ptr[cta], g1 = ha.group_ptr[cta + 1];
    const HpChunk ch = ha.chunks[cta];
    // hot ring of this CTA: kHS stages in the hot region, then stages in the
    // q_latent region (and the code buffers when the CTA has no chunk)
    const uint32_t nst = ch.n_pages ? L::kStagesChunk : L::kStagesFree;
    // hot ring stage s: kHS stages in the hot region, the rest from the q_latent region on
#define HSTAGE(s) (smem + ((s) < kHS ? L::hot + (s) * L::kHotStage : L::qlg + ((s) - kHS) * L::kHotStage))
    const bool has_qt = i1 > i0 && ha.items[i0].type == FI_QLAT;

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) { mbar_init(&full_d[i], 1); mbar_init(&empty_d[i], 1); }
        for (uint32_t i = 0; i < kMaxHotStages; ++i) { mbar_init(&full_h[i], 1); mbar_init(&empty_h[i], 1); }
        mbar_init(qfree, 1);
        for (int i = 0; i < 2; ++i) { mbar_init(&full_q[i], 1); mbar_init(&empty_q[i], 1); }
        mbar_init(kbar, 33);  // 32 cp.async arrivals + the invalid-page bits
        mbar_init(vbar, 32);
        mbar_init(qbar, 1);
        mbar_init(firstqt, 1);
        fence_barrier_init();
        if (ha.trace)
            for (uint32_t i = 0; i < kTraceSlots; ++i) ha.trace[cta * kTraceSlots + i] = 0;
        stamp(ha, TR_START);
    }
    // query rows R..7 of the q_latent tiles' B operand are zero
    for (uint32_t i = tid; i < 2 * 8 * D; i += kThreads)
        if ((i / D) % 8 >= R) qb[i] = __float2half_rn(0.0f);
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            // ---- dictionary producer: K_dict tiles (+ query rows), then V_dict tiles
            if (i1 > i0) {
                prefetch_tensormap(&tm_kd);
                prefetch_tensormap(&tm_vd);
            }
            uint32_t k = 0;
            bool prefetched = false;
            // the first q_latent tile goes out one load after kernel start
            const FusedItem f0 = ha.first_item[cta];
            if (f0.type == FI_QLAT) {
                mbar_arrive_expect_tx(&full_d[0], L::kDictSlot + nq * G * D * 2);
                const int32_t y = static_cast<int32_t>(f0.g * a.dict_row_stride + f0.a * kAtomTile);
#pragma unroll
                for (uint32_t bx = 0; bx < L::kBoxes; ++bx)
                    tma_load_2d(dict + bx * L::kDictBox, &tm_kd, &full_d[0], bx * 64, y);
                for (uint32_t j = 0; j < nq; ++j)
                    bulk_load(qb + (j * G) * D, a.q + ((static_cast<uint64_t>(f0.b) * nq + j) * Hq + f0.g * G) * D,
                              G * D * 2, &full_d[0]);
                k = 1;
            }
            for (uint32_t i = i0 + k; i < i1; ++i) {
                const FusedItem it = ha.items[i];
                const uint32_t s = k & 1u;
                const bool qt = it.type == FI_QLAT;
                if (!qt && !prefetched) {
                    // V_dict tiles of the contraction: into L2 now, into shared memory later
                    prefetched = true;
                    if (ch.n_pages) mbar_wait(vbar, 0, a.status, 1);
                    else if (has_qt) mbar_wait(firstqt, 0, a.status, 20);
                    for (uint32_t j = i; j < i1; ++j) {
                        const FusedItem cj = ha.items[j];
                        const uint32_t rows = min(kAtomTile, A - cj.a * kAtomTile);
                        bulk_prefetch_l2(a.v_dict + (cj.g * a.dict_row_stride + cj.a * kAtomTile) * D, rows * D * 2);
                    }
                }
                if (k >= 2 && !mbar_wait(&empty_d[s], ((k >> 1) - 1) & 1, a.status, 2)) break;
                const uint32_t qbytes = qt ? nq * G * D * 2 : 0;
                mbar_arrive_expect_tx(&full_d[s], L::kDictSlot + qbytes);
                const int32_t y = static_cast<int32_t>(it.g * a.dict_row_stride + it.a * kAtomTile);
#pragma unroll
                for (uint32_t bx = 0; bx < L::kBoxes; ++bx)
                    tma_load_2d(dict + s * L::kDictSlot + bx * L::kDictBox, qt ? &tm_kd : &tm_vd, &full_d[s],
                                bx * 64, y);
                if (qt)
                    for (uint32_t j = 0; j < nq; ++j)
                        bulk_load(qb + (s * 8 + j * G) * D, a.q + ((static_cast<uint64_t>(it.b) * nq + j) * Hq + it.g * G) * D,
                                  G * D * 2, &full_d[s]);
                ++k;
            }
            drain_ring(full_d, 2, k);
        }
    } else if (warp == 1) {
        // ---- hot producer: K/V blocks of this CTA's hot groups, each group's
        // query rows.  The whole warp walks the blocks, its lanes fetching 32
        // block references at a time; lane 0 issues the copies.
        if (g1 > g0) {
            if (lane == 0) {
                prefetch_tensormap(&tm_hk);
                prefetch_tensormap(&tm_hv);
            }
            // the q_latent tiles and the chunk's K codes head the cold critical
            // path: let them land first (the ring then keeps up to nst blocks
            // in flight, enough to stream the rest from HBM)
            if (ch.n_pages) {
                mbar_wait(kbar, 0, a.status, 3);
            } else if (has_qt) {
                mbar_wait(firstqt, 0, a.status, 19);
            }
            __syncwarp();
        }
        uint32_t k = 0, n = 0;
        bool stop = false;
        for (uint32_t gi = g0; gi < g1 && !stop; ++gi, ++n) {
            const FusedHotGroup gr = ha.groups[gi];
            const uint32_t qs = n & 1u;
            if (n >= 2 && !__all_sync(0xffffffffu, mbar_wait(&empty_q[qs], ((n >> 1) - 1) & 1, a.status, 4))) break;
            if (lane == 0) {
                mbar_arrive_expect_tx(&full_q[qs], nq * G * D * 2);
                for (uint32_t j = 0; j < nq; ++j)
                    bulk_load(qhb + (qs * RP + j * G) * D,
                              a.q + ((static_cast<uint64_t>(gr.b) * nq + j) * Hq + gr.g * G) * D, G * D * 2, &full_q[qs]);
            }
            for (uint32_t p0 = gr.page_begin; p0 < gr.page_end && !stop; p0 += 32) {
                const uint32_t phys_l = p0 + lane < gr.page_end ? a.hot_refs[p0 + lane] & kRefMask : 0u;
                const uint32_t nb = min(32u, gr.page_end - p0);
                for (uint32_t j = 0; j < nb; ++j) {
                    const uint32_t phys = __shfl_sync(0xffffffffu, phys_l, j);
                    const uint32_t s = k % nst;
                    if (k >= nst && !__all_sync(0xffffffffu, mbar_wait(&empty_h[s], ((k / nst) - 1) & 1, a.status, 5))) {
                        stop = true;
                        break;
                    }
                    // the first stage past the hot region: the chunk's q_latent must be dead
                    if (k == kHS && nst > kHS && ch.n_pages && !__all_sync(0xffffffffu, mbar_wait(qfree, 0, a.status, 22))) {
                        stop = true;
                        break;
                    }
                    if (lane == 0) {
                        const bool valid = phys < a.hot_pool_blocks;
                        if (!valid) atomicOr(a.status, DEVERR_REF_RANGE);
                        hflags[s] = valid ? 1u : 0u;
                        mbar_arrive_expect_tx(&full_h[s], valid ? L::kHotStage : 0u);
                        if (valid) {
                            uint8_t* dst = HSTAGE(s);
#pragma unroll
                            for (uint32_t bx = 0; bx < L::kBoxes; ++bx) {
                                const int32_t x = static_cast<int32_t>(gr.g * D + bx * 64);
                                const int32_t y = static_cast<int32_t>(phys * kBlock);
                                tma_load_2d(dst + bx * L::kHotBox, &tm_hk, &full_h[s], x, y);
                                tma_load_2d(dst + L::kHotPage + bx * L::kHotBox, &tm_hv, &full_h[s], x, y);
                            }
                        }
                    }
                    ++k;
                }
            }
        }
        if (lane == 0) {
            drain_ring(full_h, nst, k);
            drain_ring(full_q, 2, n);
        }
    } else if (warp == 2) {
        if (ch.n_pages) {
            // ---- code producer (whole warp): this CTA's chunk of K codes, then
            // V codes, one 16-byte cp.async per token, tracked by kbar / vbar
            uint32_t bad[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t p = q * 32 + lane;
                uint32_t phys = 0;
                bool invalid = false;
                if (p < ch.n_pages) {
                    phys = a.cold_refs[ch.page_begin + p] & kRefMask;
                    invalid = phys >= a.cold_pool_blocks;
                    if (invalid) atomicOr(a.status, DEVERR_REF_RANGE);
                    cphys[p] = phys;
                }
                bad[q] = __ballot_sync(0xffffffffu, invalid);
            }
            if (lane == 0) {
#pragma unroll
                for (int q = 0; q < 4; ++q) cinv[q] = bad[q];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(kbar);  // publishes cinv and cphys
            const uint32_t ntok = ch.n_pages * kBlock;
            for (int pass = 0; pass < 2; ++pass) {
                const uint4* pool = pass ? a.cold_v : a.cold_k;
                uint8_t* dst = pass ? vbuf : kbuf;
                // V codes are first needed at the scatter: issue them once the K
                // codes have landed, off the q_latent tiles' and K codes' way
                if (pass) mbar_wait(kbar, 0, a.status, 23);
                for (uint32_t tok = lane; tok < ntok; tok += 32) {
                    const uint32_t page = tok >> 4;
                    if ((bad[page >> 5] >> (page & 31)) & 1u) continue;
                    cp_async16(dst + tok * 16,
                               pool + (static_cast<uint64_t>(cphys[page]) * kBlock + (tok & 15)) * Hkv + ch.g);
                }
                cp_async_arrive_noinc(pass ? vbar : kbar);
            }
            cp_async_wait_all();
        }
    } else if (warp < 7) {
        // =================== cold consumers (128 threads) ===================
        const uint32_t ct = tid - 96, cw = ct >> 5;
        const bool leader = ct == 0;
        uint32_t kd = 0;
        uint32_t i = i0;
        uint32_t merge_bg = ~0u, merge_s0 = 0, merge_ns = 0;  // a merge this group owes (see the end)
        bool merge_cold = false;

        // ---- q_latent tiles: qlat16[bg][atom][r] = scale * q_r . K_dict[g][atom]
        for (; i < i1 && ha.items[i].type == FI_QLAT; ++i, ++kd) {
            const FusedItem it = ha.items[i];
            const uint32_t bg = it.b * Hkv + it.g, t = it.a, s = kd & 1u;
            // warp-uniform and converged: ldmatrix / mma below are .sync.aligned
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&full_d[s], (kd >> 1) & 1, a.status, 6));
            if (leader) stamp(ha, TR_QT_LAST_LANDED);
            if (kd == 0 && leader) {
                mbar_arrive(firstqt);
                stamp(ha, TR_QT_LANDED);
            }
            if (ok) {
                const uint8_t* tile = dict + s * L::kDictSlot;
                const __half* qs = qb + s * 8 * D;
                const uint32_t gid = lane >> 2, tig = lane & 3;
                float c[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) c[mt][e] = 0.0f;
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(qs + gid * D + ks * 16 + 2 * tig);
                    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(qs + gid * D + ks * 16 + 8 + 2 * tig);
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt) {
                        const uint32_t row = cw * 32 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                        const uint32_t kc = ks * 2 + (lane >> 4);
                        uint32_t af[4];
                        ldmatrix_x4(af, tile + (kc >> 3) * L::kDictBox + swz128(row, kc & 7));
                        mma_16816(c[mt], af, b0, b1);
                    }
                }
                __half* ql = ha.qlat16 + static_cast<uint64_t>(bg) * A * RP;
                if (2 * tig < RP) {
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                        for (int hi = 0; hi < 2; ++hi) {
                            const uint32_t atom = t * kAtomTile + cw * 32 + mt * 16 + gid + hi * 8;
                            if (atom >= A) continue;
                            const float v0 = c[mt][hi * 2] * a.scale, v1 = c[mt][hi * 2 + 1] * a.scale;
                            if constexpr (RP >= 2) {
                                const __half2 h = __floats2half2_rn(v0, v1);
                                __stcg(reinterpret_cast<unsigned int*>(ql + atom * RP + 2 * tig),
                                       *reinterpret_cast<const unsigned int*>(&h));
                            } else {
                                ql[atom] = __float2half_rn(v0);
                            }
                        }
                }
            }
            // zero this tile's per-atom weights; the head's first tile also resets
            // its cold output, l and score maximum
            {
                const uint32_t atom = t * kAtomTile + ct;
                if (atom < A) {
                    float z[RP];
#pragma unroll
                    for (int r = 0; r < RP; ++r) z[r] = 0.0f;
                    store_rows<RP>(ha.wsum + static_cast<uint64_t>(bg) * wstride + atom * RP, z);
                }
                if (t == 0) {
                    float* oc = ha.ocold + static_cast<uint64_t>(bg) * RP * D;
                    for (uint32_t x = ct; x < RP * D; x += 128) oc[x] = 0.0f;
                    if (ct < 4) ha.wsum[static_cast<uint64_t>(bg) * wstride + A * RP + ct] = 0.0f;
                    if (ct < RP) ha.mkey[bg * RP + ct] = fkey(-INFINITY);
                }
            }
            named_bar(kColdBar, 128);
            if (leader) {
                mbar_arrive(&empty_d[s]);
                red_release_gpu(&cnt[HC_QLAT * NB + bg], 1u);
            }
        }
        if (leader && kd) stamp(ha, TR_QLAT_DONE);

        // ---- this CTA's cold chunk: scores, then the scatter of p * coeff into
        // the head's per-atom weights (red.global.add at L2, relative to the
        // head's score maximum once every chunk of the head has published its own)
        if (ch.n_pages) {
            const uint32_t bg = ch.b * Hkv + ch.g;
            const uint32_t ntok = ch.n_pages * kBlock;
            if (leader) {
                spin_until(&cnt[HC_QLAT * NB + bg], a.n_atom_tiles, a.status, 7);
                stamp(ha, TR_SCORE_WAIT);
                fence_proxy_async_global();
                const uint32_t bytes = A * RP * 2;
                const uint8_t* src = reinterpret_cast<const uint8_t*>(ha.qlat16 + static_cast<uint64_t>(bg) * A * RP);
                mbar_arrive_expect_tx(qbar, bytes);
                for (uint32_t off = 0; off < bytes; off += kBulkPiece)
                    bulk_load(reinterpret_cast<uint8_t*>(qlg) + off, src + off, min(kBulkPiece, bytes - off), qbar);
            }
            const bool okk = mbar_wait(kbar, 0, a.status, 8);
            if (leader) stamp(ha, TR_CODES_LANDED);
            const bool okq = mbar_wait(qbar, 0, a.status, 9);
            if (leader) stamp(ha, TR_QLAT_LANDED);
            const uint32_t inv0 = cinv[0], inv1 = cinv[1], inv2 = cinv[2], inv3 = cinv[3];
#define PAGE_OK(tok) (!(((((tok) >> 4) < 32 ? inv0 : ((tok) >> 4) < 64 ? inv1 : ((tok) >> 4) < 96 ? inv2 : inv3) >> (((tok) >> 4) & 31)) & 1u))
            // scores: this group takes tokens ct, ct + 256, ...; the hot warps the others
            float mx[RP];
#pragma unroll
            for (int r = 0; r < RP; ++r) mx[r] = -INFINITY;
            if (okk && okq) score_tokens<RP>(ct, ntok, A, cinv, kbuf, qlg, a.status, mx);
#pragma unroll
            for (int r = 0; r < RP; ++r) {
                const float m = warp_max(mx[r]);
                if (lane == 0) cred[cw * RP + r] = m;
            }
            named_bar(kScoreBar, 256);  // both groups' scores written
            if (leader) mbar_arrive(qfree);  // q_latent is dead: the hot ring may use its region
            if (leader) {
#pragma unroll
                for (int r = 0; r < RP; ++r) {
                    float m = -INFINITY;
#pragma unroll
                    for (int w2 = 0; w2 < 8; ++w2) m = fmaxf(m, cred[w2 * RP + r]);
                    atomicMax(&ha.mkey[bg * RP + r], fkey(m));
                }
                red_release_gpu(&cnt[HC_SCORE * NB + bg], 1u);
                stamp(ha, TR_SCORED);
                spin_until(&cnt[HC_SCORE * NB + bg], ha.n_chunks[bg], a.status, 10);
#pragma unroll
                for (int r = 0; r < RP; ++r) cscr[r] = unkey(__ldcg(&ha.mkey[bg * RP + r]));
                stamp(ha, TR_SCATTER_WAIT);
            }
            const bool okv = mbar_wait(vbar, 0, a.status, 11) && okk && okq;
            named_bar(kColdBar, 128);
            float M[RP];
#pragma unroll
            for (int r = 0; r < RP; ++r) M[r] = cscr[r];
            float ls[RP];
#pragma unroll
            for (int r = 0; r < RP; ++r) ls[r] = 0.0f;
            float* wh = ha.wsum + static_cast<uint64_t>(bg) * wstride;
            if (okv) {
                for (uint32_t t0 = ct; t0 < ntok; t0 += 256) {
                    uint4 code[2];
                    float pr[2][RP];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t tok = t0 + 128u * u;
                        const bool live = tok < ntok && PAGE_OK(tok);
                        code[u] = live ? *reinterpret_cast<const uint4*>(vbuf + tok * 16) : make_uint4(0, 0, 0, 0);
                        float sv[RP];
                        if (live) {
                            load_rows_smem<RP>(reinterpret_cast<const float*>(kbuf + tok * 16), sv);
                        } else {
#pragma unroll
                            for (int r = 0; r < RP; ++r) sv[r] = -INFINITY;
                        }
#pragma unroll
                        for (int r = 0; r < RP; ++r) {
                            pr[u][r] = exp_shift(sv[r], M[r]);
                            ls[r] += pr[u][r];
                        }
                    }
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint32_t iw[2] = {code[u].x, code[u].y};
                        const uint32_t cw2[2] = {code[u].z, code[u].w};
                        const uint32_t tok = t0 + 128u * u;
                        if (tok >= ntok || !PAGE_OK(tok)) continue;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint32_t idx = (iw[k >> 1] >> (16 * (k & 1))) & 0xFFFFu;
                            if (idx >= A) {
                                atomicOr(a.status, DEVERR_ATOM_RANGE);
                                continue;
                            }
                            const float c = h2f(static_cast<uint16_t>(cw2[k >> 1] >> (16 * (k & 1))));
                            float* dst = wh + idx * RP;
                            if constexpr (RP == 4) {
                                red_add_v4(dst, c * pr[u][0], c * pr[u][1], c * pr[u][2], c * pr[u][3]);
                            } else if constexpr (RP == 2) {
                                red_add_v2(dst, c * pr[u][0], c * pr[u][1]);
                            } else {
                                atomicAdd(dst, c * pr[u][0]);
                            }
                        }
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < RP; ++r) {
                const float l = warp_sum(ls[r]);
                if (lane == 0) atomicAdd(&wh[A * RP + r], l);
            }
            named_bar(kColdBar, 128);  // every thread's reductions precede the release below
            if (leader) {
                red_release_gpu(&cnt[HC_SCATTER * NB + bg], 1u);
                stamp(ha, TR_SCATTER_DONE);
            }
        }

#undef PAGE_OK
        // ---- contraction tiles: ocold[bg][r] += sum_atom w[atom][r] * V_dict[g][atom]
        // on tensor cores: O (rows x D) += W (rows x 128 atoms) . V (128 atoms x D);
        // warp cw takes atoms cw*32 .. cw*32+31.  The planner gives a CTA only
        // tiles of its own chunk's head: one wait, the weights of up to kCtBatch
        // tiles loaded together, one reduction into ocold, one finish count.
        if (i < i1) {
            const FusedItem it0 = ha.items[i];
            const uint32_t bg = it0.b * Hkv + it0.g;
            const uint32_t n_ct = i1 - i;
            // the pair's merge inputs and finisher count, read now, used after the tiles
            const uint32_t ms0 = ha.slot_ptr[bg], mns = ha.slot_ptr[bg + 1] - ms0, mfin = fin_target(ha, bg);
            if (leader) {
                spin_until(&cnt[HC_SCATTER * NB + bg], ha.n_chunks[bg], a.status, 12);
                stamp(ha, TR_CONTRACT_WAIT);
            }
            named_bar(kColdBar, 128);
            constexpr int NT = D / 8;
            float o[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
            const uint32_t gid = lane >> 2, tig = lane & 3;
            const float* wh = ha.wsum + static_cast<uint64_t>(bg) * wstride;
            for (uint32_t c0 = 0; c0 < n_ct; c0 += kCtBatch) {
                const uint32_t nb = min(kCtBatch, n_ct - c0);
                for (uint32_t u = 0; u < nb; ++u) {
                    const uint32_t atom = ha.items[i + c0 + u].a * kAtomTile + ct;
                    float v[RP];
                    if (atom < A) {
                        load_rows<RP>(wh + atom * RP, v);
                    } else {
#pragma unroll
                        for (int r = 0; r < RP; ++r) v[r] = 0.0f;
                    }
                    store_rows<RP>(ws + (u * 128 + ct) * RP, v);
                }
                named_bar(kColdBar, 128);
                if (leader && c0 == 0) stamp(ha, TR_WS_READY);
                for (uint32_t u = 0; u < nb; ++u, ++kd) {
                    const uint32_t s = kd & 1u;
                    const bool ok = __all_sync(0xffffffffu, mbar_wait(&full_d[s], (kd >> 1) & 1, a.status, 13));
                    if (ok) {
                        const uint8_t* tile = dict + s * L::kDictSlot;
                        const float* wt = ws + u * 128 * RP;
#pragma unroll
                        for (int ks = 0; ks < 2; ++ks) {
                            const uint32_t k0 = cw * 32 + ks * 16;
                            uint32_t wa0 = 0u, wa2 = 0u;
                            if (gid < static_cast<uint32_t>(RP)) {
                                const __half2 x0 = __floats2half2_rn(wt[(k0 + 2 * tig) * RP + gid], wt[(k0 + 2 * tig + 1) * RP + gid]);
                                const __half2 x2 =
                                    __floats2half2_rn(wt[(k0 + 8 + 2 * tig) * RP + gid], wt[(k0 + 9 + 2 * tig) * RP + gid]);
                                wa0 = *reinterpret_cast<const uint32_t*>(&x0);
                                wa2 = *reinterpret_cast<const uint32_t*>(&x2);
                            }
#pragma unroll
                            for (int j = 0; j < NT; j += 2) {
                                const uint32_t arow = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
                                const uint32_t dch = j + (lane >> 4);
                                uint32_t vb[4];
                                ldmatrix_x4_trans(vb, tile + (dch >> 3) * L::kDictBox + swz128(arow, dch & 7));
                                mma_16816(o[j], wa0, 0u, wa2, 0u, vb[0], vb[1]);
                                mma_16816(o[j + 1], wa0, 0u, wa2, 0u, vb[2], vb[3]);
                            }
                        }
                    }
                    __syncwarp();
                    named_bar(kColdBar, 128);  // every warp done with this V tile and its weights
                    if (leader) mbar_arrive(&empty_d[s]);
                }
            }
            if (gid < R) {
                float* oc = ha.ocold + (static_cast<uint64_t>(bg) * RP + gid) * D + 2 * tig;
#pragma unroll
                for (int j = 0; j < NT; ++j) red_add_v2(oc + j * 8, o[j][0], o[j][1]);
            }
            named_bar(kColdBar, 128);
            if (leader) {
                const uint32_t old = atom_add_acq_rel_gpu(&cnt[HC_FIN * NB + bg], n_ct);
                *cflag = (old + n_ct == mfin) ? 1u : 0u;
                stamp(ha, TR_CONTRACT_DONE);
            }
            named_bar(kColdBar, 128);
            if (*cflag) {
                if (leader) stamp(ha, TR_HOT_WIDE);
                merge_bg = bg, merge_s0 = ms0, merge_ns = mns, merge_cold = true;
            }
        }
        // the cold group's merges through one call site (the code is large and
        // shared-instruction-cache space is what this kernel runs short of):
        // the contraction's (b, g) when it finished last, and on CTA 0 the
        // (b, g) pairs without any block, whose outputs are zeros
        const uint32_t n_merge = (merge_bg != ~0u ? 1u : 0u) + (cta == 0 ? ha.n_empty : 0u);
        for (uint32_t e = 0; e < n_merge; ++e) {
            const bool own = merge_bg != ~0u && e == 0;
            const uint32_t ebg = own ? merge_bg : ha.empty_bg[e - (merge_bg != ~0u ? 1u : 0u)];
            final_merge<D, RP>(ha, ebg, own ? merge_s0 : 0u, own ? merge_ns : 0u, own && merge_cold, ct, kColdBar, cmrg, ws);
            if (leader && own) stamp(ha, TR_MERGE_DONE);
        }
    } else {
        // =================== hot consumers (128 threads) ====================
        // Tensor-core attention per 16-token block (mma.sync m16n8k16, f16 in,
        // fp32 accumulate), FlashAttention-2 register layout: S^T = Q K^T puts
        // row gid, tokens 2tig, 2tig+1 (+8) in each lane, which is exactly the
        // A-operand layout of P for O += P V.  Query rows are M = 16 rows of
        // which the first RP (<= 8) are real.
        const uint32_t ht = tid - 224, hw = ht >> 5;
        const uint32_t gid = lane >> 2, tig = lane & 3;
        constexpr int KS = D / 16;   // k-steps over head_dim
        constexpr int NT = D / 8;    // n-tiles of the output
        if (ch.n_pages) {
            // help score this CTA's cold chunk first (the hot stream starts
            // after the chunk's codes have landed anyway)
            const bool okk = mbar_wait(kbar, 0, a.status, 16);
            const bool okq = mbar_wait(qbar, 0, a.status, 17);
            float mx[RP];
#pragma unroll
            for (int r = 0; r < RP; ++r) mx[r] = -INFINITY;
            if (okk && okq) score_tokens<RP>(128 + ht, ch.n_pages * kBlock, A, cinv, kbuf, qlg, a.status, mx);
#pragma unroll
            for (int r = 0; r < RP; ++r) {
                const float m = warp_max(mx[r]);
                if (lane == 0) cred[(4 + hw) * RP + r] = m;
            }
            named_bar(kScoreBar, 256);
        }
        uint32_t k = 0;
        for (uint32_t gi = g0; gi < g1; ++gi) {
            const FusedHotGroup gr = ha.groups[gi];
            const uint32_t b = gr.b, g = gr.g, bg = b * Hkv + g;
            const uint32_t np = gr.page_end - gr.page_begin;
            const uint32_t Th = (a.hot_indptr[b + 1] - a.hot_indptr[b]) * kBlock;
            // the pair's merge inputs and finisher count, read now, used after the pages
            const uint32_t ms0 = ha.slot_ptr[bg], mns = ha.slot_ptr[bg + 1] - ms0, mfin = fin_target(ha, bg);
            const bool mcold = ha.n_chunks[bg] > 0;
            // query fragments (A operand of S^T = Q K^T), rows >= R zero
            uint32_t qf[KS][2];
            {
                const uint32_t n = gi - g0, qs = n & 1u;
                const bool okq = __all_sync(0xffffffffu, mbar_wait(&full_q[qs], (n >> 1) & 1, a.status, 14));
                const __half* qrow = qhb + (qs * RP + (gid < RP ? gid : 0)) * D;
                const bool live = okq && gid < R;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    qf[ks][0] = live ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * tig) : 0u;
                    qf[ks][1] = live ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * tig) : 0u;
                }
                named_bar(kHotBar, 128);
                if (ht == 0) mbar_arrive(&empty_q[qs]);
            }
            // causal limit of this lane's query row (row gid)
            int32_t limit = static_cast<int32_t>(Th);
            if ((a.flags & 1u) && gid < R)
                limit = static_cast<int32_t>(Th) - static_cast<int32_t>(nq) + 1 + static_cast<int32_t>(gid / G);
            float m_run = -INFINITY, l_run = 0.0f;
            float o[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
            for (uint32_t i = hw; i < np; i += 4) {
                const uint32_t kk = k + i, s = kk % nst;
                // warp-uniform and converged: ldmatrix / mma below are .sync.aligned
                if (!__all_sync(0xffffffffu, mbar_wait(&full_h[s], (kk / nst) & 1, a.status, 15))) break;
                const bool pvalid = hflags[s] != 0;
                const uint8_t* Ks = HSTAGE(s);
                const uint8_t* Vs = Ks + L::kHotPage;
                // S^T[row][tok]: c[0] tokens 0-7, c[1] tokens 8-15
                float c[2][4];
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int e = 0; e < 4; ++e) c[h][e] = 0.0f;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    // B = K^T: rows of K (tokens), two 16-byte d-chunks; x4 covers both token halves
                    const uint32_t trow = (lane & 7) + (lane >> 4) * 8;
                    const uint32_t dch = ks * 2 + ((lane >> 3) & 1);
                    uint32_t kb[4];
                    ldmatrix_x4(kb, Ks + (dch >> 3) * L::kHotBox + swz128(trow, dch & 7));
                    mma_16816(c[0], qf[ks][0], 0u, qf[ks][1], 0u, kb[0], kb[1]);
                    mma_16816(c[1], qf[ks][0], 0u, qf[ks][1], 0u, kb[2], kb[3]);
                }
                // scale, mask, online softmax for row gid (4 lanes share a row)
                const int32_t pos0 = static_cast<int32_t>(gr.pos_base + i * kBlock);
                float sv[4];
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int32_t pos = pos0 + h * 8 + 2 * static_cast<int32_t>(tig) + e;
                        sv[h * 2 + e] = (pvalid && pos < limit) ? c[h][e] * a.scale : -INFINITY;
                    }
                float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                const float m_new = fmaxf(m_run, mx);
                const float alpha = exp_shift(m_run, m_new);
                float pv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) pv[e] = exp_shift(sv[e], m_new);
                l_run = l_run * alpha + (pv[0] + pv[1]) + (pv[2] + pv[3]);
                m_run = m_new;
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    o[j][0] *= alpha;
                    o[j][1] *= alpha;
                }
                // O += P V: A = P (row gid; tokens 2tig.. and 8+2tig..), B = V via transposed loads
                const __half2 p01 = __floats2half2_rn(pv[0], pv[1]);
                const __half2 p89 = __floats2half2_rn(pv[2], pv[3]);
                const uint32_t pa0 = *reinterpret_cast<const uint32_t*>(&p01);
                const uint32_t pa2 = *reinterpret_cast<const uint32_t*>(&p89);
#pragma unroll
                for (int j = 0; j < NT; j += 2) {
                    const uint32_t trow = (lane & 7) + ((lane >> 3) & 1) * 8;
                    const uint32_t dch = j + (lane >> 4);
                    uint32_t vb[4];
                    ldmatrix_x4_trans(vb, Vs + (dch >> 3) * L::kHotBox + swz128(trow, dch & 7));
                    mma_16816(o[j], pa0, 0u, pa2, 0u, vb[0], vb[1]);
                    mma_16816(o[j + 1], pa0, 0u, pa2, 0u, vb[2], vb[3]);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty_h[s]);
            }
            k += np;
            // this warp's (m, l, o) for row gid
            l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
            l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
            if (gid < static_cast<uint32_t>(RP)) {
                if (tig == 0) {
                    hcm[hw * RP + gid] = m_run;
                    hcl[hw * RP + gid] = l_run;
                }
#pragma unroll
                for (int j = 0; j < NT; ++j)
                    *reinterpret_cast<float2*>(&hco[(hw * RP + gid) * D + j * 8 + 2 * tig]) = make_float2(o[j][0], o[j][1]);
            }
            named_bar(kHotBar, 128);
            for (uint32_t idx = ht; idx < RP * D; idx += 128) {
                const uint32_t r = idx / D, dim = idx % D;
                float M = -INFINITY;
#pragma unroll
                for (int w2 = 0; w2 < 4; ++w2) M = fmaxf(M, hcm[w2 * RP + r]);
                float Ls = 0.0f, O = 0.0f;
#pragma unroll
                for (int w2 = 0; w2 < 4; ++w2) {
                    const float f = exp_shift(hcm[w2 * RP + r], M);
                    Ls += hcl[w2 * RP + r] * f;
                    O += hco[(w2 * RP + r) * D + dim] * f;
                }
                if (dim == 0) {
                    __stcg(&ha.sm[gr.slot * RP + r], M);
                    __stcg(&ha.sl[gr.slot * RP + r], Ls);
                }
                __stcg(&ha.so[(static_cast<uint64_t>(gr.slot) * RP + r) * D + dim], O);
            }
            named_bar(kHotBar, 128);
            if (gi + 1 == g1 && ht == 0) stamp(ha, TR_HOT_DONE);
            if (ht == 0) {
                const uint32_t old = atom_add_acq_rel_gpu(&cnt[HC_FIN * NB + bg], 1u);
                *hflag = (old + 1 == mfin) ? 1u : 0u;
            }
            named_bar(kHotBar, 128);
            if (*hflag) {
                if (ht == 0) stamp(ha, TR_HOT_MERGE);
                final_merge<D, RP>(ha, bg, ms0, mns, mcold, ht, kHotBar, hmrg, hco);
                if (ht == 0) stamp(ha, TR_MERGE_DONE);
            }
        }
    }

#undef HSTAGE
    // ---- exit: the last CTA resets the dependency counters for the next step
    __syncthreads();
    if (tid == 0) {
        stamp(ha, TR_EXIT);
        const uint32_t done = atom_add_acq_rel_gpu(&cnt[HC_KINDS * NB], 1u);
        if (done == ha.n_ctas - 1) {
            for (uint32_t i = 0; i < HC_KINDS * NB + 1; ++i) cnt[i] = 0u;
            if (ha.ll_world) ha.ll_state[0] += 1u;  // the next step's tag
            __threadfence();
        }
    }
}

namespace {

template <int D, int RP>
constexpr size_t hp_bytes() {
    return HpLayout<D, RP>::total + 1024;  // + alignment slack
}

template <int D, int RP>
cudaError_t hp_occupancy_t(int* n) {
    const size_t smem = hp_bytes<D, RP>();
    cudaError_t e = cudaFuncSetAttribute(hp_step_kernel<D, RP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, hp_step_kernel<D, RP>, kThreads, smem);
}

template <int D, int RP>
cudaError_t launch_hp_t(const HpArgs& ha, const CUtensorMap& hk, const CUtensorMap& hv, const CUtensorMap& kd,
                        const CUtensorMap& vd, const CUtensorMap& kc, const CUtensorMap& vc, cudaStream_t s) {
    const size_t smem = hp_bytes<D, RP>();
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(hp_step_kernel<D, RP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ha.n_ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, hp_step_kernel<D, RP>, hk, hv, kd, vd, kc, vc, ha);
}

}  // namespace

size_t hp_smem_bytes(uint32_t D, uint32_t RP) {
    size_t b = 0;
    if (D == 128) {
        if (RP == 1) b = hp_bytes<128, 1>();
        else if (RP == 2) b = hp_bytes<128, 2>();
        else if (RP == 4) b = hp_bytes<128, 4>();
    } else if (D == 64) {
        if (RP == 1) b = hp_bytes<64, 1>();
        else if (RP == 2) b = hp_bytes<64, 2>();
        else if (RP == 4) b = hp_bytes<64, 4>();
    }
    return b <= 227 * 1024 ? b : 0;
}

cudaError_t hp_occupancy(uint32_t D, uint32_t RP, int* n) {
    *n = 0;
    if (D == 128) {
        if (RP == 1) return hp_occupancy_t<128, 1>(n);
        if (RP == 2) return hp_occupancy_t<128, 2>(n);
        if (RP == 4) return hp_occupancy_t<128, 4>(n);
    } else if (D == 64) {
        if (RP == 1) return hp_occupancy_t<64, 1>(n);
        if (RP == 2) return hp_occupancy_t<64, 2>(n);
        if (RP == 4) return hp_occupancy_t<64, 4>(n);
    }
    return cudaSuccess;
}

cudaError_t launch_hp(const HpArgs& ha, const CUtensorMap& hk, const CUtensorMap& hv, const CUtensorMap& kd,
                      const CUtensorMap& vd, const CUtensorMap& kc, const CUtensorMap& vc, cudaStream_t s) {
    const uint32_t D = ha.r.D, RP = ha.r.RP;
    if (D == 128) {
        if (RP == 1) return launch_hp_t<128, 1>(ha, hk, hv, kd, vd, kc, vc, s);
        if (RP == 2) return launch_hp_t<128, 2>(ha, hk, hv, kd, vd, kc, vc, s);
        if (RP == 4) return launch_hp_t<128, 4>(ha, hk, hv, kd, vd, kc, vc, s);
    } else if (D == 64) {
        if (RP == 1) return launch_hp_t<64, 1>(ha, hk, hv, kd, vd, kc, vc, s);
        if (RP == 2) return launch_hp_t<64, 2>(ha, hk, hv, kd, vd, kc, vc, s);
        if (RP == 4) return launch_hp_t<64, 4>(ha, hk, hv, kd, vd, kc, vc, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace weaver
