// weaver_fused.cu — the whole decode step as one persistent, warp-specialised
// kernel (one CTA per SM, cooperative launch so every CTA is resident).
//
// Every CTA owns a byte-balanced share of all the step's HBM traffic and
// starts streaming it at once through three TMA rings:
//   dict ring (2 x 128-atom tiles): K_dict tiles for q_latent, later V_dict
//                                   tiles for the contraction,
//   code ring (6 x 8 KB):          K-code and V-code blocks,
//   hot ring  (8 stages):          hot K/V blocks of one kv head.
// Warp roles (10 warps):
//   warp 0  lane 0 dict producer, lane 1 code producer
//   warp 1  lane 0 hot producer
//   warps 2-5  cold consumers: q_latent tiles -> cold scores -> scatter of
//              p*cV into per-atom weights w -> w . V_dict -> final merge
//   warps 6-9  hot consumers: exact split-KV attention, one (m, l, o)
//              partial per (CTA, sequence, kv head) group
// The cold chain's dependencies are per-sequence counters in global memory
// (release: fence + atomicAdd; acquire: ld.acquire polled by one thread, then
// a named barrier).  Each CTA runs its cold list in phase order (all q_latent
// tiles, then scores, then scatters, then contractions, then merge rows) and
// every wait is on an earlier phase, so with all CTAs resident no wait can
// deadlock.  Every wait is bounded: on expiry it records DEVERR_TIMEOUT and the
// kernel carries on to its end.  The last CTA to finish resets the counters.
#include "weaver_device.cuh"
#include "weaver_internal.hpp"

namespace weaver {
namespace {

constexpr int kThreads = 320;
constexpr int kDictSlots = 2;
constexpr int kCodeSlots = 6;
constexpr int kHotStages = 8;
constexpr uint32_t kCodeSlotBytes = 8192;
constexpr uint32_t kColdBar = 1, kHotBar = 2;
constexpr int kMergeBatch = 32;             // hot slots loaded per round in the merge

template <int D, int RP>
struct Layout {
    static constexpr uint32_t kBoxes = D / 64;
    static constexpr uint32_t kDictBox = kAtomTile * 128;        // 128 rows x 64 f16
    static constexpr uint32_t kDictSlot = kBoxes * kDictBox;
    static constexpr uint32_t kHotBox = kBlock * 128;            // 16 rows x 64 f16
    static constexpr uint32_t kHotPage = kBoxes * kHotBox;
    static constexpr uint32_t kHotStage = 2 * kHotPage;          // K then V
    static constexpr uint32_t dict = 0;
    static constexpr uint32_t hot = dict + kDictSlots * kDictSlot;
    static constexpr uint32_t code = hot + kHotStages * kHotStage;
    static constexpr uint32_t hcm = code + kCodeSlots * kCodeSlotBytes;  // [4][RP]
    static constexpr uint32_t hcl = hcm + 4 * RP * 4;                     // [4][RP]
    static constexpr uint32_t hco = hcl + 4 * RP * 4;                     // [4][RP][D]
    static constexpr uint32_t cred = hco + 4 * RP * D * 4;                // [128][RP]
    static constexpr uint32_t ws = cred + 128 * RP * 4;                   // [128][RP] w tile
    static constexpr uint32_t ms = ws + 128 * RP * 4;                     // [128][RP] cold max per head
    static constexpr uint32_t hvalid = ms + 128 * RP * 4;                 // [kHotStages] u32
    static constexpr uint32_t cvalid = hvalid + kHotStages * 4;           // [kCodeSlots] u32
    static constexpr uint32_t bars = (cvalid + kCodeSlots * 4 + 7) / 8 * 8;
    // full/empty for dict, code, hot
    static constexpr uint32_t nbars = 2 * (kDictSlots + kCodeSlots + kHotStages);
    static constexpr uint32_t total = bars + nbars * 8;
};

template <int RP>
__device__ __forceinline__ void ldcg_rows(const float* p, float v[RP]) {
    if constexpr (RP >= 4) {
#pragma unroll
        for (int r = 0; r < RP; r += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(p + r));
            v[r] = x.x;
            v[r + 1] = x.y;
            v[r + 2] = x.z;
            v[r + 3] = x.w;
        }
    } else if constexpr (RP == 2) {
        const float2 x = __ldcg(reinterpret_cast<const float2*>(p));
        v[0] = x.x;
        v[1] = x.y;
    } else {
        v[0] = __ldcg(p);
    }
}

template <int RP>
__device__ __forceinline__ void stcg_rows(float* p, const float v[RP]) {
    if constexpr (RP >= 4) {
#pragma unroll
        for (int r = 0; r < RP; r += 4) __stcg(reinterpret_cast<float4*>(p + r), make_float4(v[r], v[r + 1], v[r + 2], v[r + 3]));
    } else if constexpr (RP == 2) {
        __stcg(reinterpret_cast<float2*>(p), make_float2(v[0], v[1]));
    } else {
        __stcg(p, v[0]);
    }
}

// One thread waits until cnt0 >= t0 and cnt1 >= t1 (bounded by kWaitNs, fail
// fast after another timeout), then the named group of 128 threads syncs.
__device__ __forceinline__ void wait_counts(const uint32_t* cnt0, uint32_t t0, const uint32_t* cnt1, uint32_t t1,
                                            uint32_t* status, bool leader, uint32_t bar_id) {
    if (leader) {
        auto ready = [&]() { return ld_acquire_gpu(cnt0) >= t0 && (!cnt1 || ld_acquire_gpu(cnt1) >= t1); };
        if (!ready()) {
            const uint64_t start = globaltimer_ns();
            uint32_t ns = 32;
            while (!ready()) {
                if (timed_out(status)) break;
                if (globaltimer_ns() - start > kWaitNs) {
                    atomicOr(status, DEVERR_TIMEOUT);
                    break;
                }
                __nanosleep(ns);
                if (ns < 256) ns <<= 1;
            }
        }
    }
    named_bar(bar_id, 128);
}

__device__ __forceinline__ void wait_count(const uint32_t* cnt, uint32_t target, uint32_t* status, bool leader,
                                           uint32_t bar_id) {
    wait_counts(cnt, target, nullptr, 0, status, leader, bar_id);
}

// Producer exit: wait (bounded) until every copy it issued into a ring of
// `slots` barriers has landed, so no copy is in flight when the CTA exits.
__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t slots, uint32_t issued) {
    for (uint32_t s = 0; s < slots && s < issued; ++s) {
        const uint32_t last = s + ((issued - 1 - s) / slots) * slots;  // last copy into slot s
        mbar_drain(&full[s], (last / slots) & 1);
    }
}

__device__ __forceinline__ void stamp(const FusedArgs& fa, uint32_t slot) {
    if (fa.trace) fa.trace[blockIdx.x * kTraceSlots + slot] = globaltimer_ns();
}

__device__ __forceinline__ const __half* q_row(const RunArgs& a, uint32_t b, uint32_t g, uint32_t row) {
    const uint32_t j = row / a.G, hh = row % a.G;
    return a.q + ((static_cast<uint64_t>(b) * a.nq + j) * a.Hq + g * a.G + hh) * a.D;
}

}  // namespace

template <int D, int RP>
__global__ void __launch_bounds__(kThreads, 1)
    fused_step_kernel(const __grid_constant__ CUtensorMap tm_hk, const __grid_constant__ CUtensorMap tm_hv,
                      const __grid_constant__ CUtensorMap tm_kd, const __grid_constant__ CUtensorMap tm_vd,
                      const FusedArgs fa) {
    using L = Layout<D, RP>;
    const RunArgs& a = fa.r;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* dict = smem + L::dict;
    uint8_t* hot = smem + L::hot;
    uint8_t* code = smem + L::code;
    float* hcm = reinterpret_cast<float*>(smem + L::hcm);
    float* hcl = reinterpret_cast<float*>(smem + L::hcl);
    float* hco = reinterpret_cast<float*>(smem + L::hco);
    float* cred = reinterpret_cast<float*>(smem + L::cred);
    float* ws = reinterpret_cast<float*>(smem + L::ws);
    float* ms = reinterpret_cast<float*>(smem + L::ms);
    uint32_t* hvalid = reinterpret_cast<uint32_t*>(smem + L::hvalid);
    uint32_t* cvalid = reinterpret_cast<uint32_t*>(smem + L::cvalid);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bars);
    uint64_t* full_d = bars;
    uint64_t* empty_d = full_d + kDictSlots;
    uint64_t* full_c = empty_d + kDictSlots;
    uint64_t* empty_c = full_c + kCodeSlots;
    uint64_t* full_h = empty_c + kCodeSlots;
    uint64_t* empty_h = full_h + kHotStages;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t cta = blockIdx.x;
    const uint32_t B = a.B, Hkv = a.Hkv, A = a.A, R = a.R;
    uint32_t* cnt = fa.counters;
    const uint32_t qlat_target = Hkv * a.n_atom_tiles;

    if (tid == 0) {
        for (int i = 0; i < kDictSlots; ++i) { mbar_init(&full_d[i], 1); mbar_init(&empty_d[i], 1); }
        for (int i = 0; i < kCodeSlots; ++i) { mbar_init(&full_c[i], 1); mbar_init(&empty_c[i], 1); }
        for (int i = 0; i < kHotStages; ++i) { mbar_init(&full_h[i], 1); mbar_init(&empty_h[i], 1); }
        fence_barrier_init();
        if (fa.trace)
            for (uint32_t i = 0; i < kTraceSlots; ++i) fa.trace[cta * kTraceSlots + i] = 0;
        stamp(fa, TR_START);
    }
    __syncthreads();

    const uint32_t i0 = fa.item_ptr[cta], i1 = fa.item_ptr[cta + 1];
    const uint32_t g0 = fa.group_ptr[cta], g1 = fa.group_ptr[cta + 1];

    if (warp == 0) {
        if (lane == 0) {
            // ---- dict producer: K_dict tiles (q_latent), then V_dict tiles (contraction)
            if (i1 > i0) {
                prefetch_tensormap(&tm_kd);
                prefetch_tensormap(&tm_vd);
            }
            uint32_t k = 0;
            for (uint32_t i = i0; i < i1; ++i) {
                const FusedItem it = fa.items[i];
                if (it.type != FI_QLAT && it.type != FI_CONTRACT) continue;
                const uint32_t s = k % kDictSlots;
                if (k >= kDictSlots && !mbar_wait(&empty_d[s], ((k / kDictSlots) - 1) & 1, a.status)) break;
                const CUtensorMap* map = it.type == FI_QLAT ? &tm_kd : &tm_vd;
                const int32_t y = static_cast<int32_t>(it.g * a.dict_row_stride + it.a * kAtomTile);
                mbar_arrive_expect_tx(&full_d[s], L::kDictSlot);
#pragma unroll
                for (uint32_t bx = 0; bx < L::kBoxes; ++bx)
                    tma_load_2d(dict + s * L::kDictSlot + bx * L::kDictBox, map, &full_d[s], bx * 64, y);
                ++k;
            }
            drain_ring(full_d, kDictSlots, k);
        } else if (lane == 1) {
            // ---- code producer: K-code blocks (scores), then V-code blocks (scatter)
            const uint32_t page_bytes = kBlock * Hkv * 16;
            uint32_t k = 0;
            for (uint32_t i = i0; i < i1; ++i) {
                const FusedItem it = fa.items[i];
                if (it.type != FI_SCORE && it.type != FI_SCATTER) continue;
                const uint32_t s = k % kCodeSlots;
                if (k >= kCodeSlots && !mbar_wait(&empty_c[s], ((k / kCodeSlots) - 1) & 1, a.status)) break;
                const uint4* pool = it.type == FI_SCORE ? a.cold_k : a.cold_v;
                uint32_t valid = 0, bytes = 0;
                for (uint32_t p = 0; p < it.n; ++p) {
                    const uint32_t phys = a.cold_refs[it.a + p] & kRefMask;
                    if (phys < a.cold_pool_blocks) {
                        valid |= 1u << p;
                        bytes += page_bytes;
                    } else {
                        atomicOr(a.status, DEVERR_REF_RANGE);
                    }
                }
                cvalid[s] = valid;
                mbar_arrive_expect_tx(&full_c[s], bytes);
                for (uint32_t p = 0; p < it.n; ++p) {
                    if (!((valid >> p) & 1u)) continue;
                    const uint32_t phys = a.cold_refs[it.a + p] & kRefMask;
                    bulk_load(code + s * kCodeSlotBytes + p * page_bytes,
                              pool + static_cast<uint64_t>(phys) * kBlock * Hkv, page_bytes, &full_c[s]);
                }
                ++k;
            }
            drain_ring(full_c, kCodeSlots, k);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- hot producer: K/V blocks of this CTA's hot groups, in order
            if (g1 > g0) {
                prefetch_tensormap(&tm_hk);
                prefetch_tensormap(&tm_hv);
            }
            // let this CTA's q_latent dictionary tiles (the head of the cold
            // critical path) land before the hot stream competes for HBM
            uint32_t n_first = 0;
            for (uint32_t i = i0; i < i1 && n_first < kDictSlots && fa.items[i].type == FI_QLAT; ++i) ++n_first;
            for (uint32_t s = 0; s < n_first; ++s) mbar_drain(&full_d[s], 0);
            uint32_t k = 0;
            for (uint32_t gi = g0; gi < g1; ++gi) {
                const FusedHotGroup gr = fa.groups[gi];
                for (uint32_t p = gr.page_begin; p < gr.page_end; ++p, ++k) {
                    const uint32_t s = k % kHotStages;
                    if (k >= kHotStages && !mbar_wait(&empty_h[s], ((k / kHotStages) - 1) & 1, a.status)) {
                        gi = g1;
                        break;
                    }
                    const uint32_t phys = a.hot_refs[p] & kRefMask;
                    if (phys >= a.hot_pool_blocks) {
                        atomicOr(a.status, DEVERR_REF_RANGE);
                        hvalid[s] = 0;
                        mbar_arrive(&full_h[s]);
                        continue;
                    }
                    hvalid[s] = 1;
                    uint8_t* dst = hot + s * L::kHotStage;
                    mbar_arrive_expect_tx(&full_h[s], L::kHotStage);
#pragma unroll
                    for (uint32_t bx = 0; bx < L::kBoxes; ++bx) {
                        const int32_t x = static_cast<int32_t>(gr.g * D + bx * 64);
                        const int32_t y = static_cast<int32_t>(phys * kBlock);
                        tma_load_2d(dst + bx * L::kHotBox, &tm_hk, &full_h[s], x, y);
                        tma_load_2d(dst + L::kHotPage + bx * L::kHotBox, &tm_hv, &full_h[s], x, y);
                    }
                }
            }
            drain_ring(full_h, kHotStages, k);
        }
    } else if (warp < 6) {
        // =================== cold consumers (128 threads) ===================
        const uint32_t ct = tid - 64, cw = ct >> 5;
        const bool leader = ct == 0;
        uint32_t kd = 0, kc = 0;
        for (uint32_t i = i0; i < i1; ++i) {
            const FusedItem it = fa.items[i];
            const uint32_t b = it.b;
            if (it.type == FI_QLAT) {
                const uint32_t g = it.g, t = it.a, s = kd % kDictSlots;
                const uint32_t gid = lane >> 2, tig = lane & 3;
                if (t == 0) {
                    // first tile of (b, g): reset the cold accumulators of this step
                    float* oc = fa.ocold + (static_cast<uint64_t>(b) * Hkv + g) * RP * D;
                    for (uint32_t idx = ct; idx < RP * D; idx += 128) oc[idx] = 0.0f;
                    if (ct < RP) {
                        fa.lcold[(b * Hkv + g) * RP + ct] = 0.0f;
                        fa.mkey[(b * Hkv + g) * RP + ct] = fkey(-INFINITY);
                    }
                }
                // q_latent tile on tensor cores: C (128 atoms x 8 query rows) =
                // K_dict tile (A operand, ldmatrix from the swizzled TMA tile) .
                // q^T (B operand: f16 query rows straight from global memory)
                const bool ok = __all_sync(0xffffffffu, mbar_wait(&full_d[s], (kd / kDictSlots) & 1, a.status));
                float cq[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) cq[mt][e] = 0.0f;
                if (ok) {
                    const uint8_t* tile = dict + s * L::kDictSlot;
                    const bool qlive = gid < R;
                    const __half* qr = q_row(a, b, g, qlive ? gid : 0);
#pragma unroll
                    for (int ks = 0; ks < D / 16; ++ks) {
                        const uint32_t b0 = qlive ? *reinterpret_cast<const uint32_t*>(qr + ks * 16 + 2 * tig) : 0u;
                        const uint32_t b1 = qlive ? *reinterpret_cast<const uint32_t*>(qr + ks * 16 + 8 + 2 * tig) : 0u;
#pragma unroll
                        for (int mt = 0; mt < 2; ++mt) {
                            const uint32_t arow = cw * 32 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                            const uint32_t kc = ks * 2 + (lane >> 4);
                            uint32_t af[4];
                            ldmatrix_x4(af, tile + (kc >> 3) * L::kDictBox + swz128(arow, kc & 7));
                            mma_16816(cq[mt], af, b0, b1);
                        }
                    }
                }
                // C fragment: atom rows gid / gid + 8, query rows 2tig, 2tig + 1
                if (2 * tig < static_cast<uint32_t>(RP)) {
#pragma unroll
                    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                        for (int hi = 0; hi < 2; ++hi) {
                            const uint32_t atom = t * kAtomTile + cw * 32 + mt * 16 + gid + hi * 8;
                            if (atom >= A) continue;
                            float* dst = a.qlat + ((static_cast<uint64_t>(b) * Hkv + g) * A + atom) * RP + 2 * tig;
                            if constexpr (RP >= 2) {
                                __stcg(reinterpret_cast<float2*>(dst),
                                       make_float2(cq[mt][hi * 2] * a.scale, cq[mt][hi * 2 + 1] * a.scale));
                            } else {
                                __stcg(dst, cq[mt][hi * 2] * a.scale);
                            }
                        }
                }
                {
                    const uint32_t atom = t * kAtomTile + ct;
                    if (atom < A) {
                        float z[RP];
#pragma unroll
                        for (int r = 0; r < RP; ++r) z[r] = 0.0f;
                        stcg_rows<RP>(a.w + ((static_cast<uint64_t>(b) * Hkv + g) * A + atom) * RP, z);
                    }
                }
                named_bar(kColdBar, 128);
                if (leader) {
                    mbar_arrive(&empty_d[s]);
                    __threadfence();
                    atomicAdd(&cnt[CNT_QLAT * B + b], 1u);
                    stamp(fa, TR_QLAT_DONE);
                }
                ++kd;
            } else if (it.type == FI_SCORE || it.type == FI_SCATTER) {
                // A run: consecutive SCORE (or SCATTER) items of one sequence, all
                // resident in the code ring at once, processed as one pair space
                // with kBatch pairs per thread in flight and one signal at the end.
                const bool scoring = it.type == FI_SCORE;
                uint32_t n_run = 1;
                while (i + n_run < i1 && n_run < kCodeSlots && fa.items[i + n_run].type == it.type &&
                       fa.items[i + n_run].b == b)
                    ++n_run;
                if (scoring) {
                    wait_count(&cnt[CNT_QLAT * B + b], qlat_target, a.status, leader, kColdBar);
                    if (leader) stamp(fa, TR_SCORE_WAIT);
                } else {
                    wait_count(&cnt[CNT_SCORE * B + b], fa.code_items[b], a.status, leader, kColdBar);
                    if (leader) stamp(fa, TR_SCATTER_WAIT);
                    if (ct < Hkv * RP) ms[ct] = unkey(__ldcg(&fa.mkey[b * Hkv * RP + ct]));
                }
                const uint32_t per_page = kBlock * Hkv;
                uint32_t off[kCodeSlots + 1];
                uint32_t valid[kCodeSlots];
                bool ok = true;
                off[0] = 0;
#pragma unroll
                for (uint32_t u = 0; u < kCodeSlots; ++u) {
                    if (u < n_run) {
                        const uint32_t su = (kc + u) % kCodeSlots;
                        ok = mbar_wait(&full_c[su], ((kc + u) / kCodeSlots) & 1, a.status) && ok;
                        valid[u] = ok ? cvalid[su] : 0u;
                        off[u + 1] = off[u] + fa.items[i + u].n * per_page;
                    } else {
                        valid[u] = 0u;
                        off[u + 1] = off[u];
                    }
                }
                named_bar(kColdBar, 128);  // ms[] visible
                const uint32_t total = off[n_run];
                constexpr int kBatch = RP >= 8 ? 2 : 4;
                float acc[RP];  // running max (scores) or sum of p (scatter)
#pragma unroll
                for (int r = 0; r < RP; ++r) acc[r] = scoring ? -INFINITY : 0.0f;
                const float* qbase = a.qlat + static_cast<uint64_t>(b) * Hkv * A * RP;
                float* wbase = a.w + static_cast<uint64_t>(b) * Hkv * A * RP;
                for (uint32_t q0 = 0; q0 < total; q0 += 128 * kBatch) {
                    uint4 cd[kBatch];
                    uint32_t gq[kBatch];
                    uint64_t tok[kBatch];
                    bool live[kBatch];
#pragma unroll
                    for (int m = 0; m < kBatch; ++m) {
                        const uint32_t q = q0 + ct + 128u * m;
                        live[m] = false;
                        gq[m] = 0;
                        tok[m] = 0;
                        cd[m] = make_uint4(0, 0, 0, 0);
                        if (q < total) {
                            uint32_t u = 0;
#pragma unroll
                            for (uint32_t v = 1; v < kCodeSlots; ++v) u += (q >= off[v]) ? 1u : 0u;
                            const uint32_t pi = q - off[u], p = pi / per_page, rem = pi % per_page;
                            gq[m] = rem % Hkv;
                            tok[m] = static_cast<uint64_t>(fa.items[i + u].a + p) * kBlock + rem / Hkv;
                            if ((valid[u] >> p) & 1u) {
                                live[m] = true;
                                cd[m] = reinterpret_cast<const uint4*>(code + ((kc + u) % kCodeSlots) * kCodeSlotBytes)[pi];
                            }
                        }
                    }
                    if (scoring) {
                        float v[kBatch][4][RP];
#pragma unroll
                        for (int m = 0; m < kBatch; ++m) {
                            const uint16_t* idx = reinterpret_cast<const uint16_t*>(&cd[m].x);
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                if (live[m] && idx[k] < A) {
                                    ldcg_rows<RP>(qbase + (static_cast<uint64_t>(gq[m]) * A + idx[k]) * RP, v[m][k]);
                                } else {
#pragma unroll
                                    for (int r = 0; r < RP; ++r) v[m][k][r] = 0.0f;
                                }
                            }
                        }
#pragma unroll
                        for (int m = 0; m < kBatch; ++m) {
                            const uint32_t q = q0 + ct + 128u * m;
                            if (q >= total) continue;
                            const uint16_t* idx = reinterpret_cast<const uint16_t*>(&cd[m].x);
                            const uint16_t* cf = reinterpret_cast<const uint16_t*>(&cd[m].z);
                            float sc[RP];
#pragma unroll
                            for (int r = 0; r < RP; ++r) sc[r] = live[m] ? 0.0f : -INFINITY;
                            if (live[m]) {
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    if (idx[k] >= A) {
                                        atomicOr(a.status, DEVERR_ATOM_RANGE);
                                        continue;
                                    }
                                    const float c = h2f(cf[k]);
#pragma unroll
                                    for (int r = 0; r < RP; ++r) sc[r] = fmaf(c, v[m][k][r], sc[r]);
                                }
                            }
                            stcg_rows<RP>(a.scores + (static_cast<uint64_t>(gq[m]) * a.cold_tokens + tok[m]) * RP, sc);
#pragma unroll
                            for (int r = 0; r < RP; ++r) acc[r] = fmaxf(acc[r], sc[r]);
                        }
                    } else {
                        float sv[kBatch][RP];
#pragma unroll
                        for (int m = 0; m < kBatch; ++m) {
                            if (live[m]) {
                                ldcg_rows<RP>(a.scores + (static_cast<uint64_t>(gq[m]) * a.cold_tokens + tok[m]) * RP, sv[m]);
                            } else {
#pragma unroll
                                for (int r = 0; r < RP; ++r) sv[m][r] = -INFINITY;
                            }
                        }
#pragma unroll
                        for (int m = 0; m < kBatch; ++m) {
                            if (!live[m]) continue;
                            float pr[RP];
#pragma unroll
                            for (int r = 0; r < RP; ++r) {
                                pr[r] = exp_shift(sv[m][r], ms[gq[m] * RP + r]);
                                acc[r] += pr[r];
                            }
                            const uint16_t* idx = reinterpret_cast<const uint16_t*>(&cd[m].x);
                            const uint16_t* cf = reinterpret_cast<const uint16_t*>(&cd[m].z);
                            float* wb = wbase + static_cast<uint64_t>(gq[m]) * A * RP;
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                if (idx[k] >= A) {
                                    atomicOr(a.status, DEVERR_ATOM_RANGE);
                                    continue;
                                }
                                const float c = h2f(cf[k]);
                                float* dst = wb + static_cast<uint64_t>(idx[k]) * RP;
                                if constexpr (RP >= 4) {
#pragma unroll
                                    for (int r = 0; r < RP; r += 4)
                                        red_add_v4(dst + r, c * pr[r], c * pr[r + 1], c * pr[r + 2], c * pr[r + 3]);
                                } else if constexpr (RP == 2) {
                                    red_add_v2(dst, c * pr[0], c * pr[1]);
                                } else {
                                    atomicAdd(dst, c * pr[0]);
                                }
                            }
                        }
                    }
                }
                // per-head reduction: thread ct always sees head ct % Hkv (Hkv divides 128)
#pragma unroll
                for (int r = 0; r < RP; ++r) cred[ct * RP + r] = acc[r];
                named_bar(kColdBar, 128);
                if (ct < Hkv * RP) {
                    const uint32_t g = ct / RP, r = ct % RP;
                    float x = scoring ? -INFINITY : 0.0f;
                    for (uint32_t t2 = g; t2 < 128; t2 += Hkv)
                        x = scoring ? fmaxf(x, cred[t2 * RP + r]) : x + cred[t2 * RP + r];
                    if (scoring) atomicMax(&fa.mkey[(b * Hkv + g) * RP + r], fkey(x));
                    else atomicAdd(&fa.lcold[(b * Hkv + g) * RP + r], x);
                }
                named_bar(kColdBar, 128);
                if (leader) {
                    for (uint32_t u = 0; u < n_run; ++u) mbar_arrive(&empty_c[(kc + u) % kCodeSlots]);
                    __threadfence();
                    atomicAdd(&cnt[(scoring ? CNT_SCORE : CNT_SCATTER) * B + b], n_run);
                    stamp(fa, scoring ? TR_SCORE_DONE : TR_SCATTER_DONE);
                }
                kc += n_run;
                i += n_run - 1;
            } else {  // FI_CONTRACT
                const uint32_t g = it.g, t = it.a, s = kd % kDictSlots;
                wait_count(&cnt[CNT_SCATTER * B + b], fa.code_items[b], a.status, leader, kColdBar);
                if (leader && fa.trace && !fa.trace[cta * kTraceSlots + TR_CONTRACT_WAIT]) stamp(fa, TR_CONTRACT_WAIT);
                {
                    const uint32_t atom = t * kAtomTile + ct;
                    float v[RP];
                    if (atom < A) {
                        ldcg_rows<RP>(a.w + ((static_cast<uint64_t>(b) * Hkv + g) * A + atom) * RP, v);
                    } else {
#pragma unroll
                        for (int r = 0; r < RP; ++r) v[r] = 0.0f;
                    }
#pragma unroll
                    for (int r = 0; r < RP; ++r) ws[ct * RP + r] = v[r];
                }
                named_bar(kColdBar, 128);
                // contraction on tensor cores: O (query rows x D) += W (rows x 128
                // atoms, f16 from the staged fp32 weights) . V_dict tile (ldmatrix.trans);
                // warp cw takes atoms cw*32 .. cw*32+31
                const bool ok = __all_sync(0xffffffffu, mbar_wait(&full_d[s], (kd / kDictSlots) & 1, a.status));
                constexpr int NT = D / 8;
                const uint32_t gid = lane >> 2, tig = lane & 3;
                float o[NT][4];
#pragma unroll
                for (int j = 0; j < NT; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
                if (ok) {
                    const uint8_t* tile = dict + s * L::kDictSlot;
#pragma unroll
                    for (int ks = 0; ks < 2; ++ks) {
                        const uint32_t k0 = cw * 32 + ks * 16;
                        uint32_t wa0 = 0u, wa2 = 0u;
                        if (gid < static_cast<uint32_t>(RP)) {
                            const __half2 x0 = __floats2half2_rn(ws[(k0 + 2 * tig) * RP + gid], ws[(k0 + 2 * tig + 1) * RP + gid]);
                            const __half2 x2 = __floats2half2_rn(ws[(k0 + 8 + 2 * tig) * RP + gid], ws[(k0 + 9 + 2 * tig) * RP + gid]);
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
                if (gid < R) {
                    float* oc = fa.ocold + ((static_cast<uint64_t>(b) * Hkv + g) * RP + gid) * D + 2 * tig;
#pragma unroll
                    for (int j = 0; j < NT; ++j) red_add_v2(oc + j * 8, o[j][0], o[j][1]);
                }
                named_bar(kColdBar, 128);
                if (leader) {
                    mbar_arrive(&empty_d[s]);
                    __threadfence();
                    atomicAdd(&cnt[CNT_CONTRACT * B + b], 1u);
                    stamp(fa, TR_CONTRACT_DONE);
                }
                ++kd;
            }
        }
        // ---- merge rows: hot slots of (b, g) + the cold partial
        const uint32_t m0 = fa.merge_ptr[cta], m1 = fa.merge_ptr[cta + 1];
        for (uint32_t mi = m0; mi < m1; ++mi) {
            const uint32_t row = fa.merge_rows[mi];
            const uint32_t h = row % a.Hq, j = (row / a.Hq) % a.nq, b = row / (a.Hq * a.nq);
            const uint32_t g = h / a.G, r = j * a.G + h % a.G;
            const bool has_cold = fa.code_items[b] > 0;
            // wait for every contraction and every hot group of the sequence
            wait_counts(&cnt[CNT_HOT * B + b], fa.hot_groups[b], has_cold ? &cnt[CNT_CONTRACT * B + b] : nullptr,
                        qlat_target, a.status, leader, kColdBar);
            if (leader) stamp(fa, TR_MERGE_WAIT);
            const uint32_t dim = ct;
            if (dim < D) {
                float M = -INFINITY, Mc = -INFINITY, lc = 0.0f, oc = 0.0f;
                const uint32_t bg = b * Hkv + g;
                if (has_cold) {
                    Mc = unkey(__ldcg(&fa.mkey[bg * RP + r]));
                    lc = __ldcg(&fa.lcold[bg * RP + r]);
                    oc = __ldcg(&fa.ocold[(static_cast<uint64_t>(bg) * RP + r) * D + dim]);
                    M = Mc;
                }
                const uint32_t s0 = fa.slot_ptr[bg], s1 = fa.slot_ptr[bg + 1];
                float L = 0.0f, O = 0.0f;
                // running rescale over batches of hot slots (loads of a batch issued together)
                for (uint32_t sb = s0; sb < s1; sb += kMergeBatch) {
                    float mv[kMergeBatch], lv[kMergeBatch], ov[kMergeBatch];
#pragma unroll
                    for (int q = 0; q < kMergeBatch; ++q) {
                        if (sb + q < s1) {
                            const uint32_t sl = sb + q;  // the slots of (b, g) are contiguous
                            mv[q] = __ldcg(&fa.sm[sl * RP + r]);
                            lv[q] = __ldcg(&fa.sl[sl * RP + r]);
                            ov[q] = __ldcg(&fa.so[(static_cast<uint64_t>(sl) * RP + r) * D + dim]);
                        } else {
                            mv[q] = -INFINITY;
                            lv[q] = 0.0f;
                            ov[q] = 0.0f;
                        }
                    }
                    float Mb = M;
#pragma unroll
                    for (int q = 0; q < kMergeBatch; ++q) Mb = fmaxf(Mb, mv[q]);
                    const float f0 = exp_shift(M, Mb);
                    L *= f0;
                    O *= f0;
#pragma unroll
                    for (int q = 0; q < kMergeBatch; ++q) {
                        const float f = exp_shift(mv[q], Mb);
                        L += lv[q] * f;
                        O += ov[q] * f;
                    }
                    M = Mb;
                }
                if (has_cold) {
                    const float f = exp_shift(Mc, M);
                    L += lc * f;
                    O += oc * f;
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
            named_bar(kColdBar, 128);
            if (leader) stamp(fa, TR_MERGE_DONE);
        }
    } else {
        // =================== hot consumers (128 threads) ====================
        // Tensor-core attention per 16-token block (mma.sync m16n8k16, f16 in,
        // fp32 accumulate) in the FlashAttention-2 register layout: S^T = Q K^T
        // leaves row gid, tokens 2tig, 2tig+1 (+8) in each lane, which is the
        // A-operand layout of P for O += P V.  The first RP (<= 8) of the 16
        // rows are the group's query rows.
        const uint32_t ht = tid - 192, hw = ht >> 5;
        const uint32_t gid = lane >> 2, tig = lane & 3;
        constexpr int KS = D / 16;
        constexpr int NT = D / 8;
        uint32_t k = 0;
        for (uint32_t gi = g0; gi < g1; ++gi) {
            const FusedHotGroup gr = fa.groups[gi];
            const uint32_t b = gr.b, g = gr.g;
            const uint32_t np = gr.page_end - gr.page_begin;
            const uint32_t Th = (a.hot_indptr[b + 1] - a.hot_indptr[b]) * kBlock;
            // query fragments straight from global memory (rows >= R zero)
            uint32_t qf[KS][2];
            {
                const bool live = gid < R;
                const __half* qrow = q_row(a, b, g, live ? gid : 0);
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    qf[ks][0] = live ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * tig) : 0u;
                    qf[ks][1] = live ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * tig) : 0u;
                }
            }
            int32_t limit = static_cast<int32_t>(Th);
            if ((a.flags & 1u) && gid < R)
                limit = static_cast<int32_t>(Th) - static_cast<int32_t>(a.nq) + 1 + static_cast<int32_t>(gid / a.G);
            float m_run = -INFINITY, l_run = 0.0f;
            float o[NT][4];
#pragma unroll
            for (int j = 0; j < NT; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[j][e] = 0.0f;
            for (uint32_t i = hw; i < np; i += 4) {
                const uint32_t kk = k + i, s = kk % kHotStages;
                // warp-uniform and converged: ldmatrix / mma below are .sync.aligned
                if (!__all_sync(0xffffffffu, mbar_wait(&full_h[s], (kk / kHotStages) & 1, a.status))) break;
                const bool pvalid = hvalid[s] != 0;
                const uint8_t* Ks = hot + s * L::kHotStage;
                const uint8_t* Vs = Ks + L::kHotPage;
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
                    ldmatrix_x4(kb, Ks + (dch >> 3) * L::kHotBox + swz128(trow, dch & 7));
                    mma_16816(c[0], qf[ks][0], 0u, qf[ks][1], 0u, kb[0], kb[1]);
                    mma_16816(c[1], qf[ks][0], 0u, qf[ks][1], 0u, kb[2], kb[3]);
                }
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
                    __stcg(&fa.sm[gr.slot * RP + r], M);
                    __stcg(&fa.sl[gr.slot * RP + r], Ls);
                }
                __stcg(&fa.so[(static_cast<uint64_t>(gr.slot) * RP + r) * D + dim], O);
            }
            named_bar(kHotBar, 128);
            if (ht == 0) {
                __threadfence();
                atomicAdd(&cnt[CNT_HOT * B + b], 1u);
            }
        }
        if (ht == 0) stamp(fa, TR_HOT_DONE);
    }

    // ---- exit: the last CTA resets the dependency counters for the next step
    __syncthreads();
    if (tid == 0) {
        stamp(fa, TR_EXIT);
        __threadfence();
        const uint32_t done = atomicAdd(&cnt[CNT_KINDS * B], 1u);
        if (done == fa.n_ctas - 1) {
            for (uint32_t i = 0; i < CNT_KINDS * B + 1; ++i) cnt[i] = 0u;
            __threadfence();
        }
    }
}

size_t fused_smem_bytes(uint32_t D, uint32_t RP, uint32_t kv_heads) {
    if (kv_heads == 0 || 128 % kv_heads) return 0;
    if (kBlock * kv_heads * 16 > kCodeSlotBytes) return 0;
    size_t bytes = 0;
    if (D == 128) {
        switch (RP) {
            case 1: bytes = Layout<128, 1>::total; break;
            case 2: bytes = Layout<128, 2>::total; break;
            case 4: bytes = Layout<128, 4>::total; break;
            case 8: bytes = Layout<128, 8>::total; break;
            default: return 0;
        }
    } else if (D == 64) {
        switch (RP) {
            case 1: bytes = Layout<64, 1>::total; break;
            case 2: bytes = Layout<64, 2>::total; break;
            case 4: bytes = Layout<64, 4>::total; break;
            case 8: bytes = Layout<64, 8>::total; break;
            default: return 0;
        }
    } else {
        return 0;
    }
    bytes += 1024;  // alignment slack
    return bytes <= 227 * 1024 ? bytes : 0;
}

namespace {
template <int D, int RP>
cudaError_t occupancy_t(int* n) {
    const size_t smem = Layout<D, RP>::total + 1024;
    cudaError_t e = cudaFuncSetAttribute(fused_step_kernel<D, RP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(n, fused_step_kernel<D, RP>, kThreads, smem);
}

template <int D, int RP>
cudaError_t launch_fused_t(const FusedArgs& fa, const CUtensorMap& hk, const CUtensorMap& hv, const CUtensorMap& kd,
                           const CUtensorMap& vd, cudaStream_t s) {
    const size_t smem = Layout<D, RP>::total + 1024;
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(fused_step_kernel<D, RP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(fa.n_ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fused_step_kernel<D, RP>, hk, hv, kd, vd, fa);
}
}  // namespace

cudaError_t fused_occupancy(uint32_t D, uint32_t RP, int* n) {
    *n = 0;
    if (D == 128) {
        switch (RP) {
            case 1: return occupancy_t<128, 1>(n);
            case 2: return occupancy_t<128, 2>(n);
            case 4: return occupancy_t<128, 4>(n);
            case 8: return occupancy_t<128, 8>(n);
        }
    } else if (D == 64) {
        switch (RP) {
            case 1: return occupancy_t<64, 1>(n);
            case 2: return occupancy_t<64, 2>(n);
            case 4: return occupancy_t<64, 4>(n);
            case 8: return occupancy_t<64, 8>(n);
        }
    }
    return cudaSuccess;
}

cudaError_t launch_fused(const FusedArgs& fa, const CUtensorMap& hk, const CUtensorMap& hv, const CUtensorMap& kd,
                         const CUtensorMap& vd, cudaStream_t s) {
    const uint32_t D = fa.r.D, RP = fa.r.RP;
    if (D == 128) {
        switch (RP) {
            case 1: return launch_fused_t<128, 1>(fa, hk, hv, kd, vd, s);
            case 2: return launch_fused_t<128, 2>(fa, hk, hv, kd, vd, s);
            case 4: return launch_fused_t<128, 4>(fa, hk, hv, kd, vd, s);
            case 8: return launch_fused_t<128, 8>(fa, hk, hv, kd, vd, s);
        }
    } else if (D == 64) {
        switch (RP) {
            case 1: return launch_fused_t<64, 1>(fa, hk, hv, kd, vd, s);
            case 2: return launch_fused_t<64, 2>(fa, hk, hv, kd, vd, s);
            case 4: return launch_fused_t<64, 4>(fa, hk, hv, kd, vd, s);
            case 8: return launch_fused_t<64, 8>(fa, hk, hv, kd, vd, s);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace weaver
