// weaver_api.cu — C ABI (include/weaver_cuda.h): engine, plans, host-slice
// decode, model/fabric helpers.  All device memory a plan needs is allocated
// when the plan is created; weaver_run only encodes tensor maps and launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/weaver_cuda.h"
#include "weaver_internal.hpp"

using namespace weaver;

namespace {

thread_local std::string g_last_error = "no error";

int fail(int status, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(WEAVER_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define WEAVER_CUDA_TRY(expr, what)                 \
    do {                                            \
        cudaError_t e_ = (expr);                    \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D f16 tensor [rows][cols] with row pitch `pitch_elems`, 64-column x
// `box_rows` boxes, 128-byte swizzle.
int encode_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
              uint32_t box_rows, const char* what) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(WEAVER_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch_elems * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WEAVER_ERR_CUDA, "tensor map for %s failed (CUresult %d)", what, (int)r);
    return WEAVER_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

uint32_t round_rows(uint32_t R) {
    uint32_t p = 1;
    while (p < R) p <<= 1;
    return p;
}

struct DevBuf {
    void* ptr = nullptr;
    size_t cap = 0;
    ~DevBuf() {
        if (ptr) cudaFree(ptr);
    }
    // grow-only (weaver.rs:252-255)
    cudaError_t reserve(size_t bytes) {
        if (bytes <= cap && ptr) return cudaSuccess;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
        cudaError_t e = cudaMalloc(&ptr, bytes ? bytes : 16);
        if (e == cudaSuccess) cap = bytes;
        return e;
    }
};

}  // namespace

struct weaver_engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaDeviceProp prop{};
    // host-slice path (weaver.rs:40-55): persistent device copies
    DevBuf q, ql, hot, cold, refs, dict, out;
    weaver_plan* host_plan = nullptr;
    weaver_params host_params{};
    // host-buffer batched path: persistent device copies of every view
    DevBuf b_q, b_ql, b_hk, b_hv, b_hr, b_ck, b_cv, b_cr, b_kd, b_vd, b_out, b_pm, b_pl, b_po;
    weaver_plan* batch_plan = nullptr;
    weaver_shape batch_shape{};
    std::vector<uint32_t> batch_hip, batch_cip;
    // multi-query attention's split-KV partials (grow-only)
    DevBuf mha;
};

struct weaver_combine {
    weaver_engine* engine = nullptr;  // creation only: the object may outlive it
    int device = 0;
    uint32_t world = 0, rank = 0, rows = 0, D = 0;
    size_t recv_bytes = 0;            // offset of the flags in every rank's allocation
    size_t ll_off = 0;                // offset of the fused path's (value, tag) receive region
    size_t ll_state_off = 0;          // offset of the fused path's [step tag, status]
    uint8_t* base = nullptr;          // own allocation
    uint8_t* peer[kCombineMaxRanks] = {};
    bool opened[kCombineMaxRanks] = {};
    cudaStream_t last_stream = nullptr;
};

struct weaver_plan {
    weaver_engine* engine = nullptr;  // creation only: the plan may outlive it
    int device = 0;
    weaver_shape shape{};
    RunArgs base{};
    void* arena = nullptr;
    // fused single-kernel step (used when the geometry qualifies)
    bool fused = false;
    FusedArgs fargs{};
    void* farena = nullptr;
    // head-partitioned single-kernel step (preferred when it qualifies)
    bool hp = false;
    HpArgs hargs{};
    void* harena = nullptr;
    uint32_t row_groups = 1;
    uint32_t contract_splits = 1;  // atom splits of the tensor-core contraction
    cudaStream_t side = nullptr;   // the multi-kernel step's hot pass (forked from the run's stream)
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    uint32_t n_hot_pages = 0;
    uint32_t n_cold_pages = 0;
    cudaStream_t last_stream = nullptr;
    weaver_combine* combine = nullptr;  // split-KV merge fused into the step (weaver_plan_attach_combine)
};

// Hot page-heads (one 16-token block of one kv head) in (b, g, page) order,
// cut into per-CTA runs so that every CTA's hot bytes top its cold bytes up to
// an equal share of the step.  Slots are numbered in (b, g, page) order, so
// the slots of one (b, g) form one contiguous range.
struct HotCut {
    std::vector<std::vector<FusedHotGroup>> glists;  // [P]
    std::vector<uint32_t> slot_ptr;                  // [B*Hkv + 1]
    std::vector<uint32_t> groups_of;                 // [B*Hkv]
    uint32_t n_slots = 0;
};

static HotCut cut_hot_groups(uint32_t B, uint32_t Hkv, uint32_t P, const uint32_t* hot_indptr,
                             const std::vector<double>& cold_bytes, double page_head_bytes) {
    HotCut hc;
    hc.glists.resize(P);
    hc.slot_ptr.assign(static_cast<size_t>(B) * Hkv + 1, 0);
    hc.groups_of.assign(static_cast<size_t>(B) * Hkv, 0);
    uint64_t n_ph = 0;
    for (uint32_t b = 0; b < B; ++b) n_ph += static_cast<uint64_t>(hot_indptr[b + 1] - hot_indptr[b]) * Hkv;
    double cold_total = 0.0;
    for (double c : cold_bytes) cold_total += c;
    const double target = (cold_total + n_ph * page_head_bytes) / P;
    std::vector<double> quota(P);
    double qsum = 0.0;
    for (uint32_t c = 0; c < P; ++c) {
        quota[c] = std::max(0.0, target - cold_bytes[c]);
        qsum += quota[c];
    }
    std::vector<uint64_t> cut(P + 1, 0);
    double acc = 0.0;
    for (uint32_t c = 0; c < P; ++c) {
        acc += quota[c];
        cut[c + 1] = qsum > 0 ? static_cast<uint64_t>(std::llround(acc / qsum * static_cast<double>(n_ph))) : n_ph;
    }
    cut[P] = n_ph;
    uint64_t x = 0;  // index into the (b, g, page) sequence
    uint32_t c = 0;
    for (uint32_t b = 0; b < B; ++b) {
        const uint32_t h0 = hot_indptr[b], h1 = hot_indptr[b + 1];
        for (uint32_t g = 0; g < Hkv; ++g) {
            const size_t bg = static_cast<size_t>(b) * Hkv + g;
            hc.slot_ptr[bg] = hc.n_slots;
            uint32_t p = h0;
            while (p < h1) {
                while (c < P && x >= cut[c + 1]) ++c;
                const uint64_t room = (c < P) ? cut[c + 1] - x : (h1 - p);
                const uint32_t take = static_cast<uint32_t>(std::min<uint64_t>(room, h1 - p));
                const uint32_t cc = std::min(c, P - 1);
                hc.glists[cc].push_back(FusedHotGroup{b, g, p, p + take, (p - h0) * kBlock, hc.n_slots});
                ++hc.groups_of[bg];
                ++hc.n_slots;
                p += take;
                x += take;
            }
        }
    }
    hc.slot_ptr[static_cast<size_t>(B) * Hkv] = hc.n_slots;
    return hc;
}

// Builds the fused single-kernel schedule for `plan` when its geometry
// qualifies (R <= 8 query rows per kv head, kv_heads dividing 128, model
// semantics); otherwise leaves plan->fused false and the multi-kernel path runs.
static int build_fused_plan(weaver_plan* plan, const uint32_t* hot_indptr, const uint32_t* cold_indptr) {
    const weaver_shape& sh = plan->shape;
    const RunArgs& a = plan->base;
    if (sh.flags & WEAVER_FLAG_QLATENT_INPUT) return WEAVER_OK;
    if (a.R > 8) return WEAVER_OK;
    const size_t smem = fused_smem_bytes(a.D, a.RP, a.Hkv);
    if (smem == 0) return WEAVER_OK;
    weaver_engine* eng = plan->engine;
    const uint32_t P = static_cast<uint32_t>(eng->prop.multiProcessorCount);
    const uint32_t B = a.B, Hkv = a.Hkv, D = a.D, RP = a.RP;
    const uint32_t code_pages = std::min<uint32_t>(32u, std::max<uint32_t>(1u, 8192u / (kBlock * Hkv * 16u)));
    const double dict_tile_bytes = (D / 64) * 128.0 * 128.0;
    const double page_code_bytes = kBlock * Hkv * 16.0;
    const double page_head_bytes = 2.0 * kBlock * D * 2.0;

    std::vector<std::vector<FusedItem>> lists(P);
    std::vector<double> cold_bytes(P, 0.0);
    std::vector<uint32_t> code_items(B, 0);
    uint32_t rr = 0;
    auto put = [&](const FusedItem& it, double bytes) {
        lists[rr % P].push_back(it);
        cold_bytes[rr % P] += bytes;
        ++rr;
    };
    // phase-major so every CTA's list is ordered q_latent, score, scatter, contract
    for (int phase = 0; phase < 4; ++phase) {
        for (uint32_t b = 0; b < B; ++b) {
            const uint32_t c0 = cold_indptr[b], c1 = cold_indptr[b + 1];
            if (c1 == c0) continue;
            if (phase == FI_QLAT || phase == FI_CONTRACT) {
                for (uint32_t g = 0; g < Hkv; ++g)
                    for (uint32_t t = 0; t < a.n_atom_tiles; ++t)
                        put(FusedItem{static_cast<uint16_t>(phase), static_cast<uint16_t>(g), b, t, 0}, dict_tile_bytes);
            } else {
                uint32_t n_items = 0;
                for (uint32_t p = c0; p < c1; p += code_pages, ++n_items) {
                    const uint32_t n = std::min(code_pages, c1 - p);
                    put(FusedItem{static_cast<uint16_t>(phase), 0, b, p, n}, n * page_code_bytes);
                }
                code_items[b] = n_items;
            }
        }
    }
    // hot page-heads in (b, g, page) order, cut into per-CTA runs by byte quota
    HotCut hc = cut_hot_groups(B, Hkv, P, hot_indptr, cold_bytes, page_head_bytes);
    std::vector<std::vector<FusedHotGroup>>& glists = hc.glists;
    std::vector<uint32_t> hot_groups(B, 0);
    for (uint32_t b = 0; b < B; ++b)
        for (uint32_t g = 0; g < Hkv; ++g) hot_groups[b] += hc.groups_of[static_cast<size_t>(b) * Hkv + g];
    const uint32_t n_slots = hc.n_slots;
    const uint32_t rows = B * a.nq * a.Hq;
    std::vector<std::vector<uint32_t>> mlists(P);
    for (uint32_t r = 0; r < rows; ++r) mlists[(P - 1 - (r % P))].push_back(r);

    // flatten
    std::vector<FusedItem> items;
    std::vector<uint32_t> item_ptr(P + 1, 0), group_ptr(P + 1, 0), merge_ptr(P + 1, 0);
    std::vector<FusedHotGroup> groups;
    std::vector<uint32_t> merge_rows, slot_ptr = hc.slot_ptr, slot_ids(n_slots);
    for (uint32_t i = 0; i < n_slots; ++i) slot_ids[i] = i;
    for (uint32_t c = 0; c < P; ++c) {
        item_ptr[c] = static_cast<uint32_t>(items.size());
        items.insert(items.end(), lists[c].begin(), lists[c].end());
        group_ptr[c] = static_cast<uint32_t>(groups.size());
        groups.insert(groups.end(), glists[c].begin(), glists[c].end());
        merge_ptr[c] = static_cast<uint32_t>(merge_rows.size());
        merge_rows.insert(merge_rows.end(), mlists[c].begin(), mlists[c].end());
    }
    item_ptr[P] = static_cast<uint32_t>(items.size());
    group_ptr[P] = static_cast<uint32_t>(groups.size());
    merge_ptr[P] = static_cast<uint32_t>(merge_rows.size());

    // device arena: tables + fused scratch
    struct Piece { size_t bytes; size_t raw; size_t off; const void* src; };
    std::vector<Piece> pc;
    auto add = [&](size_t bytes, const void* src) {
        pc.push_back({align_up(std::max<size_t>(bytes, 16), 256), bytes, 0, src});
        return pc.size() - 1;
    };
    const size_t p_items = add(sizeof(FusedItem) * items.size(), items.data());
    const size_t p_iptr = add(sizeof(uint32_t) * item_ptr.size(), item_ptr.data());
    const size_t p_groups = add(sizeof(FusedHotGroup) * groups.size(), groups.data());
    const size_t p_gptr = add(sizeof(uint32_t) * group_ptr.size(), group_ptr.data());
    const size_t p_mrows = add(sizeof(uint32_t) * merge_rows.size(), merge_rows.data());
    const size_t p_mptr = add(sizeof(uint32_t) * merge_ptr.size(), merge_ptr.data());
    const size_t p_sptr = add(sizeof(uint32_t) * slot_ptr.size(), slot_ptr.data());
    const size_t p_sids = add(sizeof(uint32_t) * slot_ids.size(), slot_ids.data());
    const size_t p_citems = add(sizeof(uint32_t) * B, code_items.data());
    const size_t p_hgroups = add(sizeof(uint32_t) * B, hot_groups.data());
    const size_t p_cnt = add(sizeof(uint32_t) * (CNT_KINDS * B + 1), nullptr);
    const size_t p_mkey = add(sizeof(int) * B * Hkv * RP, nullptr);
    const size_t p_lcold = add(sizeof(float) * B * Hkv * RP, nullptr);
    const size_t p_ocold = add(sizeof(float) * B * Hkv * RP * D, nullptr);
    const size_t p_sm = add(sizeof(float) * std::max<uint32_t>(n_slots, 1) * RP, nullptr);
    const size_t p_sl = add(sizeof(float) * std::max<uint32_t>(n_slots, 1) * RP, nullptr);
    const size_t p_so = add(sizeof(float) * std::max<uint32_t>(n_slots, 1) * RP * D, nullptr);
    const char* tr = getenv("WEAVER_TRACE");
    const bool tracing = tr && tr[0] == '1';
    const size_t p_trace = add(tracing ? sizeof(uint64_t) * P * kTraceSlots : 16, nullptr);
    size_t total = 0;
    for (auto& q : pc) { q.off = total; total += q.bytes; }
    cudaError_t e = cudaMalloc(&plan->farena, total);
    if (e != cudaSuccess) return cuda_fail(e, "fused plan allocation");
    uint8_t* base = static_cast<uint8_t*>(plan->farena);
    cudaStream_t s = eng->stream;
    for (auto& q : pc) {
        if (q.src && q.raw) e = cudaMemcpyAsync(base + q.off, q.src, q.raw, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "fused plan upload");
    }
    e = cudaMemsetAsync(base + pc[p_cnt].off, 0, pc[p_cnt].bytes, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "fused plan upload");
    int per_sm = 0;
    e = fused_occupancy(D, RP, &per_sm);
    if (e != cudaSuccess) return cuda_fail(e, "fused occupancy query");
    if (per_sm < 1) return WEAVER_OK;  // cannot be resident: keep the multi-kernel path
    auto P32 = [&](size_t i) { return reinterpret_cast<uint32_t*>(base + pc[i].off); };
    FusedArgs& f = plan->fargs;
    f.code_pages = code_pages;
    f.n_ctas = P;
    f.items = reinterpret_cast<const FusedItem*>(base + pc[p_items].off);
    f.item_ptr = P32(p_iptr);
    f.groups = reinterpret_cast<const FusedHotGroup*>(base + pc[p_groups].off);
    f.group_ptr = P32(p_gptr);
    f.merge_rows = P32(p_mrows);
    f.merge_ptr = P32(p_mptr);
    f.slot_ptr = P32(p_sptr);
    f.slot_ids = P32(p_sids);
    f.code_items = P32(p_citems);
    f.hot_groups = P32(p_hgroups);
    f.counters = P32(p_cnt);
    f.mkey = reinterpret_cast<int*>(base + pc[p_mkey].off);
    f.lcold = reinterpret_cast<float*>(base + pc[p_lcold].off);
    f.ocold = reinterpret_cast<float*>(base + pc[p_ocold].off);
    f.sm = reinterpret_cast<float*>(base + pc[p_sm].off);
    f.sl = reinterpret_cast<float*>(base + pc[p_sl].off);
    f.so = reinterpret_cast<float*>(base + pc[p_so].off);
    f.trace = tracing ? reinterpret_cast<uint64_t*>(base + pc[p_trace].off) : nullptr;
    plan->fused = true;
    return WEAVER_OK;
}

// Builds the head-partitioned single-kernel schedule when the geometry
// qualifies: model semantics, RP <= 4 query rows per kv head, one kv head's f16
// q_latent within 32 KB, head_dim 64 or 128, and cold blocks that split into
// at most one chunk (<= 128 blocks of one (sequence, kv head)) per SM.
// Otherwise leaves plan->hp false and the next path is tried.
static int build_hp_plan(weaver_plan* plan, const uint32_t* hot_indptr, const uint32_t* cold_indptr) {
    const weaver_shape& sh = plan->shape;
    const RunArgs& a = plan->base;
    if (sh.flags & WEAVER_FLAG_QLATENT_INPUT) return WEAVER_OK;
    if (a.RP > 4 || (a.D != 64 && a.D != 128)) return WEAVER_OK;
    const uint64_t ql_bytes = static_cast<uint64_t>(a.A) * a.RP * 2;
    if (ql_bytes > kHpQlatBytes || ql_bytes % 16) return WEAVER_OK;
    if (hp_smem_bytes(a.D, a.RP) == 0) return WEAVER_OK;
    weaver_engine* eng = plan->engine;
    const uint32_t P = static_cast<uint32_t>(eng->prop.multiProcessorCount);
    const uint32_t B = a.B, Hkv = a.Hkv, D = a.D, RP = a.RP, A = a.A, NT = a.n_atom_tiles;
    const uint32_t NB = B * Hkv;
    auto chunks_for = [&](uint32_t cap) {
        uint64_t n = 0;
        for (uint32_t b = 0; b < B; ++b) n += static_cast<uint64_t>(Hkv) * ((cold_indptr[b + 1] - cold_indptr[b] + cap - 1) / cap);
        return n;
    };
    if (chunks_for(kHpMaxChunkPages) > P) return WEAVER_OK;
    uint32_t lo = 1, hi = kHpMaxChunkPages;  // smallest cap whose chunks all get a CTA
    while (lo < hi) {
        const uint32_t mid = (lo + hi) / 2;
        if (chunks_for(mid) <= P) hi = mid;
        else lo = mid + 1;
    }
    const uint32_t cap = lo;
    const double dict_tile_bytes = (D / 64) * 128.0 * 128.0;
    const double page_head_bytes = 2.0 * kBlock * D * 2.0;

    // cold chunks: chunk c -> CTA c; equal-sized runs within a (b, g)
    std::vector<HpChunk> chunks(P, HpChunk{0, 0, 0, 0});
    std::vector<uint32_t> n_chunks(NB, 0);
    std::vector<double> cold_bytes(P, 0.0);
    uint32_t nc = 0;
    for (uint32_t b = 0; b < B; ++b) {
        const uint32_t c0 = cold_indptr[b], n = cold_indptr[b + 1] - c0;
        if (!n) continue;
        const uint32_t k = (n + cap - 1) / cap;
        for (uint32_t g = 0; g < Hkv; ++g) {
            for (uint32_t j = 0; j < k; ++j) {
                const uint32_t p0 = c0 + static_cast<uint32_t>(static_cast<uint64_t>(n) * j / k);
                const uint32_t p1 = c0 + static_cast<uint32_t>(static_cast<uint64_t>(n) * (j + 1) / k);
                chunks[nc] = HpChunk{b, g, p0, p1 - p0};
                cold_bytes[nc] += (p1 - p0) * kBlock * 16.0 * 2.0;
                ++nc;
            }
            n_chunks[b * Hkv + g] = k;
        }
    }
    // q_latent tiles round-robin over all CTAs; a head's contraction tiles on
    // the CTAs that hold its chunks (their one wait is on that head's scatter)
    std::vector<std::vector<FusedItem>> lists(P);
    std::vector<uint32_t> chunk_base(NB, 0);
    {
        uint32_t c = 0;
        for (uint32_t bg = 0; bg < NB; ++bg) {
            chunk_base[bg] = c;
            c += n_chunks[bg];
        }
    }
    uint32_t rr = 0;
    for (uint32_t b = 0; b < B; ++b) {
        if (cold_indptr[b + 1] == cold_indptr[b]) continue;
        for (uint32_t g = 0; g < Hkv; ++g)
            for (uint32_t t = 0; t < NT; ++t) {
                lists[rr % P].push_back(FusedItem{FI_QLAT, static_cast<uint16_t>(g), b, t, 0});
                cold_bytes[rr % P] += dict_tile_bytes;
                ++rr;
            }
    }
    for (uint32_t b = 0; b < B; ++b) {
        if (cold_indptr[b + 1] == cold_indptr[b]) continue;
        for (uint32_t g = 0; g < Hkv; ++g) {
            const uint32_t bg = b * Hkv + g;
            for (uint32_t t = 0; t < NT; ++t) {
                const uint32_t c = chunk_base[bg] + t % n_chunks[bg];
                lists[c].push_back(FusedItem{FI_CONTRACT, static_cast<uint16_t>(g), b, t, 0});
                cold_bytes[c] += dict_tile_bytes;
            }
        }
    }
    HotCut hc = cut_hot_groups(B, Hkv, P, hot_indptr, cold_bytes, page_head_bytes);
    for (uint32_t bg = 0; bg < NB; ++bg)
        if (hc.groups_of[bg] > kHpMaxSlots) return WEAVER_OK;  // the merge's shared scratch holds 64 slots
    std::vector<uint32_t> empty_bg;
    for (uint32_t bg = 0; bg < NB; ++bg)
        if (!n_chunks[bg] && !hc.groups_of[bg]) empty_bg.push_back(bg);

    std::vector<FusedItem> items;
    std::vector<FusedHotGroup> groups;
    std::vector<uint32_t> item_ptr(P + 1, 0), group_ptr(P + 1, 0);
    for (uint32_t c = 0; c < P; ++c) {
        item_ptr[c] = static_cast<uint32_t>(items.size());
        items.insert(items.end(), lists[c].begin(), lists[c].end());
        group_ptr[c] = static_cast<uint32_t>(groups.size());
        groups.insert(groups.end(), hc.glists[c].begin(), hc.glists[c].end());
    }
    item_ptr[P] = static_cast<uint32_t>(items.size());
    group_ptr[P] = static_cast<uint32_t>(groups.size());
    std::vector<FusedItem> first_item(P, FusedItem{0xFFFF, 0, 0, 0, 0});
    for (uint32_t c = 0; c < P; ++c)
        if (item_ptr[c + 1] > item_ptr[c]) first_item[c] = items[item_ptr[c]];

    struct Piece { size_t bytes; size_t raw; size_t off; const void* src; };
    std::vector<Piece> pc;
    auto add = [&](size_t bytes, const void* src) {
        pc.push_back({align_up(std::max<size_t>(bytes, 16), 256), bytes, 0, src});
        return pc.size() - 1;
    };
    const size_t n_slots = std::max<size_t>(hc.n_slots, 1);
    const size_t p_items = add(sizeof(FusedItem) * items.size(), items.data());
    const size_t p_iptr = add(sizeof(uint32_t) * item_ptr.size(), item_ptr.data());
    const size_t p_first = add(sizeof(FusedItem) * first_item.size(), first_item.data());
    const size_t p_chunks = add(sizeof(HpChunk) * chunks.size(), chunks.data());
    const size_t p_groups = add(sizeof(FusedHotGroup) * groups.size(), groups.data());
    const size_t p_gptr = add(sizeof(uint32_t) * group_ptr.size(), group_ptr.data());
    const size_t p_sptr = add(sizeof(uint32_t) * hc.slot_ptr.size(), hc.slot_ptr.data());
    const size_t p_nch = add(sizeof(uint32_t) * NB, n_chunks.data());
    const size_t p_hg = add(sizeof(uint32_t) * NB, hc.groups_of.data());
    const size_t p_empty = add(sizeof(uint32_t) * empty_bg.size(), empty_bg.data());
    const size_t p_cnt = add(sizeof(uint32_t) * (HC_KINDS * NB + 1), nullptr);
    const size_t p_ql = add(static_cast<size_t>(NB) * A * RP * 2, nullptr);
    const size_t p_w = add(sizeof(float) * NB * (static_cast<size_t>(A) * RP + 4), nullptr);
    const size_t p_mkey = add(sizeof(int) * NB * RP, nullptr);
    const size_t p_oc = add(sizeof(float) * NB * RP * D, nullptr);
    const size_t p_sm = add(sizeof(float) * n_slots * RP, nullptr);
    const size_t p_sl = add(sizeof(float) * n_slots * RP, nullptr);
    const size_t p_so = add(sizeof(float) * n_slots * RP * D, nullptr);
    const char* tr = getenv("WEAVER_TRACE");
    const bool tracing = tr && tr[0] == '1';
    const size_t p_trace = add(tracing ? sizeof(uint64_t) * P * kTraceSlots : 16, nullptr);
    size_t total = 0;
    for (auto& q : pc) { q.off = total; total += q.bytes; }
    int per_sm = 0;
    cudaError_t e = hp_occupancy(D, RP, &per_sm);
    if (e != cudaSuccess) return cuda_fail(e, "head-partitioned occupancy query");
    if (per_sm < 1) return WEAVER_OK;
    e = cudaMalloc(&plan->harena, total);
    if (e != cudaSuccess) return cuda_fail(e, "head-partitioned plan allocation");
    uint8_t* base = static_cast<uint8_t*>(plan->harena);
    cudaStream_t s = eng->stream;
    for (auto& q : pc) {
        if (q.src && q.raw) e = cudaMemcpyAsync(base + q.off, q.src, q.raw, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return cuda_fail(e, "head-partitioned plan upload");
    }
    e = cudaMemsetAsync(base + pc[p_cnt].off, 0, pc[p_cnt].bytes, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "head-partitioned plan upload");
    auto U32 = [&](size_t i) { return reinterpret_cast<uint32_t*>(base + pc[i].off); };
    auto F32 = [&](size_t i) { return reinterpret_cast<float*>(base + pc[i].off); };
    HpArgs& h = plan->hargs;
    h.n_ctas = P;
    h.n_empty = static_cast<uint32_t>(empty_bg.size());
    h.items = reinterpret_cast<const FusedItem*>(base + pc[p_items].off);
    h.item_ptr = U32(p_iptr);
    h.first_item = reinterpret_cast<const FusedItem*>(base + pc[p_first].off);
    h.chunks = reinterpret_cast<const HpChunk*>(base + pc[p_chunks].off);
    h.groups = reinterpret_cast<const FusedHotGroup*>(base + pc[p_groups].off);
    h.group_ptr = U32(p_gptr);
    h.slot_ptr = U32(p_sptr);
    h.n_chunks = U32(p_nch);
    h.hot_groups = U32(p_hg);
    h.empty_bg = U32(p_empty);
    h.counters = U32(p_cnt);
    h.qlat16 = reinterpret_cast<__half*>(base + pc[p_ql].off);
    h.wsum = F32(p_w);
    h.mkey = reinterpret_cast<int*>(base + pc[p_mkey].off);
    h.ocold = F32(p_oc);
    h.sm = F32(p_sm);
    h.sl = F32(p_sl);
    h.so = F32(p_so);
    h.trace = tracing ? reinterpret_cast<uint64_t*>(base + pc[p_trace].off) : nullptr;
    plan->hp = true;
    return WEAVER_OK;
}

// 2-D u16 view of a SparseCode pool [blocks][16][Hkv] as rows of tokens with
// Hkv x 8 u16 each; boxes of 16 tokens x one head's 16 bytes, no swizzle.
int encode_codes(CUtensorMap* map, const void* base, uint64_t pool_blocks, uint64_t Hkv, const char* what) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(WEAVER_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[2] = {Hkv * 8, pool_blocks * kBlock};
    cuuint64_t strides[1] = {Hkv * 16};
    cuuint32_t box[2] = {8, kBlock};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(WEAVER_ERR_CUDA, "tensor map for %s failed (CUresult %d)", what, (int)r);
    return WEAVER_OK;
}

extern "C" {

int weaver_abi_version(void) { return WEAVER_ABI_VERSION; }

const char* weaver_last_error(void) { return g_last_error.c_str(); }

const char* weaver_status_string(int s) {
    switch (s) {
        case WEAVER_OK: return "ok";
        case WEAVER_ERR_INVALID_ARGUMENT: return "invalid argument";
        case WEAVER_ERR_UNSUPPORTED: return "unsupported geometry";
        case WEAVER_ERR_MISALIGNED: return "misaligned device view";
        case WEAVER_ERR_OUT_OF_RANGE: return "block reference or atom index out of range";
        case WEAVER_ERR_CUDA: return "CUDA error";
        case WEAVER_ERR_NO_DEVICE: return "no sm_100 CUDA device";
        case WEAVER_ERR_TIMEOUT: return "device wait timed out";
        case WEAVER_ERR_CAPACITY: return "capacity exceeded";
        default: return "unknown status";
    }
}

// ---- ModelDims / WeaverParams / FabricRegions ----------------------------

int weaver_model_dims_preset(const char* name, weaver_model_dims* out) {
    if (!name || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    // trait defaults (types.rs:150-164): Llama-3.1-8B
    weaver_model_dims d{32, 32, 8, 128, 32 * 128, 14336, 128256, 16, 4, 512, 0};
    if (!strcmp(name, "llama8b")) {
    } else if (!strcmp(name, "granite2b")) {  // types.rs:171-181
        d.layers = 40; d.q_heads = 32; d.kv_heads = 8; d.head_dim = 64;
        d.hidden_size = 2048; d.intermediate_size = 8192; d.vocab_size = 49155;
    } else if (!strcmp(name, "qwen05b")) {  // types.rs:183-193
        d.layers = 24; d.q_heads = 14; d.kv_heads = 2; d.head_dim = 64;
        d.hidden_size = 896; d.intermediate_size = 4864; d.vocab_size = 151936;
    } else if (!strcmp(name, "deepseek_r1_1_5b")) {  // types.rs:195-204
        d.layers = 28; d.q_heads = 12; d.kv_heads = 2; d.head_dim = 128;
        d.hidden_size = 1536; d.intermediate_size = 8960; d.vocab_size = 151936;
    } else {
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "unknown ModelDims preset '%s'", name);
    }
    d.gqa_group = d.q_heads / d.kv_heads;
    *out = d;
    return WEAVER_OK;
}

int weaver_params_from_loom(const weaver_model_dims* d, const weaver_loom_descriptor* loom, weaver_params* out) {
    if (!d || !loom || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    weaver_params p{};
    p.q_heads = d->q_heads;
    p.kv_heads = d->kv_heads;
    p.head_dim = d->head_dim;
    p.block_size = d->block_size;
    p.gqa_group = d->gqa_group;
    p.hot_count = loom->hot_count;
    p.cold_count = loom->cold_count;
    p.dict_size = d->dict_size;
    p.sparsity_k = d->sparsity_k;
    *out = p;
    return WEAVER_OK;
}

int weaver_fabric_regions_compute(const weaver_model_dims* d, weaver_fabric_regions* out) {
    if (!d || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    const uint64_t header = 9 + 4 + 64;  // magic "AETHER1.3" + version + signature (types.rs:486)
    const uint64_t h = d->hidden_size, inter = d->intermediate_size, vocab = d->vocab_size;
    const uint64_t kv = d->kv_heads, q = d->q_heads, hd = d->head_dim;
    const uint64_t per_layer =
        2 * (q * hd * h + kv * hd * h + kv * hd * h + q * hd * h + h * inter + h * inter + inter * h + h + h);
    const uint64_t global = 2 * (vocab * h + h);
    const uint64_t raw = d->layers * per_layer + global;
    const uint64_t est = static_cast<uint64_t>(static_cast<double>(raw) * 1.25);
    const uint64_t max_hot = 8192, max_cold = 32768;  // FabricLayout (types.rs:500-503)
    weaver_fabric_regions r{};
    r.weights_offset = align_up(header, 16384);
    r.weights_size = align_up(est, 16384);
    r.hot_pool_offset = align_up(r.weights_offset + r.weights_size, 16384);
    r.hot_pool_size = max_hot * d->block_size * kv * hd * 2;
    r.cold_pool_offset = align_up(r.hot_pool_offset + r.hot_pool_size, 16384);
    r.cold_pool_size = max_cold * d->block_size * kv * sizeof(weaver_sparse_code);
    r.dict_offset = align_up(r.cold_pool_offset + r.cold_pool_size, 16384);
    r.dict_size = kv * d->dict_size * hd * 2;
    r.looms_offset = align_up(r.dict_offset + r.dict_size, 4096);
    r.looms_size = 4 * sizeof(weaver_loom_descriptor);
    r.radix_offset = align_up(r.looms_offset + r.looms_size, 4096);
    r.radix_size = (max_hot + max_cold) * 3 * 4;
    r.obs_offset = align_up(r.radix_offset + r.radix_size, 16384);
    r.obs_size = 256ull * 1024 * 1024;
    r.trace_offset = align_up(r.obs_offset + r.obs_size, 16384);
    r.trace_size = 128ull * 1024 * 1024;
    r.total_size = align_up(r.trace_offset + r.trace_size + 64, 16384);
    *out = r;
    return WEAVER_OK;
}

// ---- engine ----------------------------------------------------------------

int weaver_engine_create(int device, weaver_engine** out) {
    if (!out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return fail(WEAVER_ERR_NO_DEVICE, "no CUDA device (%s)", cudaGetErrorString(e));
    if (device < 0 || device >= n) return fail(WEAVER_ERR_NO_DEVICE, "device %d out of range (%d devices)", device, n);
    weaver_engine* eng = new weaver_engine();
    eng->device = device;
    if ((e = cudaSetDevice(device)) != cudaSuccess || (e = cudaGetDeviceProperties(&eng->prop, device)) != cudaSuccess) {
        delete eng;
        return cuda_fail(e, "cudaSetDevice");
    }
    if (eng->prop.major != 10) {
        const int cc = eng->prop.major * 10 + eng->prop.minor;
        delete eng;
        return fail(WEAVER_ERR_NO_DEVICE, "device %d is sm_%d; this library is built for sm_100a", device, cc);
    }
    if ((e = cudaStreamCreateWithFlags(&eng->stream, cudaStreamNonBlocking)) != cudaSuccess) {
        delete eng;
        return cuda_fail(e, "cudaStreamCreate");
    }
    *out = eng;
    return WEAVER_OK;
}

void weaver_engine_destroy(weaver_engine* eng) {
    if (!eng) return;
    cudaSetDevice(eng->device);
    if (eng->host_plan) weaver_plan_destroy(eng->host_plan);
    if (eng->batch_plan) weaver_plan_destroy(eng->batch_plan);
    if (eng->stream) {
        cudaStreamSynchronize(eng->stream);
        cudaStreamDestroy(eng->stream);
    }
    delete eng;
}

int weaver_engine_device_name(const weaver_engine* eng, char* buf, size_t len) {
    if (!eng || !buf || len == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    snprintf(buf, len, "%s", eng->prop.name);
    return WEAVER_OK;
}

int weaver_engine_max_threads_per_block(const weaver_engine* eng, uint64_t* out) {
    if (!eng || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    *out = static_cast<uint64_t>(eng->prop.maxThreadsPerBlock);
    return WEAVER_OK;
}

// ---- plans -------------------------------------------------------------------

int weaver_plan_create(weaver_engine* eng, const weaver_shape* sh, const uint32_t* hot_indptr,
                       const uint32_t* cold_indptr, weaver_plan** out) {
    if (!eng || !sh || !hot_indptr || !cold_indptr || !out)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument to weaver_plan_create");
    *out = nullptr;
    const uint32_t B = sh->num_seqs, nq = sh->num_queries, Hq = sh->q_heads, Hkv = sh->kv_heads;
    const uint32_t D = sh->head_dim, A = sh->dict_size;
    if (B == 0 || nq == 0 || Hq == 0 || Hkv == 0 || A == 0)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "zero dimension in shape");
    if (Hq % Hkv) return fail(WEAVER_ERR_INVALID_ARGUMENT, "q_heads %u not a multiple of kv_heads %u", Hq, Hkv);
    if (D != 64 && D != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u (built for 64 and 128)", D);
    if (A > 65536) return fail(WEAVER_ERR_UNSUPPORTED, "dict_size %u exceeds u16 atom indices", A);
    const uint32_t G = Hq / Hkv, R = nq * G;
    if (R > 64) return fail(WEAVER_ERR_UNSUPPORTED, "num_queries*gqa_group = %u > 64", R);
    for (uint32_t b = 0; b < B; ++b)
        if (hot_indptr[b + 1] < hot_indptr[b] || cold_indptr[b + 1] < cold_indptr[b])
            return fail(WEAVER_ERR_INVALID_ARGUMENT, "indptr not monotone at sequence %u", b);
    if ((sh->flags & WEAVER_FLAG_CAUSAL) && nq > 1)
        for (uint32_t b = 0; b < B; ++b)
            if ((hot_indptr[b + 1] - hot_indptr[b]) * kBlock + 1 < nq)
                return fail(WEAVER_ERR_INVALID_ARGUMENT, "sequence %u has fewer hot tokens than queries", b);

    WEAVER_CUDA_TRY(cudaSetDevice(eng->device), "cudaSetDevice");
    const uint32_t RP = round_rows(R);
    const uint32_t RM = R >= kHotRows ? kHotRows : RP;
    const uint32_t rgroups = (R + RM - 1) / RM;
    const uint32_t n_tiles = (A + kAtomTile - 1) / kAtomTile;
    const uint32_t hot_pages = hot_indptr[B] - hot_indptr[0];
    const uint32_t cold_pages = cold_indptr[B] - cold_indptr[0];
    if (hot_indptr[0] != 0 || cold_indptr[0] != 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "indptr[0] must be 0");

    // hot items: enough CTAs for ~2 waves of resident hot CTAs over the GPU
    const uint64_t target = 2ull * eng->prop.multiProcessorCount;
    const uint64_t work = static_cast<uint64_t>(hot_pages) * Hkv * rgroups;
    uint32_t chunk = static_cast<uint32_t>(std::max<uint64_t>(2, (work + target - 1) / std::max<uint64_t>(target, 1)));
    std::vector<HotItem> hot_items;
    std::vector<uint32_t> hot_item_ptr(B + 1, 0);
    for (uint32_t b = 0; b < B; ++b) {
        hot_item_ptr[b] = static_cast<uint32_t>(hot_items.size());
        for (uint32_t p = hot_indptr[b]; p < hot_indptr[b + 1]; p += chunk) {
            HotItem it{b, p, std::min(p + chunk, hot_indptr[b + 1]), (p - hot_indptr[b]) * kBlock};
            hot_items.push_back(it);
        }
    }
    hot_item_ptr[B] = static_cast<uint32_t>(hot_items.size());
    std::vector<ColdItem> cold_items;
    std::vector<uint32_t> cold_item_ptr(B + 1, 0);
    for (uint32_t b = 0; b < B; ++b) {
        cold_item_ptr[b] = static_cast<uint32_t>(cold_items.size());
        for (uint32_t p = cold_indptr[b]; p < cold_indptr[b + 1]; p += kColdItemPages) {
            ColdItem it{b, p, std::min(p + kColdItemPages, cold_indptr[b + 1]), 0};
            cold_items.push_back(it);
        }
    }
    cold_item_ptr[B] = static_cast<uint32_t>(cold_items.size());
    if (hot_items.size() > 0x7FFFFFFF || cold_items.size() > 0x7FFFFFFF)
        return fail(WEAVER_ERR_CAPACITY, "too many work items");
    // chunks for the shared-memory cold passes: runs of one sequence's items,
    // as few items per chunk as keeps all (chunk, kv head, row slice) CTAs
    // within the fewest full waves of resident CTAs
    const uint32_t cs_rs = cold_smem_slice_rows(A, RP);
    std::vector<ColdChunk> cold_chunks;
    if (cs_rs && !cold_items.empty()) {
        const uint64_t per_seq = static_cast<uint64_t>(Hkv) * (RP / cs_rs);
        const uint64_t slots = static_cast<uint64_t>(eng->prop.multiProcessorCount) * cold_smem_ctas_per_sm(A, cs_rs);
        uint32_t max_items = 0, seqs = 0;
        for (uint32_t b = 0; b < B; ++b) {
            const uint32_t n = cold_item_ptr[b + 1] - cold_item_ptr[b];
            max_items = std::max(max_items, n);
            seqs += n ? 1u : 0u;
        }
        const uint64_t waves = std::max<uint64_t>(1, (seqs * per_seq + slots - 1) / slots);
        const uint64_t target = waves * slots;
        auto count = [&](uint32_t ipc) {
            uint64_t c = 0;
            for (uint32_t b = 0; b < B; ++b) c += (cold_item_ptr[b + 1] - cold_item_ptr[b] + ipc - 1) / ipc;
            return c * per_seq;
        };
        const uint32_t max_ipc = kCsMaxPages / kColdItemPages;
        uint32_t ipc = static_cast<uint32_t>(std::max<uint64_t>(1, (cold_items.size() * per_seq + target - 1) / target));
        ipc = std::min(ipc, max_ipc);
        while (ipc < max_items && ipc < max_ipc && count(ipc) > target) ++ipc;
        for (uint32_t b = 0; b < B; ++b) {
            const uint32_t i0 = cold_item_ptr[b], n = cold_item_ptr[b + 1] - i0;
            if (!n) continue;
            const uint32_t k = (n + ipc - 1) / ipc;
            for (uint32_t j = 0; j < k; ++j)
                cold_chunks.push_back(ColdChunk{b, i0 + static_cast<uint32_t>(static_cast<uint64_t>(n) * j / k),
                                                i0 + static_cast<uint32_t>(static_cast<uint64_t>(n) * (j + 1) / k), 0});
        }
    }

    const uint64_t nh = hot_items.size(), nc = cold_items.size();
    const uint64_t cold_tokens = static_cast<uint64_t>(cold_pages) * kBlock;
    const bool need_cold = nc > 0;
    // arena layout (256-byte aligned pieces)
    struct Piece { size_t bytes; size_t off; };
    std::vector<Piece> pieces;
    auto add = [&](size_t bytes) { pieces.push_back({align_up(bytes, 256), 0}); return pieces.size() - 1; };
    const size_t i_hot_items = add(sizeof(HotItem) * std::max<uint64_t>(nh, 1));
    const size_t i_hot_ptr = add(sizeof(uint32_t) * (B + 1));
    const size_t i_hot_indptr = add(sizeof(uint32_t) * (B + 1));
    const size_t i_cold_items = add(sizeof(ColdItem) * std::max<uint64_t>(nc, 1));
    const size_t i_cold_ptr = add(sizeof(uint32_t) * (B + 1));
    const size_t i_cold_chunks = add(sizeof(ColdChunk) * std::max<size_t>(cold_chunks.size(), 1));
    const uint64_t bga = static_cast<uint64_t>(B) * Hkv * A * RP;
    const size_t i_qlat = add(need_cold ? sizeof(float) * bga : 16);
    const size_t i_w = add(need_cold ? sizeof(float) * bga : 16);
    const size_t i_scores = add(need_cold ? sizeof(float) * Hkv * cold_tokens * RP : 16);
    const size_t i_cmax = add(sizeof(float) * std::max<uint64_t>(nc, 1) * Hkv * RP);
    const size_t i_csum = add(sizeof(float) * std::max<uint64_t>(nc, 1) * Hkv * RP);
    const size_t i_cbound = add(sizeof(float) * std::max<uint64_t>(nc, 1) * Hkv * RP);
    const size_t i_ocold = add(need_cold ? sizeof(float) * B * Hkv * n_tiles * RP * D : 16);
    const size_t i_hm = add(sizeof(float) * std::max<uint64_t>(nh, 1) * Hkv * RP);
    const size_t i_hl = add(sizeof(float) * std::max<uint64_t>(nh, 1) * Hkv * RP);
    const size_t i_ho = add(sizeof(float) * std::max<uint64_t>(nh, 1) * Hkv * RP * D);
    const size_t i_status = add(256);
    size_t total = 0;
    for (auto& p : pieces) { p.off = total; total += p.bytes; }

    weaver_plan* plan = new weaver_plan();
    plan->engine = eng;
    plan->device = eng->device;
    plan->shape = *sh;
    cudaError_t e = cudaMalloc(&plan->arena, total);
    if (e != cudaSuccess) {
        delete plan;
        return cuda_fail(e, "plan scratch allocation");
    }
    auto at = [&](size_t i) { return static_cast<uint8_t*>(plan->arena) + pieces[i].off; };
    RunArgs& a = plan->base;
    a.B = B; a.nq = nq; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.A = A; a.G = G; a.R = R; a.RP = RP;
    a.scale = sh->scale;
    a.flags = sh->flags;
    a.n_atom_tiles = n_tiles;
    a.hot_items = reinterpret_cast<const HotItem*>(at(i_hot_items));
    a.n_hot_items = static_cast<uint32_t>(nh);
    a.hot_item_ptr = reinterpret_cast<const uint32_t*>(at(i_hot_ptr));
    a.hot_indptr = reinterpret_cast<const uint32_t*>(at(i_hot_indptr));
    a.cold_items = reinterpret_cast<const ColdItem*>(at(i_cold_items));
    a.n_cold_items = static_cast<uint32_t>(nc);
    a.cold_item_ptr = reinterpret_cast<const uint32_t*>(at(i_cold_ptr));
    a.cold_tokens = cold_tokens;
    a.cold_chunks = cold_chunks.empty() ? nullptr : reinterpret_cast<const ColdChunk*>(at(i_cold_chunks));
    a.n_cold_chunks = static_cast<uint32_t>(cold_chunks.size());
    a.cold_slice_rows = cs_rs;
    a.cold_score_rows = cs_rs ? cold_smem_score_rows(A, RP, cs_rs) : 0;
    a.qlat = reinterpret_cast<float*>(at(i_qlat));
    a.w = reinterpret_cast<float*>(at(i_w));
    a.scores = reinterpret_cast<float*>(at(i_scores));
    a.cmax = reinterpret_cast<float*>(at(i_cmax));
    a.csum = reinterpret_cast<float*>(at(i_csum));
    a.cbound = reinterpret_cast<float*>(at(i_cbound));
    a.ocold = reinterpret_cast<float*>(at(i_ocold));
    a.hm = reinterpret_cast<float*>(at(i_hm));
    a.hl = reinterpret_cast<float*>(at(i_hl));
    a.ho = reinterpret_cast<float*>(at(i_ho));
    a.status = reinterpret_cast<uint32_t*>(at(i_status));
    plan->row_groups = rgroups;
    plan->contract_splits = contract_mma_splits(a, static_cast<uint32_t>(eng->prop.multiProcessorCount));
    plan->n_hot_pages = hot_pages;
    plan->n_cold_pages = cold_pages;

    cudaStream_t s = eng->stream;
    e = cudaSuccess;
    if (nh) e = cudaMemcpyAsync(at(i_hot_items), hot_items.data(), sizeof(HotItem) * nh, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(at(i_hot_ptr), hot_item_ptr.data(), sizeof(uint32_t) * (B + 1), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(at(i_hot_indptr), hot_indptr, sizeof(uint32_t) * (B + 1), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && nc) e = cudaMemcpyAsync(at(i_cold_items), cold_items.data(), sizeof(ColdItem) * nc, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(at(i_cold_ptr), cold_item_ptr.data(), sizeof(uint32_t) * (B + 1), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && !cold_chunks.empty())
        e = cudaMemcpyAsync(at(i_cold_chunks), cold_chunks.data(), sizeof(ColdChunk) * cold_chunks.size(),
                            cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(at(i_status), 0, 256, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        weaver_plan_destroy(plan);
        return cuda_fail(e, "plan upload");
    }
    const char* no_fuse = getenv("WEAVER_DISABLE_FUSED");
    const char* no_hp = getenv("WEAVER_DISABLE_HP");
    if (!(no_fuse && no_fuse[0] == '1') && !(no_hp && no_hp[0] == '1')) {
        const int hrc = build_hp_plan(plan, hot_indptr, cold_indptr);
        if (hrc != WEAVER_OK) {
            weaver_plan_destroy(plan);
            return hrc;
        }
    }
    // A long cold context (2^19+ (token, kv head) pairs) with a q_latent slice
    // that fits shared memory runs faster as the multi-kernel pipeline with the
    // shared-memory cold passes than as the general single-kernel step, whose
    // cold passes gather from and reduce into L2 (about 1.8x on a 70B-shaped
    // layer with 131072 cold tokens);
    // WEAVER_PREFER_FUSED=1 keeps the single kernel.
    const char* pf = getenv("WEAVER_PREFER_FUSED");
    const bool long_cold = plan->base.cold_slice_rows && plan->base.cold_tokens * Hkv >= (1ull << 19) &&
                           !(pf && pf[0] == '1');
    if (!plan->hp && !long_cold && !(no_fuse && no_fuse[0] == '1')) {
        const int frc = build_fused_plan(plan, hot_indptr, cold_indptr);
        if (frc != WEAVER_OK) {
            weaver_plan_destroy(plan);
            return frc;
        }
    }
    if (!plan->hp && !plan->fused && nh && nc) {  // the multi-kernel step: a side stream for the hot pass
        e = cudaStreamCreateWithFlags(&plan->side, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&plan->ev_fork, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&plan->ev_join, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            weaver_plan_destroy(plan);
            return cuda_fail(e, "plan side stream");
        }
    }
    *out = plan;
    return WEAVER_OK;
}

void weaver_plan_destroy(weaver_plan* plan) {
    if (!plan) return;
    if (plan->arena || plan->farena || plan->harena || plan->side) {
        cudaSetDevice(plan->device);
        cudaDeviceSynchronize();
        if (plan->arena) cudaFree(plan->arena);
        if (plan->farena) cudaFree(plan->farena);
        if (plan->harena) cudaFree(plan->harena);
        if (plan->ev_fork) cudaEventDestroy(plan->ev_fork);
        if (plan->ev_join) cudaEventDestroy(plan->ev_join);
        if (plan->side) cudaStreamDestroy(plan->side);
    }
    delete plan;
}

int weaver_plan_kernel_count(const weaver_plan* plan) {
    if (!plan) return 0;
    if (plan->hp || plan->fused) return 1;
    int n = 1;  // merge
    if (plan->base.n_hot_items) n += 1;
    if (plan->base.n_cold_items) n += 4;
    return n;
}

int weaver_run(weaver_plan* plan, const weaver_views* v, void* stream) {
    if (!plan || !v) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument to weaver_run");
    RunArgs a = plan->base;
    const weaver_shape& sh = plan->shape;
    const bool has_hot = a.n_hot_items > 0, has_cold = a.n_cold_items > 0;
    const bool import_ql = (sh.flags & WEAVER_FLAG_QLATENT_INPUT) != 0;
    if (!v->q && (has_hot || (has_cold && !import_ql))) return fail(WEAVER_ERR_INVALID_ARGUMENT, "views.q is null");
    if (plan->combine && !(plan->hp && aligned16(v->q)))
        return fail(WEAVER_ERR_UNSUPPORTED, "an attached combiner needs the single-kernel step and a 16-byte aligned q");
    if (sh.flags & WEAVER_FLAG_PARTIALS) {
        if (!v->part_m || !v->part_l || !v->part_o) return fail(WEAVER_ERR_INVALID_ARGUMENT, "partial outputs are null");
    } else if (!v->out) {
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "views.out is null");
    }
    if (has_hot) {
        if (!v->hot_k || !v->hot_v || !v->hot_refs) return fail(WEAVER_ERR_INVALID_ARGUMENT, "hot views are null");
        if (!aligned16(v->hot_k) || !aligned16(v->hot_v)) return fail(WEAVER_ERR_MISALIGNED, "hot pool not 16-byte aligned");
        if (v->hot_pool_blocks == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "hot_pool_blocks is 0");
    }
    if (has_cold) {
        if (!v->cold_k || !v->cold_v || !v->cold_refs || !v->v_dict)
            return fail(WEAVER_ERR_INVALID_ARGUMENT, "cold views are null");
        if (import_ql ? !v->q_latent : !v->k_dict) return fail(WEAVER_ERR_INVALID_ARGUMENT, "q_latent / k_dict is null");
        if (!aligned16(v->cold_k) || !aligned16(v->cold_v) || !aligned16(v->v_dict) || (v->k_dict && !aligned16(v->k_dict)))
            return fail(WEAVER_ERR_MISALIGNED, "cold views not 16-byte aligned");
        if (v->dict_head_stride % sh.head_dim)
            return fail(WEAVER_ERR_MISALIGNED, "dict_head_stride %llu not a multiple of head_dim",
                        (unsigned long long)v->dict_head_stride);
        if (v->cold_pool_blocks == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "cold_pool_blocks is 0");
    }
    a.q = static_cast<const __half*>(v->q);
    a.q_latent = static_cast<const __half*>(v->q_latent);
    a.hot_refs = v->hot_refs;
    a.hot_pool_blocks = v->hot_pool_blocks;
    a.cold_k = reinterpret_cast<const uint4*>(v->cold_k);
    a.cold_v = reinterpret_cast<const uint4*>(v->cold_v);
    a.cold_pool_blocks = v->cold_pool_blocks;
    a.cold_refs = v->cold_refs;
    a.dict_row_stride = v->dict_head_stride / sh.head_dim;
    a.v_dict = static_cast<const __half*>(v->v_dict);
    a.out = static_cast<__half*>(v->out);
    a.part_m = v->part_m;
    a.part_l = v->part_l;
    a.part_o = v->part_o;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    plan->last_stream = s;
    WEAVER_CUDA_TRY(cudaSetDevice(plan->device), "cudaSetDevice");
    const uint64_t D = sh.head_dim, Hkv = sh.kv_heads;
    const uint64_t dict_rows = (Hkv - 1) * a.dict_row_stride + sh.dict_size;
    int rc;
    if (plan->hp && aligned16(v->q)) {
        CUtensorMap tm_hk{}, tm_hv{}, tm_kd{}, tm_vd{}, tm_kc{}, tm_vc{};
        if (has_hot) {
            const uint64_t rows = v->hot_pool_blocks * kBlock;
            if (rows >= (1ull << 31)) return fail(WEAVER_ERR_CAPACITY, "hot pool beyond 2^27 blocks");
            if ((rc = encode_2d(&tm_hk, v->hot_k, rows, Hkv * D, Hkv * D, kBlock, "hot_k"))) return rc;
            if ((rc = encode_2d(&tm_hv, v->hot_v, rows, Hkv * D, Hkv * D, kBlock, "hot_v"))) return rc;
        }
        if (has_cold) {
            if (v->cold_pool_blocks * kBlock >= (1ull << 31)) return fail(WEAVER_ERR_CAPACITY, "cold pool beyond 2^27 blocks");
            if ((rc = encode_2d(&tm_kd, v->k_dict, dict_rows, D, D, kAtomTile, "k_dict"))) return rc;
            if ((rc = encode_2d(&tm_vd, v->v_dict, dict_rows, D, D, kAtomTile, "v_dict"))) return rc;
            if ((rc = encode_codes(&tm_kc, v->cold_k, v->cold_pool_blocks, Hkv, "cold K codes"))) return rc;
            if ((rc = encode_codes(&tm_vc, v->cold_v, v->cold_pool_blocks, Hkv, "cold V codes"))) return rc;
        }
        HpArgs h = plan->hargs;
        h.r = a;
        if (weaver_combine* c = plan->combine) {
            h.ll_world = c->world;
            h.ll_rank = c->rank;
            h.ll_rows = c->rows;
            for (uint32_t p = 0; p < c->world; ++p) h.ll_recv[p] = reinterpret_cast<uint2*>(c->peer[p] + c->ll_off);
            h.ll_state = reinterpret_cast<uint32_t*>(c->base + c->ll_state_off);
        }
        WEAVER_CUDA_TRY(launch_hp(h, tm_hk, tm_hv, tm_kd, tm_vd, tm_kc, tm_vc, s), "head-partitioned step launch");
        return WEAVER_OK;
    }
    if (plan->fused && (reinterpret_cast<uintptr_t>(v->q) & 3u) == 0) {  // query rows read as f16 pairs
        CUtensorMap tm_hk{}, tm_hv{}, tm_kd{}, tm_vd{};
        if (has_hot) {
            const uint64_t rows = v->hot_pool_blocks * kBlock;
            if ((rc = encode_2d(&tm_hk, v->hot_k, rows, Hkv * D, Hkv * D, kBlock, "hot_k"))) return rc;
            if ((rc = encode_2d(&tm_hv, v->hot_v, rows, Hkv * D, Hkv * D, kBlock, "hot_v"))) return rc;
        }
        if (has_cold) {
            if ((rc = encode_2d(&tm_kd, v->k_dict, dict_rows, D, D, kAtomTile, "k_dict"))) return rc;
            if ((rc = encode_2d(&tm_vd, v->v_dict, dict_rows, D, D, kAtomTile, "v_dict"))) return rc;
        }
        FusedArgs f = plan->fargs;
        f.r = a;
        WEAVER_CUDA_TRY(launch_fused(f, tm_hk, tm_hv, tm_kd, tm_vd, s), "fused step launch");
        return WEAVER_OK;
    }
    // The hot pass: with cold work too it runs on the plan's side stream,
    // forked from `s` before the cold chain and joined before the merge, so
    // it overlaps the latency-bound cold passes (graph-capturable: an event
    // fork / join); WEAVER_NO_SIDE_STREAM=1 keeps it on `s`.
    auto run_hot = [&](cudaStream_t hs) -> int {
        // 4+ query rows per kv head: the hot blocks run on the tensor cores
        // (WEAVER_HOT_CUDA_CORES=1 keeps the CUDA-core kernel)
        const char* cc = getenv("WEAVER_HOT_CUDA_CORES");
        if (hot_mma_supported(a) && aligned16(v->hot_k) && aligned16(v->hot_v) && !(cc && cc[0] == '1')) {
            WEAVER_CUDA_TRY(launch_hot_mma(a, static_cast<const __half*>(v->hot_k), static_cast<const __half*>(v->hot_v), hs),
                            "hot launch");
        } else {
            CUtensorMap tm_k, tm_v;
            const uint64_t rows = v->hot_pool_blocks * kBlock;
            int hrc;
            if ((hrc = encode_2d(&tm_k, v->hot_k, rows, Hkv * D, Hkv * D, kBlock, "hot_k"))) return hrc;
            if ((hrc = encode_2d(&tm_v, v->hot_v, rows, Hkv * D, Hkv * D, kBlock, "hot_v"))) return hrc;
            WEAVER_CUDA_TRY(launch_hot(a, tm_k, tm_v, plan->row_groups, hs), "hot launch");
        }
        return WEAVER_OK;
    };
    const char* nss = getenv("WEAVER_NO_SIDE_STREAM");
    const bool forked = has_hot && has_cold && plan->side && !(nss && nss[0] == '1');
    if (forked) {
        WEAVER_CUDA_TRY(cudaEventRecord(plan->ev_fork, s), "fork event");
        WEAVER_CUDA_TRY(cudaStreamWaitEvent(plan->side, plan->ev_fork, 0), "fork wait");
        if ((rc = run_hot(plan->side))) return rc;
        WEAVER_CUDA_TRY(cudaEventRecord(plan->ev_join, plan->side), "join event");
    }
    bool contract_once = false;
    auto run_cold = [&]() -> int {
        CUtensorMap tm_vdict;
        if ((rc = encode_2d(&tm_vdict, v->v_dict, dict_rows, D, D, kAtomTile, "v_dict"))) return rc;
        if (import_ql) {
            WEAVER_CUDA_TRY(launch_qlat_import(a, s), "q_latent import launch");
        } else {
            CUtensorMap tm_kdict;
            if ((rc = encode_2d(&tm_kdict, v->k_dict, dict_rows, D, D, kAtomTile, "k_dict"))) return rc;
            if (qlat_tc_supported(a) && aligned16(v->q)) {
                WEAVER_CUDA_TRY(launch_qlat_tc(a, tm_kdict, s), "q_latent (tensor cores) launch");
            } else {
                WEAVER_CUDA_TRY(launch_qlat(a, tm_kdict, s), "q_latent launch");
            }
        }
        if (cold_smem_enabled(a)) {  // q_latent slice / weight table in shared memory
            WEAVER_CUDA_TRY(launch_cold_score_smem(a, s), "cold score launch");
            WEAVER_CUDA_TRY(launch_cold_scatter_smem(a, s), "cold scatter launch");
        } else {
            WEAVER_CUDA_TRY(launch_cold_score(a, s), "cold score launch");
            WEAVER_CUDA_TRY(launch_cold_scatter(a, s), "cold scatter launch");
        }
        const char* ccc = getenv("WEAVER_CONTRACT_CUDA_CORES");
        if (contract_mma_supported(a) && aligned16(v->v_dict) && !(ccc && ccc[0] == '1')) {
            WEAVER_CUDA_TRY(launch_cold_contract_mma(a, plan->contract_splits, s), "cold contraction launch");
            contract_once = true;
        } else {
            WEAVER_CUDA_TRY(launch_cold_contract(a, tm_vdict, s), "cold contraction launch");
        }
        return WEAVER_OK;
    };
    const int crc = has_cold ? run_cold() : WEAVER_OK;
    if (forked) WEAVER_CUDA_TRY(cudaStreamWaitEvent(s, plan->ev_join, 0), "join wait");  // joined on every path
    if (crc) return crc;
    if (has_hot && !forked) {
        if ((rc = run_hot(s))) return rc;
    }
    if (contract_once) {
        RunArgs m = a;
        m.n_atom_tiles = 1;  // the tensor-core contraction reduced its atom splits into one cold partial
        WEAVER_CUDA_TRY(launch_merge(m, s), "merge launch");
    } else {
        WEAVER_CUDA_TRY(launch_merge(a, s), "merge launch");
    }
    return WEAVER_OK;
}

int weaver_plan_trace(weaver_plan* plan, uint64_t* out, size_t n, uint32_t* slots_per_cta) {
    if (!plan || !out || !slots_per_cta) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    *slots_per_cta = kTraceSlots;
    const uint64_t* trace = plan->hp ? plan->hargs.trace : (plan->fused ? plan->fargs.trace : nullptr);
    const uint32_t n_ctas = plan->hp ? plan->hargs.n_ctas : plan->fargs.n_ctas;
    if (!trace) return fail(WEAVER_ERR_UNSUPPORTED, "plan has no fused-kernel trace");
    const size_t total = static_cast<size_t>(n_ctas) * kTraceSlots;
    if (n < total) return fail(WEAVER_ERR_CAPACITY, "trace needs %zu entries", total);
    WEAVER_CUDA_TRY(cudaSetDevice(plan->device), "cudaSetDevice");
    WEAVER_CUDA_TRY(cudaStreamSynchronize(plan->last_stream), "stream synchronize");
    WEAVER_CUDA_TRY(cudaMemcpy(out, trace, total * sizeof(uint64_t), cudaMemcpyDeviceToHost), "trace read");
    return WEAVER_OK;
}

int weaver_plan_status(weaver_plan* plan) {
    if (!plan) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null plan");
    WEAVER_CUDA_TRY(cudaSetDevice(plan->device), "cudaSetDevice");
    WEAVER_CUDA_TRY(cudaStreamSynchronize(plan->last_stream), "stream synchronize");
    uint32_t st[2] = {0, 0};
    WEAVER_CUDA_TRY(cudaMemcpy(st, plan->base.status, sizeof(st), cudaMemcpyDeviceToHost), "status read");
    if (st[0] || st[1]) WEAVER_CUDA_TRY(cudaMemset(plan->base.status, 0, sizeof(st)), "status reset");
    if (st[0] & DEVERR_TIMEOUT) {
        if (st[1] & 0x80000000u)
            return fail(WEAVER_ERR_TIMEOUT, "a device-side wait timed out (first: wait site %u in CTA %u)", st[1] & 0xFFu,
                        (st[1] >> 8) & 0x7FFFFFu);
        return fail(WEAVER_ERR_TIMEOUT, "a device-side wait timed out");
    }
    const uint32_t st0 = st[0];
    if (st0 & DEVERR_REF_RANGE) return fail(WEAVER_ERR_OUT_OF_RANGE, "a block reference was beyond its pool");
    if (st0 & DEVERR_ATOM_RANGE) return fail(WEAVER_ERR_OUT_OF_RANGE, "an atom index was >= dict_size");
    return WEAVER_OK;
}

// ---- host-slice decode (weaver.rs:139-237) -------------------------------------

int weaver_decode_host(weaver_engine* eng, const uint16_t* q_exact, size_t q_exact_len, const uint16_t* q_latent,
                       size_t q_latent_len, const uint16_t* hot_pool, size_t hot_pool_len,
                       const weaver_sparse_code* cold_pool, size_t cold_pool_len, const uint32_t* loom_refs,
                       size_t loom_refs_len, const uint16_t* dictionary, size_t dictionary_len,
                       const weaver_params* p, uint16_t* out, size_t out_len) {
    if (!eng || !p || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument to weaver_decode_host");
    if (p->q_heads == 0 || p->kv_heads == 0 || p->head_dim == 0 || p->gqa_group == 0)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "zero dimension in params");
    if (p->q_heads != p->gqa_group * p->kv_heads)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "q_heads %u != gqa_group %u * kv_heads %u", p->q_heads, p->gqa_group,
                    p->kv_heads);
    if (p->block_size != kBlock) return fail(WEAVER_ERR_UNSUPPORTED, "block_size %u (16 only)", p->block_size);
    if (p->sparsity_k != 4) return fail(WEAVER_ERR_UNSUPPORTED, "sparsity_k %u (4 only)", p->sparsity_k);
    const uint64_t D = p->head_dim, Hkv = p->kv_heads, Hq = p->q_heads, A = p->dict_size;
    const uint64_t nrefs = static_cast<uint64_t>(p->hot_count) + p->cold_count;
    if (q_exact_len != Hq * D || out_len != Hq * D) return fail(WEAVER_ERR_INVALID_ARGUMENT, "q_exact/out length");
    if (loom_refs_len < nrefs || (nrefs && !loom_refs)) return fail(WEAVER_ERR_INVALID_ARGUMENT, "loom_refs shorter than hot_count+cold_count");
    if (hot_pool_len % (kBlock * Hkv * D)) return fail(WEAVER_ERR_INVALID_ARGUMENT, "hot_pool length not whole blocks");
    if (cold_pool_len % (kBlock * Hkv)) return fail(WEAVER_ERR_INVALID_ARGUMENT, "cold_pool length not whole blocks");
    const uint64_t hot_blocks = hot_pool_len / (kBlock * Hkv * D);
    const uint64_t cold_blocks = cold_pool_len / (kBlock * Hkv);
    if (p->cold_count) {
        if (q_latent_len != Hq * A || dictionary_len != Hkv * A * D || !q_latent || !dictionary)
            return fail(WEAVER_ERR_INVALID_ARGUMENT, "q_latent/dictionary length");
    }
    for (uint32_t i = 0; i < p->hot_count; ++i)
        if ((loom_refs[i] & WEAVER_REF_MASK) >= hot_blocks)
            return fail(WEAVER_ERR_OUT_OF_RANGE, "hot ref %u -> block %u beyond %llu hot blocks", i,
                        loom_refs[i] & WEAVER_REF_MASK, (unsigned long long)hot_blocks);
    for (uint32_t i = 0; i < p->cold_count; ++i)
        if ((loom_refs[p->hot_count + i] & WEAVER_REF_MASK) >= cold_blocks)
            return fail(WEAVER_ERR_OUT_OF_RANGE, "cold ref %u -> block %u beyond %llu cold blocks", i,
                        loom_refs[p->hot_count + i] & WEAVER_REF_MASK, (unsigned long long)cold_blocks);
    WEAVER_CUDA_TRY(cudaSetDevice(eng->device), "cudaSetDevice");

    // plan cache keyed on the geometry and the block counts
    const bool same = eng->host_plan && !memcmp(&eng->host_params, p, sizeof(*p));
    if (!same) {
        if (eng->host_plan) weaver_plan_destroy(eng->host_plan);
        eng->host_plan = nullptr;
        weaver_shape sh{1, 1, p->q_heads, p->kv_heads, p->head_dim, p->dict_size, 1.0f, WEAVER_FLAG_QLATENT_INPUT};
        uint32_t hip[2] = {0, p->hot_count}, cip[2] = {0, p->cold_count};
        int rc = weaver_plan_create(eng, &sh, hip, cip, &eng->host_plan);
        if (rc) return rc;
        eng->host_params = *p;
    }
    cudaStream_t s = eng->stream;
    auto up = [&](DevBuf& buf, const void* src, size_t bytes, const char* what) -> int {
        cudaError_t e = buf.reserve(bytes);
        if (e != cudaSuccess) return cuda_fail(e, what);
        if (bytes && src) {
            e = cudaMemcpyAsync(buf.ptr, src, bytes, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, what);
        }
        return WEAVER_OK;
    };
    int rc;
    if ((rc = up(eng->q, q_exact, q_exact_len * 2, "q_exact upload"))) return rc;
    if ((rc = up(eng->ql, q_latent, q_latent_len * 2, "q_latent upload"))) return rc;
    if ((rc = up(eng->hot, hot_pool, hot_pool_len * 2, "hot_pool upload"))) return rc;
    if ((rc = up(eng->cold, cold_pool, cold_pool_len * sizeof(weaver_sparse_code), "cold_pool upload"))) return rc;
    if ((rc = up(eng->refs, loom_refs, nrefs * 4, "loom_refs upload"))) return rc;
    if ((rc = up(eng->dict, dictionary, dictionary_len * 2, "dictionary upload"))) return rc;
    {
        cudaError_t e = eng->out.reserve(out_len * 2);
        if (e != cudaSuccess) return cuda_fail(e, "output allocation");
    }
    weaver_views v{};
    v.q = eng->q.ptr;
    v.q_latent = eng->ql.ptr;
    v.hot_k = v.hot_v = eng->hot.ptr;
    v.hot_pool_blocks = hot_blocks;
    v.hot_refs = static_cast<const uint32_t*>(eng->refs.ptr);
    v.cold_k = v.cold_v = static_cast<const weaver_sparse_code*>(eng->cold.ptr);
    v.cold_pool_blocks = cold_blocks;
    v.cold_refs = static_cast<const uint32_t*>(eng->refs.ptr) + p->hot_count;
    v.k_dict = nullptr;
    v.v_dict = eng->dict.ptr;
    v.dict_head_stride = A * D;
    v.out = eng->out.ptr;
    if ((rc = weaver_run(eng->host_plan, &v, s))) return rc;
    WEAVER_CUDA_TRY(cudaMemcpyAsync(out, eng->out.ptr, out_len * 2, cudaMemcpyDeviceToHost, s), "output download");
    return weaver_plan_status(eng->host_plan);  // synchronises (weaver.rs:227-228)
}

int weaver_decode_host_batch(weaver_engine* eng, const weaver_shape* sh, const uint32_t* hot_indptr,
                             const uint32_t* cold_indptr, const weaver_views* hv) {
    if (!eng || !sh || !hot_indptr || !cold_indptr || !hv)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument to weaver_decode_host_batch");
    const uint32_t B = sh->num_seqs;
    if (B == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "num_seqs is 0");
    WEAVER_CUDA_TRY(cudaSetDevice(eng->device), "cudaSetDevice");
    const bool same = eng->batch_plan && !memcmp(&eng->batch_shape, sh, sizeof(*sh)) &&
                      eng->batch_hip.size() == B + 1 &&
                      std::equal(eng->batch_hip.begin(), eng->batch_hip.end(), hot_indptr) &&
                      std::equal(eng->batch_cip.begin(), eng->batch_cip.end(), cold_indptr);
    if (!same) {
        if (eng->batch_plan) weaver_plan_destroy(eng->batch_plan);
        eng->batch_plan = nullptr;
        int rc = weaver_plan_create(eng, sh, hot_indptr, cold_indptr, &eng->batch_plan);
        if (rc) return rc;
        eng->batch_shape = *sh;
        eng->batch_hip.assign(hot_indptr, hot_indptr + B + 1);
        eng->batch_cip.assign(cold_indptr, cold_indptr + B + 1);
    }
    const uint64_t D = sh->head_dim, Hkv = sh->kv_heads, A = sh->dict_size;
    const uint64_t rows = static_cast<uint64_t>(B) * sh->num_queries * sh->q_heads;
    const uint64_t hot_bytes = hv->hot_pool_blocks * kBlock * Hkv * D * 2;
    const uint64_t cold_bytes = hv->cold_pool_blocks * kBlock * Hkv * sizeof(weaver_sparse_code);
    const uint64_t dict_bytes = (hv->dict_head_stride ? (Hkv - 1) * hv->dict_head_stride + A * D : A * D) * 2;
    const bool partials = (sh->flags & WEAVER_FLAG_PARTIALS) != 0;
    cudaStream_t s = eng->stream;
    auto up = [&](DevBuf& buf, const void* src, size_t bytes, const char* what) -> int {
        cudaError_t e = buf.reserve(bytes);
        if (e != cudaSuccess) return cuda_fail(e, what);
        if (bytes && src) {
            e = cudaMemcpyAsync(buf.ptr, src, bytes, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return cuda_fail(e, what);
        }
        return WEAVER_OK;
    };
    int rc;
    weaver_views v = *hv;
    if ((rc = up(eng->b_q, hv->q, rows * D * 2, "q upload"))) return rc;
    v.q = hv->q ? eng->b_q.ptr : nullptr;
    if (sh->flags & WEAVER_FLAG_QLATENT_INPUT) {
        if ((rc = up(eng->b_ql, hv->q_latent, rows * A * 2, "q_latent upload"))) return rc;
        v.q_latent = hv->q_latent ? eng->b_ql.ptr : nullptr;
    }
    if (hv->hot_k) {
        if ((rc = up(eng->b_hk, hv->hot_k, hot_bytes, "hot_k upload"))) return rc;
        v.hot_k = eng->b_hk.ptr;
        if (hv->hot_v == hv->hot_k) {
            v.hot_v = v.hot_k;
        } else {
            if ((rc = up(eng->b_hv, hv->hot_v, hot_bytes, "hot_v upload"))) return rc;
            v.hot_v = hv->hot_v ? eng->b_hv.ptr : nullptr;
        }
    }
    if ((rc = up(eng->b_hr, hv->hot_refs, static_cast<size_t>(hot_indptr[B]) * 4, "hot_refs upload"))) return rc;
    v.hot_refs = hv->hot_refs ? static_cast<const uint32_t*>(eng->b_hr.ptr) : nullptr;
    if (hv->cold_k) {
        if ((rc = up(eng->b_ck, hv->cold_k, cold_bytes, "cold_k upload"))) return rc;
        v.cold_k = static_cast<const weaver_sparse_code*>(eng->b_ck.ptr);
        if (hv->cold_v == hv->cold_k) {
            v.cold_v = v.cold_k;
        } else {
            if ((rc = up(eng->b_cv, hv->cold_v, cold_bytes, "cold_v upload"))) return rc;
            v.cold_v = hv->cold_v ? static_cast<const weaver_sparse_code*>(eng->b_cv.ptr) : nullptr;
        }
    }
    if ((rc = up(eng->b_cr, hv->cold_refs, static_cast<size_t>(cold_indptr[B]) * 4, "cold_refs upload"))) return rc;
    v.cold_refs = hv->cold_refs ? static_cast<const uint32_t*>(eng->b_cr.ptr) : nullptr;
    if (hv->k_dict) {
        if ((rc = up(eng->b_kd, hv->k_dict, dict_bytes, "k_dict upload"))) return rc;
        v.k_dict = eng->b_kd.ptr;
    }
    if (hv->v_dict) {
        if (hv->v_dict == hv->k_dict) {
            v.v_dict = v.k_dict;
        } else {
            if ((rc = up(eng->b_vd, hv->v_dict, dict_bytes, "v_dict upload"))) return rc;
            v.v_dict = eng->b_vd.ptr;
        }
    }
    cudaError_t e;
    if (partials) {
        if ((e = eng->b_pm.reserve(rows * 4)) || (e = eng->b_pl.reserve(rows * 4)) ||
            (e = eng->b_po.reserve(rows * D * 4)))
            return cuda_fail(e, "partials allocation");
        v.part_m = static_cast<float*>(eng->b_pm.ptr);
        v.part_l = static_cast<float*>(eng->b_pl.ptr);
        v.part_o = static_cast<float*>(eng->b_po.ptr);
    } else {
        if ((e = eng->b_out.reserve(rows * D * 2))) return cuda_fail(e, "output allocation");
        v.out = eng->b_out.ptr;
    }
    if ((rc = weaver_run(eng->batch_plan, &v, s))) return rc;
    if (partials) {
        WEAVER_CUDA_TRY(cudaMemcpyAsync(hv->part_m, v.part_m, rows * 4, cudaMemcpyDeviceToHost, s), "m download");
        WEAVER_CUDA_TRY(cudaMemcpyAsync(hv->part_l, v.part_l, rows * 4, cudaMemcpyDeviceToHost, s), "l download");
        WEAVER_CUDA_TRY(cudaMemcpyAsync(hv->part_o, v.part_o, rows * D * 4, cudaMemcpyDeviceToHost, s), "o download");
    } else {
        WEAVER_CUDA_TRY(cudaMemcpyAsync(hv->out, v.out, rows * D * 2, cudaMemcpyDeviceToHost, s), "output download");
    }
    return weaver_plan_status(eng->batch_plan);
}

// ---- split-KV combine and atom selection ----------------------------------------

int weaver_merge_partials(uint32_t n_parts, uint32_t rows, uint32_t head_dim, const float* m, const float* l,
                          const float* o, void* out, void* stream) {
    if (!m || !l || !o || !out || n_parts == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (head_dim != 64 && head_dim != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u", head_dim);
    WEAVER_CUDA_TRY(launch_merge_partials(n_parts, rows, head_dim, m, l, o, static_cast<__half*>(out),
                                          static_cast<cudaStream_t>(stream)),
                    "merge launch");
    return WEAVER_OK;
}

int weaver_merge_partials_strided(uint32_t n_parts, uint32_t rows, uint32_t head_dim, const float* m, const float* l,
                                  const float* o, uint64_t part_stride, void* out, void* stream) {
    if (!m || !l || !o || !out || n_parts == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (head_dim != 64 && head_dim != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u", head_dim);
    if (part_stride < static_cast<uint64_t>(rows) * head_dim)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "part_stride %llu below rows*head_dim", (unsigned long long)part_stride);
    WEAVER_CUDA_TRY(launch_merge_partials_strided(n_parts, rows, head_dim, m, l, o, part_stride,
                                                  static_cast<__half*>(out), static_cast<cudaStream_t>(stream)),
                    "merge launch");
    return WEAVER_OK;
}

// ---- split-KV combine over NVLink peer memory ----------------------------------

}  // extern "C"

extern "C" {

int weaver_combine_create(weaver_engine* eng, uint32_t world, uint32_t rank, uint32_t rows, uint32_t head_dim,
                          weaver_combine** out) {
    if (!eng || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (world == 0 || world > kCombineMaxRanks || rank >= world)
        return fail(WEAVER_ERR_UNSUPPORTED, "world %u / rank %u (1..%u ranks)", world, rank, kCombineMaxRanks);
    if (head_dim != 64 && head_dim != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u", head_dim);
    if (rows == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "rows is 0");
    WEAVER_CUDA_TRY(cudaSetDevice(eng->device), "cudaSetDevice");
    const size_t slot = align_up(static_cast<uint64_t>(rows) * (head_dim + 2), 4);
    auto* c = new weaver_combine();
    c->engine = eng;
    c->device = eng->device;
    c->world = world;
    c->rank = rank;
    c->rows = rows;
    c->D = head_dim;
    c->recv_bytes = align_up(2ull * world * slot * sizeof(float), 256);
    c->ll_off = c->recv_bytes + align_up((kCombineMaxRanks + 2) * sizeof(uint32_t), 256);
    c->ll_state_off = c->ll_off + align_up(2ull * world * rows * (head_dim + 2) * 8, 256);
    const size_t total = c->ll_state_off + 256;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, total);
    if (e == cudaSuccess) e = cudaMemset(p, 0, total);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        delete c;
        return cuda_fail(e, "combine buffer");
    }
    c->base = static_cast<uint8_t*>(p);
    c->peer[rank] = c->base;
    c->opened[rank] = true;
    *out = c;
    return WEAVER_OK;
}

void weaver_combine_destroy(weaver_combine* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    for (uint32_t p = 0; p < c->world; ++p)
        if (p != c->rank && c->peer[p]) cudaIpcCloseMemHandle(c->peer[p]);
    if (c->base) cudaFree(c->base);
    delete c;
}

int weaver_combine_ipc_handle(weaver_combine* c, void* handle_out) {
    if (!c || !handle_out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == WEAVER_IPC_HANDLE_BYTES, "IPC handle size");
    WEAVER_CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    cudaIpcMemHandle_t h;
    WEAVER_CUDA_TRY(cudaIpcGetMemHandle(&h, c->base), "cudaIpcGetMemHandle");
    std::memcpy(handle_out, &h, sizeof(h));
    return WEAVER_OK;
}

int weaver_combine_open_peer(weaver_combine* c, uint32_t peer, const void* handle) {
    if (!c || !handle) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (peer >= c->world) return fail(WEAVER_ERR_INVALID_ARGUMENT, "peer %u of %u", peer, c->world);
    if (peer == c->rank || c->opened[peer]) return WEAVER_OK;
    WEAVER_CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    WEAVER_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    c->peer[peer] = static_cast<uint8_t*>(p);
    c->opened[peer] = true;
    return WEAVER_OK;
}

int weaver_combine_run(weaver_combine* c, const float* packed, void* out, void* stream) {
    if (!c || !packed || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (!aligned16(packed)) return fail(WEAVER_ERR_MISALIGNED, "packed partials not 16-byte aligned");
    CombineArgs a{};
    a.world = c->world;
    a.rank = c->rank;
    a.rows = c->rows;
    a.D = c->D;
    for (uint32_t p = 0; p < c->world; ++p) {
        if (!c->opened[p]) return fail(WEAVER_ERR_INVALID_ARGUMENT, "peer %u not opened", p);
        a.recv[p] = reinterpret_cast<float*>(c->peer[p]);
        a.flags[p] = reinterpret_cast<uint32_t*>(c->peer[p] + c->recv_bytes);
    }
    a.state = reinterpret_cast<uint32_t*>(c->base + c->recv_bytes) + kCombineMaxRanks;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    c->last_stream = s;
    WEAVER_CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    WEAVER_CUDA_TRY(launch_combine(a, packed, static_cast<__half*>(out), s), "combine launch");
    return WEAVER_OK;
}

int weaver_combine_status(weaver_combine* c) {
    if (!c) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    WEAVER_CUDA_TRY(cudaSetDevice(c->device), "cudaSetDevice");
    WEAVER_CUDA_TRY(cudaStreamSynchronize(c->last_stream), "stream synchronize");
    uint32_t* st = reinterpret_cast<uint32_t*>(c->base + c->recv_bytes) + kCombineMaxRanks + 1;
    uint32_t v = 0;
    WEAVER_CUDA_TRY(cudaMemcpy(&v, st, sizeof(v), cudaMemcpyDeviceToHost), "combine status read");
    if (v) {
        WEAVER_CUDA_TRY(cudaMemset(st, 0, sizeof(v)), "combine status reset");
        return fail(WEAVER_ERR_TIMEOUT, "a peer's partials did not arrive in time");
    }
    return WEAVER_OK;
}

int weaver_plan_attach_combine(weaver_plan* plan, weaver_combine* c) {
    if (!plan) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null plan");
    if (!c) {
        plan->combine = nullptr;
        return WEAVER_OK;
    }
    const weaver_shape& sh = plan->shape;
    if (!plan->hp) return fail(WEAVER_ERR_UNSUPPORTED, "this plan's geometry does not run the single-kernel step");
    if (sh.flags & WEAVER_FLAG_PARTIALS) return fail(WEAVER_ERR_INVALID_ARGUMENT, "plan writes partials; attach needs out");
    const uint64_t rows = static_cast<uint64_t>(sh.num_seqs) * sh.num_queries * sh.q_heads;
    if (rows != c->rows || sh.head_dim != c->D)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "combiner has %u rows of %u, plan %llu of %u", c->rows, c->D,
                    (unsigned long long)rows, sh.head_dim);
    if (plan->device != c->device) return fail(WEAVER_ERR_INVALID_ARGUMENT, "different devices");
    for (uint32_t p = 0; p < c->world; ++p)
        if (!c->opened[p]) return fail(WEAVER_ERR_INVALID_ARGUMENT, "peer %u not opened", p);
    plan->combine = c;
    return WEAVER_OK;
}

// Atom selection on the tensor cores when the geometry allows it (head_dim 64
// or 128, at least 4 atoms, a head stride of whole dictionary rows), else on
// the CUDA cores; both give the CPU rule's codes bit for bit.  The variable
// WEAVER_DISTILL_CUDA_CORES=1 keeps the CUDA-core kernel.
static bool distill_use_tc(uint32_t D, uint32_t A, uint64_t dict_head_stride) {
    const char* env = getenv("WEAVER_DISTILL_CUDA_CORES");
    if (env && env[0] == '1') return false;
    return distill_tc_supported(D, A, dict_head_stride);
}

static int run_distill_tc(DistillTcArgs p, uint32_t D, cudaStream_t s, const char* what) {
    const uint64_t stride_rows = p.dict_head_stride / D;
    const uint64_t rows = (p.Hkv - 1) * stride_rows + p.A;
    if (rows >= (1ull << 31) || stride_rows >= (1ull << 31) / 2)
        return fail(WEAVER_ERR_CAPACITY, "dictionary of %llu rows", (unsigned long long)rows);
    p.dict_row_stride = static_cast<uint32_t>(stride_rows);
    CUtensorMap tm{};
    int rc = encode_2d(&tm, p.dict, rows, D, D, 256, "dictionary");
    if (rc) return rc;
    WEAVER_CUDA_TRY(launch_distill_tc(p, D, tm, s), what);
    return WEAVER_OK;
}

static int distill_checks(const void* rows, uint32_t kv_heads, uint32_t head_dim, const void* dictionary,
                          uint32_t dict_size, uint64_t dict_head_stride, const void* out_codes) {
    if (!rows || !dictionary || !out_codes || kv_heads == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (head_dim != 64 && head_dim != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u", head_dim);
    if (dict_size == 0 || dict_size > 65536) return fail(WEAVER_ERR_UNSUPPORTED, "dict_size %u", dict_size);
    if (!aligned16(rows) || !aligned16(dictionary) || (dict_head_stride * 2) % 16)
        return fail(WEAVER_ERR_MISALIGNED, "distill inputs not 16-byte aligned");
    return WEAVER_OK;
}

int weaver_distill(const void* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t head_dim, const void* dictionary,
                   uint32_t dict_size, uint64_t dict_head_stride, weaver_sparse_code* out_codes, void* stream) {
    int rc = distill_checks(rows, kv_heads, head_dim, dictionary, dict_size, dict_head_stride, out_codes);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (distill_use_tc(head_dim, dict_size, dict_head_stride)) {
        DistillTcArgs p{};
        p.rows = static_cast<const __half*>(rows);
        p.n_rows = n_rows;
        p.Hkv = kv_heads;
        p.A = dict_size;
        p.dict_head_stride = dict_head_stride;
        p.dict = static_cast<const __half*>(dictionary);
        p.out = reinterpret_cast<uint4*>(out_codes);
        return run_distill_tc(p, head_dim, s, "distill launch");
    }
    WEAVER_CUDA_TRY(launch_distill(static_cast<const __half*>(rows), n_rows, kv_heads, head_dim,
                                   static_cast<const __half*>(dictionary), dict_size, dict_head_stride,
                                   reinterpret_cast<uint4*>(out_codes), s),
                    "distill launch");
    return WEAVER_OK;
}

int weaver_distill_stats(const void* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t head_dim,
                         const void* dictionary, uint32_t dict_size, uint64_t dict_head_stride,
                         weaver_sparse_code* out_codes, uint32_t* diag, void* stream) {
    int rc = distill_checks(rows, kv_heads, head_dim, dictionary, dict_size, dict_head_stride, out_codes);
    if (rc) return rc;
    if (!diag) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null diagnostics buffer");
    if (!distill_tc_supported(head_dim, dict_size, dict_head_stride))
        return fail(WEAVER_ERR_UNSUPPORTED, "no tensor-core atom selection for this geometry");
    DistillTcArgs p{};
    p.rows = static_cast<const __half*>(rows);
    p.n_rows = n_rows;
    p.Hkv = kv_heads;
    p.A = dict_size;
    p.dict_head_stride = dict_head_stride;
    p.dict = static_cast<const __half*>(dictionary);
    p.out = reinterpret_cast<uint4*>(out_codes);
    p.diag = diag;
    return run_distill_tc(p, head_dim, static_cast<cudaStream_t>(stream), "distill launch");
}

int weaver_block_entropy(const void* hot_pool, uint64_t n_blocks, uint32_t kv_heads, uint32_t head_dim, float* out,
                         void* stream) {
    if (!hot_pool || !out || kv_heads == 0 || head_dim == 0) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    const uint64_t vals = static_cast<uint64_t>(kBlock) * kv_heads * head_dim;
    if (vals % 8 || vals >= (1ull << 32)) return fail(WEAVER_ERR_UNSUPPORTED, "block of %llu values", (unsigned long long)vals);
    if (!aligned16(hot_pool)) return fail(WEAVER_ERR_MISALIGNED, "hot pool not 16-byte aligned");
    WEAVER_CUDA_TRY(launch_block_entropy(static_cast<const __half*>(hot_pool), n_blocks, static_cast<uint32_t>(vals), out,
                                         static_cast<cudaStream_t>(stream)),
                    "block entropy launch");
    return WEAVER_OK;
}

int weaver_migrate_blocks(const void* hot_k, const void* hot_v, uint64_t hot_pool_blocks, const uint32_t* src_blocks,
                          const uint32_t* dst_blocks, uint32_t n, uint32_t kv_heads, uint32_t head_dim,
                          const void* k_dict, const void* v_dict, uint32_t dict_size, uint64_t dict_head_stride,
                          weaver_sparse_code* cold_k, weaver_sparse_code* cold_v, uint64_t cold_pool_blocks,
                          uint32_t* bad_flag, void* stream) {
    if (n == 0) return WEAVER_OK;
    if (!hot_k || !hot_v || !src_blocks || !dst_blocks || !k_dict || !v_dict || !cold_k || !cold_v || !bad_flag ||
        kv_heads == 0)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (head_dim != 64 && head_dim != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u", head_dim);
    if (dict_size == 0 || dict_size > 65536) return fail(WEAVER_ERR_UNSUPPORTED, "dict_size %u", dict_size);
    if (!aligned16(hot_k) || !aligned16(hot_v) || !aligned16(k_dict) || !aligned16(v_dict) ||
        (dict_head_stride * 2) % 16)
        return fail(WEAVER_ERR_MISALIGNED, "migration inputs not 16-byte aligned");
    if (n > 65535) return fail(WEAVER_ERR_CAPACITY, "%u blocks in one call (at most 65535)", n);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // (the tensor-core kernel indexes code records in 32 bits)
    if (distill_use_tc(head_dim, dict_size, dict_head_stride) && cold_pool_blocks * kBlock * kv_heads < (1ull << 32)) {
        DistillTcArgs p{};
        p.src_blocks = src_blocks;
        p.dst_blocks = dst_blocks;
        p.n_blocks = n;
        p.src_limit = hot_pool_blocks;
        p.dst_limit = cold_pool_blocks;
        p.bad = bad_flag;
        p.Hkv = kv_heads;
        p.A = dict_size;
        p.dict_head_stride = dict_head_stride;
        p.pool = static_cast<const __half*>(hot_k);
        p.dict = static_cast<const __half*>(k_dict);
        p.out = reinterpret_cast<uint4*>(cold_k);
        int rc = run_distill_tc(p, head_dim, s, "K migration launch");
        if (rc) return rc;
        p.pool = static_cast<const __half*>(hot_v);
        p.dict = static_cast<const __half*>(v_dict);
        p.out = reinterpret_cast<uint4*>(cold_v);
        return run_distill_tc(p, head_dim, s, "V migration launch");
    }
    WEAVER_CUDA_TRY(launch_distill_blocks(static_cast<const __half*>(hot_k), hot_pool_blocks, src_blocks, dst_blocks, n,
                                          kv_heads, head_dim, static_cast<const __half*>(k_dict), dict_size,
                                          dict_head_stride, reinterpret_cast<uint4*>(cold_k), cold_pool_blocks, bad_flag,
                                          s),
                    "K migration launch");
    WEAVER_CUDA_TRY(launch_distill_blocks(static_cast<const __half*>(hot_v), hot_pool_blocks, src_blocks, dst_blocks, n,
                                          kv_heads, head_dim, static_cast<const __half*>(v_dict), dict_size,
                                          dict_head_stride, reinterpret_cast<uint4*>(cold_v), cold_pool_blocks, bad_flag,
                                          s),
                    "V migration launch");
    return WEAVER_OK;
}

// ops.metal:528-616 (multihead_attention, inference.rs:552-562) on the device.
int weaver_multihead_attention(weaver_engine* eng, const void* q, const void* k_cache, const void* v_cache, void* out,
                               uint32_t total_kv_len, uint32_t head_dim, uint32_t q_heads, uint32_t kv_heads,
                               uint32_t num_queries, void* stream) {
    if (!eng || !q || !k_cache || !v_cache || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (head_dim != 64 && head_dim != 128) return fail(WEAVER_ERR_UNSUPPORTED, "head_dim %u", head_dim);
    if (kv_heads == 0 || kv_heads > 65535 || q_heads == 0 || q_heads % kv_heads)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "q_heads %u is not a multiple of kv_heads %u", q_heads, kv_heads);
    if (num_queries == 0 || total_kv_len < num_queries)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "total_kv_len %u below num_queries %u", total_kv_len, num_queries);
    const uint64_t rows = static_cast<uint64_t>(num_queries) * (q_heads / kv_heads);
    if ((rows + 15) / 16 > 65535 || static_cast<uint64_t>(num_queries) * q_heads >= (1u << 31))
        return fail(WEAVER_ERR_CAPACITY, "%u queries x %u heads", num_queries, q_heads);
    if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out))
        return fail(WEAVER_ERR_MISALIGNED, "multi-query attention views not 16-byte aligned");
    WEAVER_CUDA_TRY(cudaSetDevice(eng->device), "cudaSetDevice");
    const uint32_t n_sm = static_cast<uint32_t>(eng->prop.multiProcessorCount);
    const uint64_t floats = mha_scratch_floats(total_kv_len, head_dim, q_heads, kv_heads, num_queries, n_sm);
    if (floats) WEAVER_CUDA_TRY(eng->mha.reserve(floats * sizeof(float)), "multi-query attention scratch");
    WEAVER_CUDA_TRY(launch_mha(static_cast<const __half*>(q), static_cast<const __half*>(k_cache),
                               static_cast<const __half*>(v_cache), static_cast<__half*>(out),
                               static_cast<float*>(eng->mha.ptr), total_kv_len, head_dim, q_heads, kv_heads,
                               num_queries, n_sm, static_cast<cudaStream_t>(stream)),
                    "multi-query attention launch");
    return WEAVER_OK;
}

// ---- device-resident Fabric (fabric.rs:124-186, 347-420; types.rs:311-328) ----

}  // extern "C"

struct weaver_device_fabric {
    int device = 0;
    weaver_fabric_geometry g{};
    void* base = nullptr;
    size_t bytes = 0;
    uint64_t hot_bytes = 0, cold_bytes = 0, dict_bytes = 0;  // one view of one layer
    size_t refs_off = 0;
    std::vector<size_t> off;  // per layer: hot_k, hot_v, cold_k, cold_v, k_dict, v_dict
};

extern "C" {

int weaver_device_fabric_create(int device, const weaver_fabric_geometry* g, weaver_device_fabric** out) {
    if (!g || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    *out = nullptr;
    if (g->layers == 0 || g->kv_heads == 0 || (g->head_dim != 64 && g->head_dim != 128) || g->dict_size == 0 ||
        g->dict_size > 65536)
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "fabric geometry (layers %u, kv_heads %u, head_dim %u, dict %u)",
                    g->layers, g->kv_heads, g->head_dim, g->dict_size);
    if (g->hot_blocks >= (1ull << 27) || g->cold_blocks >= (1ull << 27) || g->max_block_refs >= (1ull << 31))
        return fail(WEAVER_ERR_CAPACITY, "fabric pools beyond 2^27 blocks or 2^31 block refs");
    weaver_device_fabric* f = new weaver_device_fabric();
    f->device = device;
    f->g = *g;
    f->hot_bytes = g->hot_blocks * kBlock * g->kv_heads * g->head_dim * 2;
    f->cold_bytes = g->cold_blocks * kBlock * g->kv_heads * sizeof(weaver_sparse_code);
    f->dict_bytes = static_cast<uint64_t>(g->kv_heads) * g->dict_size * g->head_dim * 2;
    size_t total = 0;
    auto take = [&](uint64_t b) {
        const size_t o = total;
        total += align_up(b ? b : 16, 256);
        return o;
    };
    for (uint32_t l = 0; l < g->layers; ++l) {
        const size_t hk = take(f->hot_bytes), hv = g->separate_v ? take(f->hot_bytes) : hk;
        const size_t ck = take(f->cold_bytes), cv = g->separate_v ? take(f->cold_bytes) : ck;
        const size_t kd = take(f->dict_bytes), vd = g->separate_v ? take(f->dict_bytes) : kd;
        f->off.insert(f->off.end(), {hk, hv, ck, cv, kd, vd});
    }
    f->refs_off = take(g->max_block_refs * 4);
    f->bytes = total;
    cudaError_t e;
    if ((e = cudaSetDevice(device)) != cudaSuccess || (e = cudaMalloc(&f->base, total)) != cudaSuccess ||
        (e = cudaMemset(f->base, 0, total)) != cudaSuccess) {
        if (f->base) cudaFree(f->base);
        delete f;
        return cuda_fail(e, "device fabric allocation");
    }
    *out = f;
    return WEAVER_OK;
}

void weaver_device_fabric_destroy(weaver_device_fabric* f) {
    if (!f) return;
    cudaSetDevice(f->device);
    cudaDeviceSynchronize();
    if (f->base) cudaFree(f->base);
    delete f;
}

int weaver_device_fabric_layer(const weaver_device_fabric* f, uint32_t layer, weaver_fabric_layer* out) {
    if (!f || !out) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (layer >= f->g.layers) return fail(WEAVER_ERR_INVALID_ARGUMENT, "layer %u of %u", layer, f->g.layers);
    uint8_t* b = static_cast<uint8_t*>(f->base);
    const size_t* o = &f->off[static_cast<size_t>(layer) * 6];
    out->hot_k = b + o[0];
    out->hot_v = b + o[1];
    out->cold_k = reinterpret_cast<weaver_sparse_code*>(b + o[2]);
    out->cold_v = reinterpret_cast<weaver_sparse_code*>(b + o[3]);
    out->k_dict = b + o[4];
    out->v_dict = b + o[5];
    out->hot_pool_blocks = f->g.hot_blocks;
    out->cold_pool_blocks = f->g.cold_blocks;
    return WEAVER_OK;
}

int weaver_device_fabric_block_refs(const weaver_device_fabric* f, uint32_t** refs, uint64_t* capacity) {
    if (!f || !refs || !capacity) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    *refs = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(f->base) + f->refs_off);
    *capacity = f->g.max_block_refs;
    return WEAVER_OK;
}

int weaver_device_fabric_upload_aether(weaver_device_fabric* f, uint32_t layer, const void* image, uint64_t image_bytes,
                                       const weaver_fabric_regions* r, uint32_t which, void* stream) {
    if (!f || !image || !r) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (layer >= f->g.layers) return fail(WEAVER_ERR_INVALID_ARGUMENT, "layer %u of %u", layer, f->g.layers);
    if (which > 1 || (which == 1 && !f->g.separate_v))
        return fail(WEAVER_ERR_INVALID_ARGUMENT, "V regions need a fabric with separate_v");
    struct Region { uint64_t off, size, cap; size_t dst; const char* what; };
    const size_t* o = &f->off[static_cast<size_t>(layer) * 6];
    const Region regs[3] = {{r->hot_pool_offset, r->hot_pool_size, f->hot_bytes, o[0 + which], "hot pool"},
                            {r->cold_pool_offset, r->cold_pool_size, f->cold_bytes, o[2 + which], "cold pool"},
                            {r->dict_offset, r->dict_size, f->dict_bytes, o[4 + which], "dictionary"}};
    for (const Region& g : regs) {
        if (g.off > image_bytes || g.size > image_bytes - g.off)
            return fail(WEAVER_ERR_INVALID_ARGUMENT, "%s region beyond the %llu-byte image", g.what,
                        (unsigned long long)image_bytes);
        if (g.size > g.cap)
            return fail(WEAVER_ERR_CAPACITY, "%s region of %llu bytes exceeds the layer's %llu", g.what,
                        (unsigned long long)g.size, (unsigned long long)g.cap);
    }
    WEAVER_CUDA_TRY(cudaSetDevice(f->device), "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (const Region& g : regs)
        if (g.size)
            WEAVER_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(f->base) + g.dst,
                                            static_cast<const uint8_t*>(image) + g.off, g.size,
                                            cudaMemcpyHostToDevice, s),
                            "fabric region upload");
    return WEAVER_OK;
}

int weaver_device_fabric_upload_refs(weaver_device_fabric* f, const uint32_t* refs, uint64_t n, uint64_t offset,
                                     void* stream) {
    if (!f || (!refs && n)) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    if (offset > f->g.max_block_refs || n > f->g.max_block_refs - offset)
        return fail(WEAVER_ERR_CAPACITY, "%llu block refs at %llu beyond the array of %llu", (unsigned long long)n,
                    (unsigned long long)offset, (unsigned long long)f->g.max_block_refs);
    if (!n) return WEAVER_OK;
    WEAVER_CUDA_TRY(cudaSetDevice(f->device), "cudaSetDevice");
    WEAVER_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(f->base) + f->refs_off + offset * 4, refs, n * 4,
                                    cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)),
                    "block ref upload");
    return WEAVER_OK;
}

int weaver_loom_page_tables(const weaver_device_fabric* f, const weaver_loom_descriptor* looms, uint32_t n,
                            uint32_t* hot_indptr, uint32_t* cold_indptr, uint32_t* hot_refs, uint64_t hot_capacity,
                            uint32_t* cold_refs, uint64_t cold_capacity, void* stream) {
    if (!f || (!looms && n) || !hot_indptr || !cold_indptr) return fail(WEAVER_ERR_INVALID_ARGUMENT, "null argument");
    uint64_t nh = 0, nc = 0;
    hot_indptr[0] = cold_indptr[0] = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const weaver_loom_descriptor& L = looms[i];
        if (static_cast<uint64_t>(L.hot_refs_offset) + L.hot_count > f->g.max_block_refs ||
            static_cast<uint64_t>(L.cold_refs_offset) + L.cold_count > f->g.max_block_refs)
            return fail(WEAVER_ERR_INVALID_ARGUMENT, "loom %u refers past the %llu block refs", i,
                        (unsigned long long)f->g.max_block_refs);
        nh += L.hot_count;
        nc += L.cold_count;
        if (nh >= (1ull << 32) || nc >= (1ull << 32)) return fail(WEAVER_ERR_CAPACITY, "page tables beyond 2^32 refs");
        hot_indptr[i + 1] = static_cast<uint32_t>(nh);
        cold_indptr[i + 1] = static_cast<uint32_t>(nc);
    }
    if (nh > hot_capacity || nc > cold_capacity || (nh && !hot_refs) || (nc && !cold_refs))
        return fail(WEAVER_ERR_CAPACITY, "page tables need %llu hot and %llu cold refs", (unsigned long long)nh,
                    (unsigned long long)nc);
    WEAVER_CUDA_TRY(cudaSetDevice(f->device), "cudaSetDevice");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint32_t* src = reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(f->base) + f->refs_off);
    for (uint32_t i = 0; i < n; ++i) {
        const weaver_loom_descriptor& L = looms[i];
        if (L.hot_count)
            WEAVER_CUDA_TRY(cudaMemcpyAsync(hot_refs + hot_indptr[i], src + L.hot_refs_offset, L.hot_count * 4ull,
                                            cudaMemcpyDeviceToDevice, s),
                            "hot page table");
        if (L.cold_count)
            WEAVER_CUDA_TRY(cudaMemcpyAsync(cold_refs + cold_indptr[i], src + L.cold_refs_offset, L.cold_count * 4ull,
                                            cudaMemcpyDeviceToDevice, s),
                            "cold page table");
    }
    return WEAVER_OK;
}

}  // extern "C"

