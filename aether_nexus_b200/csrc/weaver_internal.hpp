// weaver_internal.hpp — structures shared by the host plan builder and the
// Weaver kernels.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace weaver {

constexpr uint32_t kBlock = 16;           // tokens per block (types.rs:159)
constexpr uint32_t kRefMask = 0x7FFFFFFFu; // weaver_kernel.metal:145,174
constexpr uint32_t kAtomTile = 128;       // atoms per q_latent / contraction tile
constexpr uint32_t kColdItemPages = 16;   // cold blocks per scoring CTA (256 tokens)
constexpr uint32_t kCsMaxPages = 2048;     // cold blocks per shared-memory pass chunk

// Device status bits (OR-ed into the plan's status word).
enum : uint32_t {
    DEVERR_REF_RANGE = 1u,   // a block reference beyond the pool
    DEVERR_ATOM_RANGE = 2u,  // an atom index >= dict_size
    DEVERR_TIMEOUT = 4u,     // a bounded wait expired
};

// A run of hot blocks of one sequence, processed by one CTA per kv head.
struct HotItem {
    uint32_t seq;
    uint32_t page_begin;  // index into hot_refs
    uint32_t page_end;
    uint32_t pos_base;    // token position of page_begin within the sequence
};

// A run of cold blocks of one sequence (<= kColdItemPages).
struct ColdItem {
    uint32_t seq;
    uint32_t page_begin;  // index into cold_refs
    uint32_t page_end;
    uint32_t pad;
};

// A run of consecutive cold items of one sequence, scored and scattered by one
// CTA per (kv head, row slice) with the q_latent slice / weight table in shared
// memory (weaver_cold_smem.cu).
struct ColdChunk {
    uint32_t seq;
    uint32_t item_begin;  // index into cold_items
    uint32_t item_end;
    uint32_t pad;
};

// Everything a launch needs besides the tensor maps.  Device pointers.
struct RunArgs {
    // geometry
    uint32_t B, nq, Hq, Hkv, D, A, G, R, RP;
    float scale;
    uint32_t flags;
    uint32_t n_atom_tiles;
    // inputs (views)
    const __half* q;
    const __half* q_latent;
    const uint32_t* hot_refs;
    uint64_t hot_pool_blocks;
    const uint4* cold_k;
    const uint4* cold_v;
    uint64_t cold_pool_blocks;
    const uint32_t* cold_refs;
    uint64_t dict_row_stride;  // rows (of D elements) between kv heads' dictionaries
    const __half* v_dict;      // [Hkv][A][D] (head stride dict_row_stride rows)
    __half* out;
    float* part_m;
    float* part_l;
    float* part_o;
    // plan tables
    const HotItem* hot_items;
    uint32_t n_hot_items;
    const uint32_t* hot_item_ptr;   // [B+1]
    const uint32_t* hot_indptr;     // [B+1]
    const ColdItem* cold_items;
    uint32_t n_cold_items;
    const uint32_t* cold_item_ptr;  // [B+1]
    uint64_t cold_tokens;           // 16 * total cold refs
    const ColdChunk* cold_chunks;   // null: the L2 cold passes
    uint32_t n_cold_chunks;
    uint32_t cold_slice_rows;       // RS: query rows per shared-memory scatter slice (0: none fits)
    uint32_t cold_score_rows;       // RSS: query rows per score CTA (f16 table; a multiple of RS)
    // scratch
    float* qlat;     // [B][Hkv][A][RP]
    float* w;        // [B][Hkv][A][RP]
    float* scores;   // [Hkv][cold_tokens][RP]
    float* cmax;     // [n_cold_items][Hkv][RP]
    float* csum;     // [n_cold_items][Hkv][RP]
    float* cbound;   // [n_cold_items][Hkv][RP] sum of exp(s - cmax) * |V coefficients| (shared-memory passes)
    float* ocold;    // [B][Hkv][n_atom_tiles][RP][D]
    float* hm;       // [n_hot_items][Hkv][RP]
    float* hl;
    float* ho;       // [n_hot_items][Hkv][RP][D]
    uint32_t* status;
};

// Kernel launchers (weaver_kernels.cu).  Each returns the launch error.
cudaError_t launch_qlat(const RunArgs& a, const CUtensorMap& tm_kdict, cudaStream_t s);
cudaError_t launch_qlat_import(const RunArgs& a, cudaStream_t s);
// q_latent on the tensor cores (tcgen05.mma, weaver_qlat_tc.cu): same output as
// launch_qlat; needs head_dim 64 or 128, RP <= 256 and a 16-byte aligned q.
bool qlat_tc_supported(const RunArgs& a);
size_t qlat_tc_smem_bytes(const RunArgs& a);
cudaError_t launch_qlat_tc(const RunArgs& a, const CUtensorMap& tm_kdict, cudaStream_t s);
cudaError_t launch_cold_score(const RunArgs& a, cudaStream_t s);
cudaError_t launch_cold_scatter(const RunArgs& a, cudaStream_t s);
cudaError_t launch_cold_contract(const RunArgs& a, const CUtensorMap& tm_vdict, cudaStream_t s);
// The two cold passes with the q_latent slice / weight table in shared memory
// (weaver_cold_smem.cu).  cold_smem_slice_rows: RS for (A, RP), 0 when no
// slice fits; cold_smem_ctas_per_sm: resident CTAs of that size.
uint32_t cold_smem_slice_rows(uint32_t A, uint32_t RP);
uint32_t cold_smem_ctas_per_sm(uint32_t A, uint32_t rs);
uint32_t cold_smem_score_rows(uint32_t A, uint32_t RP, uint32_t rs);
bool cold_smem_enabled(const RunArgs& a);
cudaError_t launch_cold_score_smem(const RunArgs& a, cudaStream_t s);
cudaError_t launch_cold_scatter_smem(const RunArgs& a, cudaStream_t s);
cudaError_t launch_hot(const RunArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                       uint32_t row_groups, cudaStream_t s);
// The hot pass on mma.sync tensor cores for 8+ query rows per kv head
// (weaver_hot_mma.cu); same outputs as launch_hot.
// The cold contraction on mma.sync tensor cores (weaver_contract_mma.cu): S
// atom splits (contract_mma_splits for a GPU of `sms` SMs) reduced into one
// cold partial per (b, g), so the merge then reads it as n_atom_tiles = 1.
bool contract_mma_supported(const RunArgs& a);
uint32_t contract_mma_splits(const RunArgs& a, uint32_t sms);
cudaError_t launch_cold_contract_mma(const RunArgs& a, uint32_t S, cudaStream_t s);
bool hot_mma_supported(const RunArgs& a);
cudaError_t launch_hot_mma(const RunArgs& a, const __half* hot_k, const __half* hot_v, cudaStream_t s);
cudaError_t launch_merge(const RunArgs& a, cudaStream_t s);
cudaError_t launch_merge_partials(uint32_t n_parts, uint32_t rows, uint32_t D, const float* m,
                                  const float* l, const float* o, __half* out, cudaStream_t s);
cudaError_t launch_merge_partials_strided(uint32_t n_parts, uint32_t rows, uint32_t D, const float* m,
                                          const float* l, const float* o, uint64_t part_stride, __half* out,
                                          cudaStream_t s);
cudaError_t launch_distill(const __half* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t D,
                           const __half* dict, uint32_t A, uint64_t dict_head_stride,
                           uint4* out, cudaStream_t s);
// The same selection over whole pool blocks: block src_blocks[i] of `pool`
// into block dst_blocks[i] of `cold` (both block lists on the device).
cudaError_t launch_distill_blocks(const __half* pool, uint64_t pool_blocks, const uint32_t* src_blocks,
                                  const uint32_t* dst_blocks, uint32_t n_blocks, uint32_t kv_heads, uint32_t D,
                                  const __half* dict, uint32_t A, uint64_t dict_head_stride, uint4* cold,
                                  uint64_t cold_blocks, uint32_t* bad, cudaStream_t s);
cudaError_t launch_block_entropy(const __half* pool, uint64_t n_blocks, uint32_t vals_per_block, float* out,
                                 cudaStream_t s);

// Atom selection on the tensor cores (weaver_distill_tc.cu), bit-exact with
// launch_distill / launch_distill_blocks.  Rows come from `rows` (row i of kv
// head i % Hkv) when src_blocks is null, else from the 16 tokens of hot
// blocks src_blocks[k] of `pool`, coded into cold block dst_blocks[k].
// diag (4 words, or null for library scratch): [largest |approximate - exact|
// / bound over re-scored atoms (float bits), rows finished by the exact scan,
// status, first expired wait].
struct DistillTcArgs {
    const __half* rows;
    uint64_t n_rows;
    const __half* pool;
    const uint32_t* src_blocks;
    const uint32_t* dst_blocks;
    uint32_t n_blocks;
    uint64_t src_limit, dst_limit;
    uint32_t* bad;
    uint32_t Hkv, A;
    uint64_t dict_head_stride;  // elements
    uint32_t dict_row_stride;   // dict_head_stride / head_dim
    const __half* dict;
    uint4* out;
    uint32_t* diag;
};
// The full loop's multi-query attention (weaver_mha.cu): split-KV over the
// cache on mma.sync tensor cores, then a merge over the chunks.
size_t mha_smem_bytes(uint32_t D);
uint64_t mha_scratch_floats(uint32_t T, uint32_t D, uint32_t Hq, uint32_t Hkv, uint32_t nq, uint32_t n_sm);
cudaError_t launch_mha(const __half* q, const __half* kc, const __half* vc, __half* out, float* scratch, uint32_t T,
                       uint32_t D, uint32_t Hq, uint32_t Hkv, uint32_t nq, uint32_t n_sm, cudaStream_t s);
bool distill_tc_supported(uint32_t D, uint32_t A, uint64_t dict_head_stride);
size_t distill_tc_smem_bytes(uint32_t D);
cudaError_t launch_distill_tc(DistillTcArgs p, uint32_t D, const CUtensorMap& tm_dict, cudaStream_t s);

// Rows handled by one hot CTA (the hot kernel is built for these).
constexpr uint32_t kHotRows = 8;

// ---------------------------------------------------------------------------
// Fused step: one persistent kernel per decode step (weaver_fused.cu).
// ---------------------------------------------------------------------------
enum : uint16_t { FI_QLAT = 0, FI_SCORE = 1, FI_SCATTER = 2, FI_CONTRACT = 3 };

// One unit of cold work of one CTA, in the CTA's phase order.
struct FusedItem {
    uint16_t type;   // FI_*
    uint16_t g;      // kv head (FI_QLAT / FI_CONTRACT)
    uint32_t b;      // sequence
    uint32_t a;      // atom tile (QLAT/CONTRACT) or first cold block index into cold_refs
    uint32_t n;      // blocks in a SCORE/SCATTER item
};

// A contiguous run of one (sequence, kv head)'s hot blocks for one CTA; its
// (m, l, o) partial goes to hot slot `slot`.
struct FusedHotGroup {
    uint32_t b, g, page_begin, page_end, pos_base, slot;
};

// Dependency counters per sequence, each counting finished work units.
enum : uint32_t { CNT_QLAT = 0, CNT_SCORE = 1, CNT_SCATTER = 2, CNT_CONTRACT = 3, CNT_HOT = 4, CNT_KINDS = 5 };

struct FusedArgs {
    RunArgs r;                       // geometry, views, status
    uint32_t code_pages;             // blocks per SCORE/SCATTER item
    uint32_t n_ctas;
    const FusedItem* items;          // per-CTA cold lists, CSR by item_ptr
    const uint32_t* item_ptr;        // [n_ctas + 1]
    const FusedHotGroup* groups;     // per-CTA hot lists, CSR by group_ptr
    const uint32_t* group_ptr;       // [n_ctas + 1]
    const uint32_t* merge_rows;      // per-CTA merge rows, CSR by merge_ptr
    const uint32_t* merge_ptr;       // [n_ctas + 1]
    const uint32_t* slot_ptr;        // hot slots of (b, g): CSR [B*Hkv + 1] into slot_ids
    const uint32_t* slot_ids;
    const uint32_t* code_items;      // [B] SCORE (= SCATTER) items of sequence b
    const uint32_t* hot_groups;      // [B] hot groups of sequence b
    uint32_t* counters;              // [CNT_KINDS][B] + 1 exit counter
    int* mkey;                       // [B][Hkv][RP] cold score max (ordered-int keys)
    float* lcold;                    // [B][Hkv][RP] cold sum of exp
    float* ocold;                    // [B][Hkv][RP][D] cold unnormalised output
    float* sm;                       // [n_slots][RP] hot partial max
    float* sl;                       // [n_slots][RP]
    float* so;                       // [n_slots][RP][D]
    uint64_t* trace;                 // optional [n_ctas][kTraceSlots] %globaltimer stamps
};

// Phase stamps of the fused kernels' timelines (when tracing is on).
enum : uint32_t {
    TR_START = 0, TR_QLAT_DONE, TR_SCORE_WAIT, TR_SCORE_DONE, TR_SCATTER_WAIT, TR_SCATTER_DONE,
    TR_CONTRACT_WAIT, TR_CONTRACT_DONE, TR_MERGE_WAIT, TR_MERGE_DONE, TR_HOT_DONE, TR_EXIT,
    TR_QT_LANDED, TR_CODES_LANDED, TR_QLAT_LANDED, TR_HOT_MERGE, TR_QT_LAST_LANDED, TR_SCORED, TR_WS_READY,
    TR_HOT_WIDE, TR_SCATTER_LOCAL, TR_VCODES, TR_PASS1, TR_HOT_SCORED, kTraceSlots = 24
};

// Shared memory the fused kernel needs for (D, RP); 0 if it does not fit.
size_t fused_smem_bytes(uint32_t D, uint32_t RP, uint32_t kv_heads);
// Resident fused CTAs per SM for (D, RP) (sets the kernel's shared-memory limit).
cudaError_t fused_occupancy(uint32_t D, uint32_t RP, int* blocks_per_sm);
cudaError_t launch_fused(const FusedArgs& a, const CUtensorMap& tm_hk, const CUtensorMap& tm_hv,
                         const CUtensorMap& tm_kd, const CUtensorMap& tm_vd, cudaStream_t s);

// ---------------------------------------------------------------------------
// Head-partitioned step (weaver_headpart.cu): one persistent kernel per decode
// step for geometries whose per-head q_latent (f16) and per-atom weights (fp32)
// fit in one CTA's shared memory.  Every CTA owns at most one chunk of one
// (sequence, kv head)'s cold blocks; its codes, scores and per-atom weights
// stay in shared memory.
// ---------------------------------------------------------------------------
constexpr uint32_t kHpMaxChunkPages = 128;   // 2048 tokens: 32 KB of codes per K / V
constexpr uint32_t kHpQlatBytes = 32768;     // A * RP * 2 (f16 q_latent of one head)

constexpr uint32_t kHpMaxSlots = 64;         // hot groups of one (sequence, kv head)

struct HpChunk {
    uint32_t b, g, page_begin, n_pages;      // n_pages == 0: the CTA has no chunk
};

// Dependency counters per (sequence, kv head).
enum : uint32_t { HC_QLAT = 0, HC_SCORE = 1, HC_SCATTER = 2, HC_FIN = 3, HC_KINDS = 4 };

struct HpArgs {
    RunArgs r;                        // geometry, views, status
    uint32_t n_ctas;
    uint32_t n_empty;                 // (b, g) pairs with no hot and no cold blocks
    const FusedItem* items;           // per-CTA q_latent then contraction tiles, CSR by item_ptr
    const uint32_t* item_ptr;         // [n_ctas + 1]
    const FusedItem* first_item;      // [n_ctas]: items[item_ptr[c]] (type 0xFFFF when none), one load away
    const HpChunk* chunks;            // [n_ctas]
    const FusedHotGroup* groups;      // per-CTA hot groups, CSR by group_ptr
    const uint32_t* group_ptr;        // [n_ctas + 1]
    const uint32_t* slot_ptr;         // [B*Hkv + 1]: hot slots of (b, g) are slot_ptr[bg] .. slot_ptr[bg+1]
    const uint32_t* n_chunks;         // [B*Hkv]
    const uint32_t* hot_groups;       // [B*Hkv]
    const uint32_t* empty_bg;         // [n_empty]
    uint32_t* counters;               // [HC_KINDS][B*Hkv] + 1 exit counter
    __half* qlat16;                   // [B*Hkv][A*RP] scale*q.K_dict, f16
    float* wsum;                      // [B*Hkv][A*RP + 4]: per-atom weights w[atom][r], then l_cold[4]
    int* mkey;                        // [B*Hkv][RP] cold score maximum (ordered-int keys)
    float* ocold;                     // [B*Hkv][RP][D]
    float* sm;                        // [n_slots][RP] hot partials
    float* sl;
    float* so;                        // [n_slots][RP][D]
    uint64_t* trace;                  // optional [n_ctas][kTraceSlots]
    // split-KV combine fused into the step (a plan with an attached combiner):
    // every (b, g)'s last finisher pushes its (m, l, o) rows to every rank as
    // 8-byte (value bits, step tag) words and merges what all ranks pushed.
    // ll_world == 0: off.
    uint32_t ll_world, ll_rank, ll_rows;
    uint2* ll_recv[8];                // each rank's receive region [2][world][rows][D + 2] (peer mappings)
    uint32_t* ll_state;               // own [step tag, status]
};

// Shared memory of the head-partitioned kernel for (D, RP); 0 if unsupported.
size_t hp_smem_bytes(uint32_t D, uint32_t RP);
cudaError_t hp_occupancy(uint32_t D, uint32_t RP, int* blocks_per_sm);
cudaError_t launch_hp(const HpArgs& a, const CUtensorMap& tm_hk, const CUtensorMap& tm_hv, const CUtensorMap& tm_kd,
                      const CUtensorMap& tm_vd, const CUtensorMap& tm_kc, const CUtensorMap& tm_vc, cudaStream_t s);

// ---------------------------------------------------------------------------
// Split-KV combine over NVLink peer memory (weaver_combine.cu).
// ---------------------------------------------------------------------------
constexpr uint32_t kCombineMaxRanks = 8;

struct CombineArgs {
    uint32_t world, rank, rows, D;
    float* recv[kCombineMaxRanks];       // every rank's receive buffer (peer mappings; own at [rank])
    uint32_t* flags[kCombineMaxRanks];   // every rank's flags[world]
    uint32_t* state;                     // own [epoch, status]
};

cudaError_t launch_combine(const CombineArgs& c, const float* packed, __half* out, cudaStream_t s);

}  // namespace weaver
