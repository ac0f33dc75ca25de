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
    // scratch
    float* qlat;     // [B][Hkv][A][RP]
    float* w;        // [B][Hkv][A][RP]
    float* scores;   // [Hkv][cold_tokens][RP]
    float* cmax;     // [n_cold_items][Hkv][RP]
    float* csum;     // [n_cold_items][Hkv][RP]
    float* ocold;    // [B][Hkv][n_atom_tiles][RP][D]
    float* hm;       // [n_hot_items][Hkv][RP]
    float* hl;
    float* ho;       // [n_hot_items][Hkv][RP][D]
    uint32_t* status;
};

// Kernel launchers (weaver_kernels.cu).  Each returns the launch error.
cudaError_t launch_qlat(const RunArgs& a, const CUtensorMap& tm_kdict, cudaStream_t s);
cudaError_t launch_qlat_import(const RunArgs& a, cudaStream_t s);
cudaError_t launch_cold_score(const RunArgs& a, cudaStream_t s);
cudaError_t launch_cold_scatter(const RunArgs& a, cudaStream_t s);
cudaError_t launch_cold_contract(const RunArgs& a, const CUtensorMap& tm_vdict, cudaStream_t s);
cudaError_t launch_hot(const RunArgs& a, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                       uint32_t row_groups, cudaStream_t s);
cudaError_t launch_merge(const RunArgs& a, cudaStream_t s);
cudaError_t launch_merge_partials(uint32_t n_parts, uint32_t rows, uint32_t D, const float* m,
                                  const float* l, const float* o, __half* out, cudaStream_t s);
cudaError_t launch_distill(const __half* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t D,
                           const __half* dict, uint32_t A, uint64_t dict_head_stride,
                           uint4* out, cudaStream_t s);

// Rows handled by one hot CTA (the hot kernel is built for these).
constexpr uint32_t kHotRows = 8;

}  // namespace weaver
