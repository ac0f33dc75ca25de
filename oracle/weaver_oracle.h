/*
 * weaver_oracle.h — CPU oracle for the Weaver decode attention.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against; it is never linked into, loaded by, or called from the
 * product library (aether_nexus_b200/libweaver_cuda.so).  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it.
 *
 * It restates, in plain C, the algorithm of the reference:
 *   - nexus-core/src/weaver_kernel.metal:118-240  (weaver_decode: hot pass,
 *     cold pass, finalize) — "literal" mode, lane order reproduced exactly;
 *   - the same algorithm generalised to the configuration semantics (scale,
 *     separate hot K/V pools, separate K/V SparseCode sets, per-head K/V
 *     dictionaries, q_latent computed from K_dict, multi-query causal rule of
 *     nexus-core/src/ops.metal:546-555, batched paged page tables);
 *   - atom selection of nexus-core/src/distiller.rs:185-234 (top-4 by dot);
 *   - the entropy proxy of nexus-core/src/distiller.rs:126-159.
 *
 * Parity pinning: see oracle/ref_driver.cpp (the reference kernel source
 * compiled as C++) and tests/golden/.
 */
#ifndef WEAVER_ORACLE_H
#define WEAVER_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 16-byte SparseCode: nexus-core/src/types.rs:218-228 (4 x u16 atom index,
 * 4 x f16 coefficient, stored as raw IEEE binary16 bits). */
typedef struct oracle_sparse_code {
    uint16_t indices[4];
    uint16_t coeffs[4];
} oracle_sparse_code;

/* WeaverParams: nexus-core/src/types.rs:351-374 (12 x u32 = 48 bytes). */
typedef struct oracle_weaver_params {
    uint32_t q_heads, kv_heads, head_dim, block_size, gqa_group;
    uint32_t hot_count, cold_count, dict_size, sparsity_k;
    uint32_t pad[3];
} oracle_weaver_params;

/* IEEE binary16 <-> binary32, round-to-nearest-even (the `half` crate's
 * f16::from_f32 / f32::from, and Metal's half(float) conversion). */
float oracle_h2f(uint16_t h);
uint16_t oracle_f2h(float f);

/* Literal restatement of weaver_decode (weaver_kernel.metal:118-240) for
 * one decode step: q_exact [q_heads][d], q_latent [q_heads][dict_size],
 * hot_pool [blocks][16][kv_heads][d] (K and V are the same rows, :163),
 * cold_pool [blocks][16][kv_heads] (one code set serves K and V, :182-218),
 * loom_refs [hot_count + cold_count] (bit 31 masked, :145,174),
 * dictionary [kv_heads][dict_size][d], out [q_heads][d] f16.
 * hot_pool_blocks / cold_pool_blocks bound the physical block ids (the
 * reference has no bound check; out-of-range ids return -1 here).
 * Returns 0 on success. */
int oracle_literal_decode(const uint16_t* q_exact, const uint16_t* q_latent,
                          const uint16_t* hot_pool, uint64_t hot_pool_blocks,
                          const oracle_sparse_code* cold_pool, uint64_t cold_pool_blocks,
                          const uint32_t* loom_refs, const uint16_t* dictionary,
                          const oracle_weaver_params* p, uint16_t* out);

/* Configuration-mode problem description (batched, paged, multi-query). */
typedef struct oracle_decode_desc {
    uint32_t num_seqs;      /* B */
    uint32_t num_queries;   /* nq query tokens per sequence (1 = decode) */
    uint32_t q_heads, kv_heads, head_dim, dict_size;
    float scale;            /* multiplies q.k (hot) and q.K_dict (cold) */
    uint32_t causal;        /* nq>1: query j sees hot positions < Th-nq+1+j */
    const uint16_t* q;          /* [B][nq][Hq][d] f16 */
    const uint16_t* q_latent;   /* optional [B][nq][Hq][A] f16, used as is */
    const uint16_t* hot_k;      /* [hot_pool_blocks][16][Hkv][d] f16 */
    const uint16_t* hot_v;
    uint64_t hot_pool_blocks;
    const uint32_t* hot_refs;   /* block refs, seq b owns [hot_indptr[b], hot_indptr[b+1]) */
    const uint32_t* hot_indptr; /* B+1 */
    const oracle_sparse_code* k_codes; /* [cold_pool_blocks][16][Hkv] */
    const oracle_sparse_code* v_codes;
    uint64_t cold_pool_blocks;
    const uint32_t* cold_refs;
    const uint32_t* cold_indptr;
    const uint16_t* k_dict;     /* [Hkv][A][d] f16 (head stride below) */
    const uint16_t* v_dict;
    uint64_t dict_head_stride;  /* elements between heads; 0 = one shared dictionary */
    uint16_t* out;              /* optional [B][nq][Hq][d] f16 */
    float* out_m;               /* optional partials: running max   [B][nq][Hq] */
    float* out_l;               /*                    sum of exp    [B][nq][Hq] */
    float* out_o;               /*                    unnormalised  [B][nq][Hq][d] */
} oracle_decode_desc;

/* Exact reference in double precision (single online softmax over the hot
 * then the cold tokens, cold values reconstructed per token as in
 * weaver_kernel.metal:192-221).  Returns 0, or -1 on an out-of-range index. */
int oracle_config_decode_f64(const oracle_decode_desc* d);

/* The same algorithm in fp32, parallelised over query rows with OpenMP
 * (threads <= 0: all available).  This is the timed CPU baseline. */
int oracle_config_decode_f32(const oracle_decode_desc* d, int threads);

/* Atom selection of distiller.rs:185-234 for n_rows token rows of length d.
 * Row i belongs to kv head (i % kv_heads) (distiller.rs:199).  For every row:
 * dot with all dict_size atoms of its head (f32, summed in dimension order
 * from -0.0 like Rust's f32 Sum), rank by score descending with ties broken
 * by ascending atom index (NaN ranks last), keep the top 4 (index, f16(dot)).
 * Rows with fewer than 4 atoms keep zero codes in the unused slots. */
int oracle_distill_rows(const uint16_t* rows, uint32_t n_rows, uint32_t kv_heads,
                        uint32_t head_dim, const uint16_t* dict, uint32_t dict_size,
                        uint64_t dict_head_stride, oracle_sparse_code* out);

/* distiller.rs:126-159: variance of the f16 values (f64), 0 for all-zero. */
float oracle_block_entropy(const uint16_t* values, uint64_t n);

/* ops.metal:528-616 (multihead_attention, the full loop's attention,
 * inference.rs:552-562): q [nq][q_heads][d], k_cache / v_cache
 * [>= total_kv_len][kv_heads][d] f16; query qi attends to positions
 * < total_kv_len - nq + 1 + qi; scale 1/sqrt(d); three-pass softmax with the
 * kernel's threadgroup reductions (min(64, d) threads: strided partials, then
 * a halving tree); out [nq][q_heads][d] f16.  Returns -2 for total_kv_len <
 * nq or q_heads not a multiple of kv_heads. */
int oracle_mha(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, uint16_t* out,
               uint32_t total_kv_len, uint32_t head_dim, uint32_t q_heads, uint32_t kv_heads,
               uint32_t num_queries);

#ifdef __cplusplus
}
#endif

#endif /* WEAVER_ORACLE_H */
