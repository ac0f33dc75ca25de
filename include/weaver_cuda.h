/*
 * weaver_cuda.h — C ABI of the B200 (sm_100a) Weaver decode attention.
 *
 * This is the drop-in boundary for AetherNexus's Weaver path.  Every entry
 * point below names the reference interface it replaces (paths relative to the
 * reference project root).  Plain pointers, sizes and status codes only: no
 * CUDA runtime, torch or C++ types appear in the signatures (streams are
 * passed as `void*` holding a `cudaStream_t`, NULL = the legacy default
 * stream).
 *
 * Semantics (see also oracle/weaver_oracle.h, the CPU checker):
 *   hot  token: s = scale * q.K[row],                 value = V[row]
 *   cold token: s = sum_k cK_k * q_latent[iK_k],      value = sum_k cV_k * V_dict[iV_k]
 *               q_latent[a] = scale * q.K_dict[a] (computed here, fp32) unless
 *               the caller supplies it (reference mode, weaver.rs:142)
 *   out = softmax over all hot and cold tokens of the sequence, f16.
 * The reference-literal call (weaver_decode_host) is the special case
 * scale = 1, V = K, one code set for K and V, caller-supplied f16 q_latent.
 *
 * Thread safety: an engine and its plans belong to one host thread at a time
 * (the reference's `&mut self`, weaver.rs:139).  weaver_last_error() is per
 * host thread.
 */
#ifndef WEAVER_CUDA_H
#define WEAVER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WEAVER_ABI_VERSION 1

#if defined(__GNUC__)
#define WEAVER_EXPORT __attribute__((visibility("default")))
#else
#define WEAVER_EXPORT
#endif

/* ModelDims::BLOCK_SIZE / SPARSITY_K (nexus-core/src/types.rs:159-160) */
#define WEAVER_BLOCK_SIZE 16
#define WEAVER_SPARSITY_K 4
/* Block references carry a flag in bit 31 that is masked off
 * (nexus-core/src/weaver_kernel.metal:145,174). */
#define WEAVER_REF_MASK 0x7FFFFFFFu

/* ---- status codes (the reference returns Result<_, String>, weaver.rs:85,148) */
enum weaver_status {
    WEAVER_OK = 0,
    WEAVER_ERR_INVALID_ARGUMENT = 1, /* null pointer, inconsistent sizes */
    WEAVER_ERR_UNSUPPORTED = 2,      /* geometry outside what the kernels build for */
    WEAVER_ERR_MISALIGNED = 3,       /* a device view is not 16-byte aligned */
    WEAVER_ERR_OUT_OF_RANGE = 4,     /* a block reference or atom index is out of range */
    WEAVER_ERR_CUDA = 5,             /* a CUDA runtime error (text in weaver_last_error) */
    WEAVER_ERR_NO_DEVICE = 6,        /* no CUDA device / not an sm_100 device */
    WEAVER_ERR_TIMEOUT = 7,          /* a bounded device-side wait expired */
    WEAVER_ERR_CAPACITY = 8          /* a size exceeds a fixed capacity */
};

/* ---- reference ABI types ------------------------------------------------ */

/* SparseCode (types.rs:218-228; MSL mirror weaver_kernel.metal:34-37):
 * 4 u16 dictionary indices + 4 IEEE binary16 coefficients (raw bits). */
typedef struct weaver_sparse_code {
    uint16_t indices[4];
    uint16_t coeffs[4];
} weaver_sparse_code;

/* WeaverParams (types.rs:351-374; MSL mirror weaver_kernel.metal:40-51).
 * hot_count / cold_count are in 16-token blocks. */
typedef struct weaver_params {
    uint32_t q_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t block_size;
    uint32_t gqa_group;
    uint32_t hot_count;
    uint32_t cold_count;
    uint32_t dict_size;
    uint32_t sparsity_k;
    uint32_t _pad[3];
} weaver_params;

/* ModelDims (types.rs:150-164) as runtime values. */
typedef struct weaver_model_dims {
    uint32_t layers, q_heads, kv_heads, head_dim, hidden_size, intermediate_size;
    uint32_t vocab_size, block_size, sparsity_k, dict_size, gqa_group;
} weaver_model_dims;

/* LoomDescriptor (types.rs:311-328), repr(C) layout: 32 bytes. */
typedef struct weaver_loom_descriptor {
    uint8_t persona; /* Persona: 0 Planner, 1 Coder, 2 Critic, 3 Reviewer */
    uint8_t _pad0[3];
    uint32_t hot_count, cold_count, hot_refs_offset, cold_refs_offset, token_pos;
    uint32_t _pad[2];
} weaver_loom_descriptor;

/* FabricRegions (fabric.rs:73-117), byte offsets into the .aether file. */
typedef struct weaver_fabric_regions {
    uint64_t weights_offset, weights_size;
    uint64_t hot_pool_offset, hot_pool_size;
    uint64_t cold_pool_offset, cold_pool_size;
    uint64_t dict_offset, dict_size;
    uint64_t looms_offset, looms_size;
    uint64_t radix_offset, radix_size;
    uint64_t obs_offset, obs_size;
    uint64_t trace_offset, trace_size;
    uint64_t total_size;
} weaver_fabric_regions;

/* ---- host helpers ------------------------------------------------------ */

WEAVER_EXPORT int weaver_abi_version(void);
/* Text for the last failing call on this host thread (never NULL). */
WEAVER_EXPORT const char* weaver_last_error(void);
WEAVER_EXPORT const char* weaver_status_string(int status);

/* ModelDims presets: "llama8b" (the trait defaults), "granite2b", "qwen05b",
 * "deepseek_r1_1_5b" (types.rs:150-204). */
WEAVER_EXPORT int weaver_model_dims_preset(const char* name, weaver_model_dims* out);
/* WeaverParams::from_loom (types.rs:380-395). */
WEAVER_EXPORT int weaver_params_from_loom(const weaver_model_dims* dims, const weaver_loom_descriptor* loom,
                            weaver_params* out);
/* FabricRegions::compute (fabric.rs:124-186). */
WEAVER_EXPORT int weaver_fabric_regions_compute(const weaver_model_dims* dims, weaver_fabric_regions* out);

/* ---- engine: WeaverEngine (weaver.rs:27-322) ----------------------------- */

typedef struct weaver_engine weaver_engine;

/* WeaverEngine::new (weaver.rs:85-132): binds CUDA device `device`, checks it
 * is an sm_100 part, creates the engine's stream.  No metallib path: the
 * kernels are linked into this library. */
WEAVER_EXPORT int weaver_engine_create(int device, weaver_engine** out);
WEAVER_EXPORT void weaver_engine_destroy(weaver_engine* engine);
/* WeaverEngine::device_name (weaver.rs:314-316). */
WEAVER_EXPORT int weaver_engine_device_name(const weaver_engine* engine, char* buf, size_t len);
/* WeaverEngine::max_threads_per_threadgroup (weaver.rs:319-321). */
WEAVER_EXPORT int weaver_engine_max_threads_per_block(const weaver_engine* engine, uint64_t* out);

/* WeaverEngine::decode (weaver.rs:139-237), same arguments and meaning:
 * host slices (lengths in elements) are copied into engine-owned device
 * buffers that grow on demand (weaver.rs:155-203), the step runs, and the
 * call blocks until `out` (q_heads*head_dim f16) is filled (weaver.rs:227-236).
 *   q_exact    [q_heads][head_dim] f16
 *   q_latent   [q_heads][dict_size] f16 (caller-projected query)
 *   hot_pool   [blocks][16][kv_heads][head_dim] f16, K and V are the same rows
 *   cold_pool  [blocks][16][kv_heads] SparseCode, one code serves K and V
 *   loom_refs  [hot_count + cold_count] block refs (bit 31 ignored)
 *   dictionary [kv_heads][dict_size][head_dim] f16
 * Unlike the reference, refs beyond the supplied pools are rejected with
 * WEAVER_ERR_OUT_OF_RANGE, and params.head_dim / params.dict_size are honoured
 * (the reference shader hard-codes 128 / 512, weaver_kernel.metal:23-26). */
WEAVER_EXPORT int weaver_decode_host(weaver_engine* engine, const uint16_t* q_exact, size_t q_exact_len,
                       const uint16_t* q_latent, size_t q_latent_len, const uint16_t* hot_pool,
                       size_t hot_pool_len, const weaver_sparse_code* cold_pool,
                       size_t cold_pool_len, const uint32_t* loom_refs, size_t loom_refs_len,
                       const uint16_t* dictionary, size_t dictionary_len,
                       const weaver_params* params, uint16_t* out, size_t out_len);

/* ---- device-resident batched decode (Fabric sub-views in HBM) ------------
 * The reference copies every input on every call (weaver.rs:155-196); here
 * the pools stay resident and a step passes device views.  A plan fixes the
 * geometry and the per-sequence block counts (the loom_refs split,
 * weaver_kernel.metal:143,172) and owns all scratch; weaver_run only
 * launches kernels on the given stream (no allocation, no host sync), so a
 * run can be captured in a CUDA graph and replayed for every layer. */

enum weaver_flags {
    WEAVER_FLAG_CAUSAL = 1u,          /* nq>1: query j sees hot positions < Th-nq+1+j (ops.metal:549) */
    WEAVER_FLAG_QLATENT_INPUT = 2u,   /* use views.q_latent (f16) instead of q.K_dict */
    WEAVER_FLAG_PARTIALS = 4u         /* write (m, l, o) fp32 partials instead of out */
};

typedef struct weaver_shape {
    uint32_t num_seqs;    /* B */
    uint32_t num_queries; /* nq query tokens per sequence (1 = decode, >1 = speculative verify) */
    uint32_t q_heads;     /* Hq */
    uint32_t kv_heads;    /* Hkv; Hq % Hkv == 0 */
    uint32_t head_dim;    /* 64 or 128 */
    uint32_t dict_size;   /* atoms per dictionary, <= 65536 */
    float scale;          /* 1/sqrt(head_dim) for model semantics, 1 for the reference kernel */
    uint32_t flags;       /* weaver_flags */
} weaver_shape;

typedef struct weaver_views {
    const void* q;        /* f16 [B][nq][Hq][d] */
    const void* q_latent; /* f16 [B][nq][Hq][A], only with WEAVER_FLAG_QLATENT_INPUT */
    const void* hot_k;    /* f16 [hot_pool_blocks][16][Hkv][d] */
    const void* hot_v;    /* f16, same layout (may equal hot_k) */
    uint64_t hot_pool_blocks;
    const uint32_t* hot_refs;  /* concatenated per-sequence hot block refs (plan indptr) */
    const weaver_sparse_code* cold_k; /* [cold_pool_blocks][16][Hkv] */
    const weaver_sparse_code* cold_v; /* same layout (may equal cold_k) */
    uint64_t cold_pool_blocks;
    const uint32_t* cold_refs; /* concatenated per-sequence cold block refs */
    const void* k_dict;   /* f16 [Hkv][A][d] (unused with WEAVER_FLAG_QLATENT_INPUT) */
    const void* v_dict;   /* f16 [Hkv][A][d] */
    uint64_t dict_head_stride; /* elements between kv heads' dictionaries: A*d, or 0 (shared) */
    void* out;            /* f16 [B][nq][Hq][d] */
    float* part_m;        /* WEAVER_FLAG_PARTIALS: [B][nq][Hq] running max */
    float* part_l;        /*                       [B][nq][Hq] sum of exp */
    float* part_o;        /*                       [B][nq][Hq][d] unnormalised output */
} weaver_views;

typedef struct weaver_plan weaver_plan;

/* hot_indptr / cold_indptr: host arrays of B+1 block offsets into hot_refs /
 * cold_refs (sequence b owns [indptr[b], indptr[b+1])).  A plan keeps its
 * device, not its engine: it may be run and destroyed after the engine that
 * created it has been destroyed (as garbage-collected hosts do). */
WEAVER_EXPORT int weaver_plan_create(weaver_engine* engine, const weaver_shape* shape,
                       const uint32_t* hot_indptr, const uint32_t* cold_indptr,
                       weaver_plan** out);
WEAVER_EXPORT void weaver_plan_destroy(weaver_plan* plan);
/* Launch one decode step on `stream` (cudaStream_t, NULL = default).  The
 * plan picks the step's form at creation: one kernel when one kv head's
 * q_latent fits shared memory or the cold context is short; else (2^19 or
 * more cold (token, kv head) pairs, or more than 8 query rows per kv head) a
 * pipeline of kernels on `stream`, whose hot pass runs on a stream the plan
 * owns, forked from `stream` by an event at the start of the step and joined
 * back before the merge (CUDA-graph capturable; the order on `stream` is
 * kept).  Only one weaver_run of a plan may be in flight at a time. */
WEAVER_EXPORT int weaver_run(weaver_plan* plan, const weaver_views* views, void* stream);
/* Number of kernels one weaver_run launches. */
WEAVER_EXPORT int weaver_plan_kernel_count(const weaver_plan* plan);
/* Synchronises the plan's last stream, then reads and clears the device status
 * word: WEAVER_OK, WEAVER_ERR_OUT_OF_RANGE (a block ref or atom index was out
 * of range; that token or code term was skipped) or WEAVER_ERR_TIMEOUT. */
WEAVER_EXPORT int weaver_plan_status(weaver_plan* plan);

/* The reference-shaped, synchronous call for the model semantics: every
 * pointer in `host_views` is a HOST pointer (sizes follow from the shape, the
 * indptr arrays and views.hot_pool_blocks / cold_pool_blocks); all inputs are
 * copied into engine-owned device buffers that grow on demand, one decode
 * step runs, and out (or the partials) are copied back before returning
 * (weaver.rs:139-237 with separate K/V pools, codes and dictionaries).  Pinned
 * host memory makes the copies asynchronous DMA. */
WEAVER_EXPORT int weaver_decode_host_batch(weaver_engine* engine, const weaver_shape* shape,
                                           const uint32_t* hot_indptr, const uint32_t* cold_indptr,
                                           const weaver_views* host_views);

/* Phase timeline of the last run of a single-kernel plan, for profiling: when
 * the plan was created with WEAVER_TRACE=1 in the environment, every CTA
 * records %globaltimer stamps (ns) of its phase boundaries.  Writes
 * n_ctas * (*slots_per_cta) values to `out` (synchronises).  No counterpart in
 * the reference (its timing is host wall clock, bench.rs:246-263). */
WEAVER_EXPORT int weaver_plan_trace(weaver_plan* plan, uint64_t* out, size_t n, uint32_t* slots_per_cta);

/* ---- allocation-free hot-pool decode ---------------------------------------
 * No counterpart in the reference.  For callers that must not allocate device
 * memory while they run — a serving loop that fixes its device-memory budget
 * at start-up and forbids later cudaMalloc/cudaFree, or a host whose device
 * memory belongs to another allocator — and so cannot create a plan (plans
 * allocate their scratch).  Exact split-KV attention of one decode step over
 * the hot pool only (one sequence, one query token): q [q_heads][head_dim] f16,
 * hot_k / hot_v [hot_pool_blocks][16][kv_heads][head_dim] f16, hot_refs
 * [n_blocks] (bit 31 ignored), out [q_heads][head_dim] f16, all device
 * pointers; out = softmax(scale * q.K) . V like weaver_run on a plan without
 * cold blocks.  An out-of-range block ref is skipped and ORs 1 into the device
 * word *bad_ref_flag (the caller zeroes it).  The per-chunk partials live in a
 * fixed 2 MiB array inside this library (every GPU that loads the library
 * holds it until exit): q_heads * (head_dim + 2) must be <= 2^19 and n_blocks
 * <= 2^24, else WEAVER_ERR_CAPACITY; kv_heads must divide q_heads with a group
 * of 1, 2, 4 or 8 and head_dim must be 64 or 128, else WEAVER_ERR_UNSUPPORTED.
 * The first call on a device looks up the array's device address and should
 * come before any stream capture.  All calls share the array: calls whose
 * kernels overlap on the GPU race and must be serialised by the caller.
 * Calls no allocator.  Returns a status code only (weaver_last_error is not
 * updated). */
WEAVER_EXPORT int weaver_hot_decode_noalloc(uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim, float scale,
                                            const void* q, const void* hot_k, const void* hot_v,
                                            uint64_t hot_pool_blocks, const uint32_t* hot_refs, uint32_t n_blocks,
                                            void* out, uint32_t* bad_ref_flag, void* stream);

/* ---- split-KV combine (multi-GPU long context) ---------------------------
 * Log-sum-exp merge of n_parts partial results for `rows` query rows:
 * m, l [n_parts][rows], o [n_parts][rows][head_dim] fp32 (device) -> out f16
 * [rows][head_dim] (device).  No counterpart in the reference (single device);
 * it combines the per-GPU (m, l, o) that WEAVER_FLAG_PARTIALS produces. */
WEAVER_EXPORT int weaver_merge_partials(uint32_t n_parts, uint32_t rows, uint32_t head_dim, const float* m,
                          const float* l, const float* o, void* out, void* stream);

/* The same merge over parts laid out `part_stride` floats apart: part p's
 * m at m + p*part_stride, l at l + p*part_stride, o at o + p*part_stride.
 * One all-gather of a packed per-rank buffer [m rows | l rows | o rows*d]
 * feeds it directly (m = buf, l = buf + rows, o = buf + 2*rows,
 * part_stride = rows*(head_dim + 2)).  No counterpart in the reference. */
WEAVER_EXPORT int weaver_merge_partials_strided(uint32_t n_parts, uint32_t rows, uint32_t head_dim, const float* m,
                          const float* l, const float* o, uint64_t part_stride, void* out, void* stream);

/* ---- split-KV combine over NVLink peer memory (the GPUs of one node) -----
 * One combine object per rank: it owns a receive buffer that the other ranks
 * write into directly (CUDA IPC peer mappings).  weaver_combine_run takes
 * this rank's packed partials [m rows | l rows | o rows*head_dim] (fp32,
 * device, 16-byte aligned; what a plan with WEAVER_FLAG_PARTIALS writes when
 * part_m/l/o point into one buffer), writes them into every rank's buffer,
 * signals, waits for every rank (bounded: 1 s, then WEAVER_ERR_TIMEOUT from
 * weaver_combine_status) and writes the merged f16 [rows][head_dim] to out.
 * Every rank must call weaver_combine_run once per step, in the same order;
 * one kernel launch, capturable in a CUDA graph.  After a wait has expired
 * (WEAVER_ERR_TIMEOUT) the combiner is unusable: a late peer may still
 * write into its buffers, so every later run writes zeros and touches no peer
 * memory; every rank must destroy it and create a new one.  Setup: create, export
 * weaver_combine_ipc_handle (WEAVER_IPC_HANDLE_BYTES bytes), exchange the
 * handles between ranks (any host channel), weaver_combine_open_peer for
 * every other rank.  Destroy only after every rank has finished its last
 * run.  No counterpart in the reference (single device). */
typedef struct weaver_combine weaver_combine;
#define WEAVER_IPC_HANDLE_BYTES 64
WEAVER_EXPORT int weaver_combine_create(weaver_engine* engine, uint32_t world, uint32_t rank, uint32_t rows,
                                        uint32_t head_dim, weaver_combine** out);
WEAVER_EXPORT void weaver_combine_destroy(weaver_combine* c);
WEAVER_EXPORT int weaver_combine_ipc_handle(weaver_combine* c, void* handle_out);
WEAVER_EXPORT int weaver_combine_open_peer(weaver_combine* c, uint32_t peer, const void* handle);
WEAVER_EXPORT int weaver_combine_run(weaver_combine* c, const float* packed, void* out, void* stream);
WEAVER_EXPORT int weaver_combine_status(weaver_combine* c);

/* The same split-KV combine fused into the decode step: after attaching, every
 * weaver_run of `plan` (this rank's shard of the blocks, created WITHOUT
 * WEAVER_FLAG_PARTIALS, rows = num_seqs*num_queries*q_heads and head_dim equal
 * to the combiner's) writes the output merged over all ranks to views.out.
 * Each (sequence, kv head)'s last finisher in the step kernel pushes its
 * (m, l, o) rows into every rank's receive buffer as 8-byte (value, step tag)
 * words over NVLink and merges all ranks' rows as they arrive (bounded wait:
 * WEAVER_ERR_TIMEOUT from weaver_plan_status, and the combiner is then
 * unusable, as above).  One kernel per step, no separate combine launch.
 * Every rank must run its plan once per step, in the same order.  Needs the
 * single-kernel step (weaver_plan_kernel_count == 1), else
 * WEAVER_ERR_UNSUPPORTED; c = NULL detaches.  No counterpart in the
 * reference (single device). */
WEAVER_EXPORT int weaver_plan_attach_combine(weaver_plan* plan, weaver_combine* c);

/* ---- atom selection: Distiller::distill_block (distiller.rs:171-246) ----
 * For n_rows f16 token rows [n_rows][head_dim] (device; row i belongs to kv
 * head i % kv_heads, distiller.rs:199): dot with all atoms of its head
 * (f32, dimension order), keep the top 4 by score descending, ties by
 * ascending atom index, coefficient = f16(dot).  Writes n_rows SparseCodes
 * (device).  Bit-exact with the CPU rule. */
WEAVER_EXPORT int weaver_distill(const void* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t head_dim,
                   const void* dictionary, uint32_t dict_size, uint64_t dict_head_stride,
                   weaver_sparse_code* out_codes, void* stream);

/* ---- device-resident Fabric: fabric.rs:124-186 / 347-420, types.rs:311-328 ----
 * The Hot / Cold / Dictionary regions live on the device for the whole run
 * (the reference maps the .aether file and copies every region into its
 * Metal buffers on every call, weaver.rs:155-196).  The device layout adds
 * a layer dimension and, optionally, separate V regions (the reference's
 * layout has neither: V rows = K rows, one code set, one dictionary).  One
 * allocation holds every layer's pools, codes and dictionaries (256-byte
 * aligned views) and the block-reference array that LoomDescriptor offsets
 * index. */
typedef struct weaver_fabric_geometry {
    uint32_t layers, kv_heads, head_dim, dict_size;
    uint64_t hot_blocks, cold_blocks; /* per layer, 16-token blocks */
    uint32_t separate_v;              /* 0: the V views alias the K views */
    uint32_t _pad;
    uint64_t max_block_refs;          /* capacity of the u32 block-reference array */
} weaver_fabric_geometry;

/* One layer's device views, ready for weaver_views. */
typedef struct weaver_fabric_layer {
    void* hot_k;
    void* hot_v;
    weaver_sparse_code* cold_k;
    weaver_sparse_code* cold_v;
    void* k_dict;
    void* v_dict;
    uint64_t hot_pool_blocks, cold_pool_blocks;
} weaver_fabric_layer;

typedef struct weaver_device_fabric weaver_device_fabric;
WEAVER_EXPORT int weaver_device_fabric_create(int device, const weaver_fabric_geometry* geometry,
                                              weaver_device_fabric** out);
WEAVER_EXPORT void weaver_device_fabric_destroy(weaver_device_fabric* fabric);
WEAVER_EXPORT int weaver_device_fabric_layer(const weaver_device_fabric* fabric, uint32_t layer, weaver_fabric_layer* out);
WEAVER_EXPORT int weaver_device_fabric_block_refs(const weaver_device_fabric* fabric, uint32_t** refs,
                                                  uint64_t* capacity);
/* Copy the Hot pool, Cold pool and Dictionary regions of an .aether image in
 * host memory (e.g. the caller's mmap of the file; offsets and sizes from
 * FabricRegions, weaver_fabric_regions_compute) into layer `layer`: its K
 * views (which = 0) or, in a fabric with separate_v, its V views (which = 1).
 * A region larger than the layer's view is refused. */
WEAVER_EXPORT int weaver_device_fabric_upload_aether(weaver_device_fabric* fabric, uint32_t layer, const void* image,
                                                     uint64_t image_bytes, const weaver_fabric_regions* regions,
                                                     uint32_t which, void* stream);
/* Copy n block refs (host) to positions offset.. of the block-reference array. */
WEAVER_EXPORT int weaver_device_fabric_upload_refs(weaver_device_fabric* fabric, const uint32_t* refs, uint64_t n,
                                                   uint64_t offset, void* stream);
/* LoomDescriptor -> a plan's page tables: loom i's hot refs are block refs
 * [hot_refs_offset, + hot_count), its cold refs [cold_refs_offset, +
 * cold_count) (types.rs:320-323).  Writes the host arrays hot_indptr /
 * cold_indptr (n + 1 entries; sequence i = loom i) and gathers the refs on
 * the device into hot_refs / cold_refs (capacities in entries). */
WEAVER_EXPORT int weaver_loom_page_tables(const weaver_device_fabric* fabric, const weaver_loom_descriptor* looms,
                                          uint32_t n, uint32_t* hot_indptr, uint32_t* cold_indptr, uint32_t* hot_refs,
                                          uint64_t hot_capacity, uint32_t* cold_refs, uint64_t cold_capacity,
                                          void* stream);

/* ---- the full loop's exact multi-query attention ----
 * Ops::multihead_attention (ops.rs:433-460, kernel ops.metal:528-616), the
 * attention of every layer of the full decode loop (inference.rs:552-562),
 * speculative verify included: q [num_queries][q_heads][head_dim], k_cache /
 * v_cache [>= total_kv_len][kv_heads][head_dim], out [num_queries][q_heads]
 * [head_dim], all f16 on the device, 16-byte aligned.  Query qi attends to
 * positions < total_kv_len - num_queries + 1 + qi; scale 1/sqrt(head_dim);
 * q head h reads kv head h / (q_heads / kv_heads).  head_dim 64 or 128;
 * total_kv_len >= num_queries (the reference's unsigned arithmetic wraps
 * below that) and, unlike the reference's 4096-entry score array, any cache
 * length.  Asynchronous on `stream`; the engine's grow-only scratch holds
 * the split-KV partials, so one call at a time per engine. */
WEAVER_EXPORT int weaver_multihead_attention(weaver_engine* engine, const void* q, const void* k_cache,
                                             const void* v_cache, void* out, uint32_t total_kv_len, uint32_t head_dim,
                                             uint32_t q_heads, uint32_t kv_heads, uint32_t num_queries, void* stream);

/* weaver_distill on the tensor cores with its diagnostics: the scores are
 * computed as a tokens x atoms GEMM (tcgen05.mma), each row's 8 best kept,
 * and the candidates that an error bound cannot rule out re-scored exactly
 * (dimension order), so the codes equal weaver_distill's bit for bit.  diag:
 * 4 device words the caller zeroes: [0] the largest |approximate - exact| /
 * bound over the re-scored atoms (float bits; must stay below 1), [1] rows
 * whose candidates the bound could not confine to 8 atoms (finished by the
 * exact full scan), [2..3] status and first expired wait.  weaver_distill
 * and weaver_migrate_blocks take this path whenever it applies (head_dim 64
 * or 128, at least 4 atoms, dict_head_stride a multiple of head_dim);
 * WEAVER_ERR_UNSUPPORTED otherwise.  No counterpart in the reference. */
WEAVER_EXPORT int weaver_distill_stats(const void* rows, uint32_t n_rows, uint32_t kv_heads, uint32_t head_dim,
                                       const void* dictionary, uint32_t dict_size, uint64_t dict_head_stride,
                                       weaver_sparse_code* out_codes, uint32_t* diag, void* stream);

/* ---- hot -> cold migration (the Distiller's REM cycle, on the GPU) ---------
 * Distiller::evaluate_entropy's proxy (distiller.rs:97-159, threshold
 * MemoryConfig::distill_entropy_threshold, types.rs:45-53): out[i] = the
 * variance of the 16*kv_heads*head_dim f16 values of hot block i (device
 * pool [blocks][16][kv_heads][head_dim]; sum and squared deviations in fp64,
 * the result rounded to f32; 0 for an all-zero block), for i < n_blocks. */
WEAVER_EXPORT int weaver_block_entropy(const void* hot_pool, uint64_t n_blocks, uint32_t kv_heads, uint32_t head_dim,
                                       float* out, void* stream);
/* Distiller::distill_block (distiller.rs:171-246) for a list of blocks, with
 * the write into the cold pool: for i < n, the 16*kv_heads K rows of hot block
 * src_blocks[i] are encoded against k_dict (the selection of weaver_distill:
 * top 4 by fp32 dot, ties by ascending atom, coefficient f16(dot)) into cold
 * block dst_blocks[i] of cold_k, and the V rows against v_dict into cold_v
 * (pass the same pool, dictionary and code pointers twice for the reference's
 * single K=V layout).  src_blocks / dst_blocks are device arrays of n <= 65535
 * entries; an entry beyond hot_pool_blocks / cold_pool_blocks is skipped and
 * ORs 1 into the device word *bad_flag (the caller zeroes it).  Asynchronous
 * on `stream`, so it can run on a side stream next to the decode steps. */
WEAVER_EXPORT int weaver_migrate_blocks(const void* hot_k, const void* hot_v, uint64_t hot_pool_blocks,
                                        const uint32_t* src_blocks, const uint32_t* dst_blocks, uint32_t n,
                                        uint32_t kv_heads, uint32_t head_dim, const void* k_dict, const void* v_dict,
                                        uint32_t dict_size, uint64_t dict_head_stride, weaver_sparse_code* cold_k,
                                        weaver_sparse_code* cold_v, uint64_t cold_pool_blocks, uint32_t* bad_flag,
                                        void* stream);

/* ---- self-test of the bounded device-side waits --------------------------
 * No counterpart in the reference (its kernel has no waits and no error
 * path).  Every wait in this library's kernels gives up after a time limit,
 * records DEVERR_TIMEOUT (bit 4) in the launch's status word and lets the
 * kernel finish, so a lost peer or arrival surfaces as WEAVER_ERR_TIMEOUT
 * with the CUDA context intact.  This call runs the three kinds of wait on
 * the current device (an mbarrier phase nobody completes, a counter nobody
 * increments, a peer (value, tag) word nobody writes) with a limit of
 * `limit_us` microseconds (1..10^6) each, and reports in *expired_mask
 * (bits 0-2) which of them gave up, in waited_ns[3] how long each waited and
 * in status_words[6] the three status pairs they recorded (either pointer may
 * be NULL).  Allocates a 256-byte buffer; synchronises the device. */
WEAVER_EXPORT int weaver_wait_selftest(uint32_t limit_us, uint32_t* expired_mask, uint64_t* waited_ns,
                                       uint32_t* status_words);

#ifdef __cplusplus
}
#endif

#endif /* WEAVER_CUDA_H */
