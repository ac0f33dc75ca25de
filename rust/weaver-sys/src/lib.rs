//! Raw bindings to `libweaver_cuda.so`, one-to-one with `include/weaver_cuda.h`
//! (kept in step by `tests/test_rust_binding.py`, which parses both files).
//!
//! The structs mirror the reference's ABI types: `SparseCode`
//! (`nexus-core/src/types.rs:218-228`), `WeaverParams` (`types.rs:351-374`),
//! `ModelDims` (`types.rs:150-164`), `LoomDescriptor` (`types.rs:311-328`) and
//! `FabricRegions` (`fabric.rs:73-117`).  Streams are `cudaStream_t` passed as
//! `*mut c_void` (null = the legacy default stream).
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const WEAVER_ABI_VERSION: c_int = 1;
pub const WEAVER_BLOCK_SIZE: u32 = 16;
pub const WEAVER_SPARSITY_K: u32 = 4;
pub const WEAVER_REF_MASK: u32 = 0x7FFF_FFFF;
pub const WEAVER_IPC_HANDLE_BYTES: usize = 64;

pub const WEAVER_OK: c_int = 0;
pub const WEAVER_ERR_INVALID_ARGUMENT: c_int = 1;
pub const WEAVER_ERR_UNSUPPORTED: c_int = 2;
pub const WEAVER_ERR_MISALIGNED: c_int = 3;
pub const WEAVER_ERR_OUT_OF_RANGE: c_int = 4;
pub const WEAVER_ERR_CUDA: c_int = 5;
pub const WEAVER_ERR_NO_DEVICE: c_int = 6;
pub const WEAVER_ERR_TIMEOUT: c_int = 7;
pub const WEAVER_ERR_CAPACITY: c_int = 8;

pub const WEAVER_FLAG_CAUSAL: u32 = 1;
pub const WEAVER_FLAG_QLATENT_INPUT: u32 = 2;
pub const WEAVER_FLAG_PARTIALS: u32 = 4;

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct weaver_sparse_code {
    pub indices: [u16; 4],
    pub coeffs: [u16; 4],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct weaver_params {
    pub q_heads: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub block_size: u32,
    pub gqa_group: u32,
    pub hot_count: u32,
    pub cold_count: u32,
    pub dict_size: u32,
    pub sparsity_k: u32,
    pub _pad: [u32; 3],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct weaver_model_dims {
    pub layers: u32,
    pub q_heads: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub hidden_size: u32,
    pub intermediate_size: u32,
    pub vocab_size: u32,
    pub block_size: u32,
    pub sparsity_k: u32,
    pub dict_size: u32,
    pub gqa_group: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct weaver_loom_descriptor {
    pub persona: u8,
    pub _pad0: [u8; 3],
    pub hot_count: u32,
    pub cold_count: u32,
    pub hot_refs_offset: u32,
    pub cold_refs_offset: u32,
    pub token_pos: u32,
    pub _pad: [u32; 2],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct weaver_fabric_regions {
    pub weights_offset: u64,
    pub weights_size: u64,
    pub hot_pool_offset: u64,
    pub hot_pool_size: u64,
    pub cold_pool_offset: u64,
    pub cold_pool_size: u64,
    pub dict_offset: u64,
    pub dict_size: u64,
    pub looms_offset: u64,
    pub looms_size: u64,
    pub radix_offset: u64,
    pub radix_size: u64,
    pub obs_offset: u64,
    pub obs_size: u64,
    pub trace_offset: u64,
    pub trace_size: u64,
    pub total_size: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq)]
pub struct weaver_shape {
    pub num_seqs: u32,
    pub num_queries: u32,
    pub q_heads: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub dict_size: u32,
    pub scale: f32,
    pub flags: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct weaver_views {
    pub q: *const c_void,
    pub q_latent: *const c_void,
    pub hot_k: *const c_void,
    pub hot_v: *const c_void,
    pub hot_pool_blocks: u64,
    pub hot_refs: *const u32,
    pub cold_k: *const weaver_sparse_code,
    pub cold_v: *const weaver_sparse_code,
    pub cold_pool_blocks: u64,
    pub cold_refs: *const u32,
    pub k_dict: *const c_void,
    pub v_dict: *const c_void,
    pub dict_head_stride: u64,
    pub out: *mut c_void,
    pub part_m: *mut f32,
    pub part_l: *mut f32,
    pub part_o: *mut f32,
}

/// Device-resident Fabric geometry (`fabric.rs:124-186` plus a layer dimension
/// and optional separate V regions).
#[repr(C)]
#[derive(Debug, Clone, Copy, Default)]
pub struct weaver_fabric_geometry {
    pub layers: u32,
    pub kv_heads: u32,
    pub head_dim: u32,
    pub dict_size: u32,
    pub hot_blocks: u64,
    pub cold_blocks: u64,
    pub separate_v: u32,
    pub _pad: u32,
    pub max_block_refs: u64,
}

#[repr(C)]
#[derive(Debug, Clone, Copy)]
pub struct weaver_fabric_layer {
    pub hot_k: *mut c_void,
    pub hot_v: *mut c_void,
    pub cold_k: *mut weaver_sparse_code,
    pub cold_v: *mut weaver_sparse_code,
    pub k_dict: *mut c_void,
    pub v_dict: *mut c_void,
    pub hot_pool_blocks: u64,
    pub cold_pool_blocks: u64,
}

/// Opaque device-resident Fabric.
#[repr(C)]
pub struct weaver_device_fabric {
    _private: [u8; 0],
}

/// Opaque engine (`WeaverEngine`, `weaver.rs:27-56`).
#[repr(C)]
pub struct weaver_engine {
    _private: [u8; 0],
}
/// Opaque decode plan (device-resident batched path).
#[repr(C)]
pub struct weaver_plan {
    _private: [u8; 0],
}
/// Opaque split-KV combiner over NVLink peer memory.
#[repr(C)]
pub struct weaver_combine {
    _private: [u8; 0],
}

extern "C" {
    pub fn weaver_abi_version() -> c_int;
    pub fn weaver_last_error() -> *const c_char;
    pub fn weaver_status_string(status: c_int) -> *const c_char;
    pub fn weaver_model_dims_preset(name: *const c_char, out: *mut weaver_model_dims) -> c_int;
    pub fn weaver_params_from_loom(dims: *const weaver_model_dims, loom: *const weaver_loom_descriptor,
                                   out: *mut weaver_params) -> c_int;
    pub fn weaver_fabric_regions_compute(dims: *const weaver_model_dims, out: *mut weaver_fabric_regions) -> c_int;

    pub fn weaver_engine_create(device: c_int, out: *mut *mut weaver_engine) -> c_int;
    pub fn weaver_engine_destroy(engine: *mut weaver_engine);
    pub fn weaver_engine_device_name(engine: *const weaver_engine, buf: *mut c_char, len: usize) -> c_int;
    pub fn weaver_engine_max_threads_per_block(engine: *const weaver_engine, out: *mut u64) -> c_int;
    pub fn weaver_decode_host(engine: *mut weaver_engine, q_exact: *const u16, q_exact_len: usize,
                              q_latent: *const u16, q_latent_len: usize, hot_pool: *const u16, hot_pool_len: usize,
                              cold_pool: *const weaver_sparse_code, cold_pool_len: usize, loom_refs: *const u32,
                              loom_refs_len: usize, dictionary: *const u16, dictionary_len: usize,
                              params: *const weaver_params, out: *mut u16, out_len: usize) -> c_int;

    pub fn weaver_plan_create(engine: *mut weaver_engine, shape: *const weaver_shape, hot_indptr: *const u32,
                              cold_indptr: *const u32, out: *mut *mut weaver_plan) -> c_int;
    pub fn weaver_plan_destroy(plan: *mut weaver_plan);
    pub fn weaver_run(plan: *mut weaver_plan, views: *const weaver_views, stream: *mut c_void) -> c_int;
    pub fn weaver_plan_kernel_count(plan: *const weaver_plan) -> c_int;
    pub fn weaver_plan_status(plan: *mut weaver_plan) -> c_int;
    pub fn weaver_decode_host_batch(engine: *mut weaver_engine, shape: *const weaver_shape, hot_indptr: *const u32,
                                    cold_indptr: *const u32, host_views: *const weaver_views) -> c_int;
    pub fn weaver_plan_trace(plan: *mut weaver_plan, out: *mut u64, n: usize, slots_per_cta: *mut u32) -> c_int;

    pub fn weaver_hot_decode_noalloc(q_heads: u32, kv_heads: u32, head_dim: u32, scale: f32, q: *const c_void,
                                     hot_k: *const c_void, hot_v: *const c_void, hot_pool_blocks: u64,
                                     hot_refs: *const u32, n_blocks: u32, out: *mut c_void, bad_ref_flag: *mut u32,
                                     stream: *mut c_void) -> c_int;

    pub fn weaver_merge_partials(n_parts: u32, rows: u32, head_dim: u32, m: *const f32, l: *const f32,
                                 o: *const f32, out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn weaver_merge_partials_strided(n_parts: u32, rows: u32, head_dim: u32, m: *const f32, l: *const f32,
                                         o: *const f32, part_stride: u64, out: *mut c_void,
                                         stream: *mut c_void) -> c_int;

    pub fn weaver_combine_create(engine: *mut weaver_engine, world: u32, rank: u32, rows: u32, head_dim: u32,
                                 out: *mut *mut weaver_combine) -> c_int;
    pub fn weaver_combine_destroy(c: *mut weaver_combine);
    pub fn weaver_combine_ipc_handle(c: *mut weaver_combine, handle_out: *mut c_void) -> c_int;
    pub fn weaver_combine_open_peer(c: *mut weaver_combine, peer: u32, handle: *const c_void) -> c_int;
    pub fn weaver_combine_run(c: *mut weaver_combine, packed: *const f32, out: *mut c_void,
                              stream: *mut c_void) -> c_int;
    pub fn weaver_combine_status(c: *mut weaver_combine) -> c_int;
    pub fn weaver_plan_attach_combine(plan: *mut weaver_plan, c: *mut weaver_combine) -> c_int;

    pub fn weaver_block_entropy(hot_pool: *const c_void, n_blocks: u64, kv_heads: u32, head_dim: u32, out: *mut f32,
                                stream: *mut c_void) -> c_int;
    pub fn weaver_migrate_blocks(hot_k: *const c_void, hot_v: *const c_void, hot_pool_blocks: u64,
                                 src_blocks: *const u32, dst_blocks: *const u32, n: u32, kv_heads: u32, head_dim: u32,
                                 k_dict: *const c_void, v_dict: *const c_void, dict_size: u32, dict_head_stride: u64,
                                 cold_k: *mut weaver_sparse_code, cold_v: *mut weaver_sparse_code,
                                 cold_pool_blocks: u64, bad_flag: *mut u32, stream: *mut c_void) -> c_int;

    pub fn weaver_wait_selftest(limit_us: u32, expired_mask: *mut u32, waited_ns: *mut u64,
                                status_words: *mut u32) -> c_int;

    pub fn weaver_distill(rows: *const c_void, n_rows: u32, kv_heads: u32, head_dim: u32,
                          dictionary: *const c_void, dict_size: u32, dict_head_stride: u64,
                          out_codes: *mut weaver_sparse_code, stream: *mut c_void) -> c_int;
    pub fn weaver_device_fabric_create(device: c_int, geometry: *const weaver_fabric_geometry,
                                       out: *mut *mut weaver_device_fabric) -> c_int;
    pub fn weaver_device_fabric_destroy(fabric: *mut weaver_device_fabric);
    pub fn weaver_device_fabric_layer(fabric: *const weaver_device_fabric, layer: u32,
                                      out: *mut weaver_fabric_layer) -> c_int;
    pub fn weaver_device_fabric_block_refs(fabric: *const weaver_device_fabric, refs: *mut *mut u32,
                                           capacity: *mut u64) -> c_int;
    pub fn weaver_device_fabric_upload_aether(fabric: *mut weaver_device_fabric, layer: u32, image: *const c_void,
                                              image_bytes: u64, regions: *const weaver_fabric_regions, which: u32,
                                              stream: *mut c_void) -> c_int;
    pub fn weaver_device_fabric_upload_refs(fabric: *mut weaver_device_fabric, refs: *const u32, n: u64, offset: u64,
                                            stream: *mut c_void) -> c_int;
    pub fn weaver_loom_page_tables(fabric: *const weaver_device_fabric, looms: *const weaver_loom_descriptor, n: u32,
                                   hot_indptr: *mut u32, cold_indptr: *mut u32, hot_refs: *mut u32,
                                   hot_capacity: u64, cold_refs: *mut u32, cold_capacity: u64,
                                   stream: *mut c_void) -> c_int;
    pub fn weaver_multihead_attention(engine: *mut weaver_engine, q: *const c_void, k_cache: *const c_void,
                                      v_cache: *const c_void, out: *mut c_void, total_kv_len: u32, head_dim: u32,
                                      q_heads: u32, kv_heads: u32, num_queries: u32, stream: *mut c_void) -> c_int;
    pub fn weaver_distill_stats(rows: *const c_void, n_rows: u32, kv_heads: u32, head_dim: u32,
                                dictionary: *const c_void, dict_size: u32, dict_head_stride: u64,
                                out_codes: *mut weaver_sparse_code, diag: *mut u32, stream: *mut c_void) -> c_int;
}

#[cfg(test)]
mod tests {
    use super::*;
    use std::mem::{align_of, size_of};

    #[test]
    fn layouts_match_the_header() {
        assert_eq!(size_of::<weaver_sparse_code>(), 16);
        assert_eq!(size_of::<weaver_params>(), 48);
        assert_eq!(size_of::<weaver_model_dims>(), 44);
        assert_eq!(size_of::<weaver_loom_descriptor>(), 32);
        assert_eq!(size_of::<weaver_fabric_regions>(), 17 * 8);
        assert_eq!(size_of::<weaver_shape>(), 32);
        assert_eq!(size_of::<weaver_views>(), 17 * 8);
        assert_eq!(align_of::<weaver_views>(), 8);
    }
}
