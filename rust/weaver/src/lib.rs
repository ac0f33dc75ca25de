//! `WeaverEngine` with the reference's API (`nexus-core/src/weaver.rs:27-322`)
//! over the CUDA library.  A drop-in for the Metal engine: `new(metallib_path)`
//! (the path is accepted and ignored, the kernels are linked into the
//! library), `decode(q_exact, q_latent, hot_pool, cold_pool, loom_refs,
//! dictionary, &params) -> Result<DecodeOutput, String>`, `device_name()` and
//! `max_threads_per_threadgroup()`.  `WeaverPlan` adds the device-resident
//! batched path (pools stay in HBM, one call per decode step on a stream).

use half::f16;
use std::ffi::CStr;
use std::os::raw::{c_char, c_void};
use weaver_sys as sys;

/// `SparseCode` (`types.rs:218-228`): 4 atom indices and 4 f16 coefficients,
/// 16 bytes, the layout of the cold pool's records.
#[repr(C, align(16))]
#[derive(Clone, Copy, Debug, Default, PartialEq)]
pub struct SparseCode {
    pub indices: [u16; 4],
    pub coeffs: [f16; 4],
}

/// `WeaverParams` (`types.rs:351-374`), passed to the library unchanged.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default, PartialEq, Eq)]
pub struct WeaverParams {
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

/// `DecodeOutput` (`weaver.rs:59-62`).
#[derive(Debug, Clone)]
pub struct DecodeOutput {
    pub data: Vec<f16>,
}

fn last_error() -> String {
    unsafe { CStr::from_ptr(sys::weaver_last_error()) }.to_string_lossy().into_owned()
}

fn check(rc: i32) -> Result<(), String> {
    if rc == sys::WEAVER_OK {
        Ok(())
    } else {
        let name = unsafe { CStr::from_ptr(sys::weaver_status_string(rc)) }.to_string_lossy().into_owned();
        Err(format!("{name}: {}", last_error()))
    }
}

/// The Weaver engine on one CUDA device (`weaver.rs:31-56`).  Single caller at
/// a time, like the reference's `&mut self`.
pub struct WeaverEngine {
    raw: *mut sys::weaver_engine,
}

impl WeaverEngine {
    /// `WeaverEngine::new` (`weaver.rs:85-132`) on device 0.
    pub fn new(_metallib_path: &str) -> Result<Self, String> {
        Self::on_device(0)
    }

    pub fn on_device(device: i32) -> Result<Self, String> {
        let mut raw = std::ptr::null_mut();
        check(unsafe { sys::weaver_engine_create(device, &mut raw) })?;
        Ok(Self { raw })
    }

    /// `WeaverEngine::decode` (`weaver.rs:139-237`): host slices are copied to
    /// the device, one step runs, the call returns the output token.
    #[allow(clippy::too_many_arguments)]
    pub fn decode(&mut self, q_exact: &[f16], q_latent: &[f16], hot_pool: &[f16], cold_pool: &[SparseCode],
                  loom_refs: &[u32], dictionary: &[f16], params: &WeaverParams) -> Result<DecodeOutput, String> {
        let n = (params.q_heads * params.head_dim) as usize;
        let mut out = vec![f16::ZERO; n];
        check(unsafe {
            sys::weaver_decode_host(self.raw, q_exact.as_ptr() as *const u16, q_exact.len(),
                                    q_latent.as_ptr() as *const u16, q_latent.len(),
                                    hot_pool.as_ptr() as *const u16, hot_pool.len(),
                                    cold_pool.as_ptr() as *const sys::weaver_sparse_code, cold_pool.len(),
                                    loom_refs.as_ptr(), loom_refs.len(), dictionary.as_ptr() as *const u16,
                                    dictionary.len(), params as *const WeaverParams as *const sys::weaver_params,
                                    out.as_mut_ptr() as *mut u16, n)
        })?;
        Ok(DecodeOutput { data: out })
    }

    /// `WeaverEngine::device_name` (`weaver.rs:314-316`).
    pub fn device_name(&self) -> String {
        let mut buf = [0 as c_char; 256];
        match check(unsafe { sys::weaver_engine_device_name(self.raw, buf.as_mut_ptr(), buf.len()) }) {
            Ok(()) => unsafe { CStr::from_ptr(buf.as_ptr()) }.to_string_lossy().into_owned(),
            Err(e) => e,
        }
    }

    /// `WeaverEngine::max_threads_per_threadgroup` (`weaver.rs:319-321`).
    pub fn max_threads_per_threadgroup(&self) -> u64 {
        let mut v = 0u64;
        let _ = check(unsafe { sys::weaver_engine_max_threads_per_block(self.raw, &mut v) });
        v
    }

    pub fn raw(&self) -> *mut sys::weaver_engine {
        self.raw
    }
}

impl Drop for WeaverEngine {
    fn drop(&mut self) {
        unsafe { sys::weaver_engine_destroy(self.raw) }
    }
}

/// A decode plan over device-resident pools (Fabric sub-views in HBM): fixes
/// the geometry and the per-sequence block counts, owns its scratch, and
/// launches one step per `run` on the caller's stream without allocating.
pub struct WeaverPlan<'e> {
    raw: *mut sys::weaver_plan,
    _engine: std::marker::PhantomData<&'e WeaverEngine>,
}

impl<'e> WeaverPlan<'e> {
    pub fn new(engine: &'e mut WeaverEngine, shape: &sys::weaver_shape, hot_indptr: &[u32],
               cold_indptr: &[u32]) -> Result<Self, String> {
        let b = shape.num_seqs as usize;
        if hot_indptr.len() != b + 1 || cold_indptr.len() != b + 1 {
            return Err("indptr arrays need num_seqs + 1 entries".to_string());
        }
        let mut raw = std::ptr::null_mut();
        check(unsafe {
            sys::weaver_plan_create(engine.raw, shape, hot_indptr.as_ptr(), cold_indptr.as_ptr(), &mut raw)
        })?;
        Ok(Self { raw, _engine: std::marker::PhantomData })
    }

    /// Launch one decode step on `stream` (a `cudaStream_t`, null = default).
    ///
    /// # Safety
    /// Every pointer in `views` must be a device address of the size the plan's
    /// shape implies, valid until the step has run.
    pub unsafe fn run(&mut self, views: &sys::weaver_views, stream: *mut c_void) -> Result<(), String> {
        check(sys::weaver_run(self.raw, views, stream))
    }

    /// Synchronise and report out-of-range references or an expired wait.
    pub fn status(&mut self) -> Result<(), String> {
        check(unsafe { sys::weaver_plan_status(self.raw) })
    }

    pub fn kernel_count(&self) -> i32 {
        unsafe { sys::weaver_plan_kernel_count(self.raw) }
    }
}

impl Drop for WeaverPlan<'_> {
    fn drop(&mut self) {
        unsafe { sys::weaver_plan_destroy(self.raw) }
    }
}

#[cfg(test)]
mod tests {
    use super::*;

    #[test]
    fn reference_types_keep_their_sizes() {
        assert_eq!(std::mem::size_of::<SparseCode>(), 16);
        assert_eq!(std::mem::size_of::<WeaverParams>(), 48);
    }
}
