"""ctypes bindings of ``libweaver_cuda.so`` (declared in ``include/weaver_cuda.h``).

Loading fails loudly: there is no CPU fallback.  If the library is missing and
``nvcc`` is available it is built in place first (``aether_nexus_b200.build``).
"""
from __future__ import annotations

import ctypes
import os

from . import build as _build

c_u8, c_u16, c_u32, c_u64 = ctypes.c_uint8, ctypes.c_uint16, ctypes.c_uint32, ctypes.c_uint64
c_int, c_float, c_void_p, c_size_t = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t

WEAVER_OK = 0
STATUS_NAMES = {
    0: "WEAVER_OK", 1: "WEAVER_ERR_INVALID_ARGUMENT", 2: "WEAVER_ERR_UNSUPPORTED",
    3: "WEAVER_ERR_MISALIGNED", 4: "WEAVER_ERR_OUT_OF_RANGE", 5: "WEAVER_ERR_CUDA",
    6: "WEAVER_ERR_NO_DEVICE", 7: "WEAVER_ERR_TIMEOUT", 8: "WEAVER_ERR_CAPACITY",
}
FLAG_CAUSAL, FLAG_QLATENT_INPUT, FLAG_PARTIALS = 1, 2, 4


class SparseCodeC(ctypes.Structure):
    _fields_ = [("indices", c_u16 * 4), ("coeffs", c_u16 * 4)]


class WeaverParamsC(ctypes.Structure):
    _fields_ = [(n, c_u32) for n in ("q_heads", "kv_heads", "head_dim", "block_size", "gqa_group",
                                      "hot_count", "cold_count", "dict_size", "sparsity_k")] + \
               [("_pad", c_u32 * 3)]


class ModelDimsC(ctypes.Structure):
    _fields_ = [(n, c_u32) for n in ("layers", "q_heads", "kv_heads", "head_dim", "hidden_size",
                                      "intermediate_size", "vocab_size", "block_size", "sparsity_k",
                                      "dict_size", "gqa_group")]


class LoomDescriptorC(ctypes.Structure):
    _fields_ = [("persona", c_u8), ("_pad0", c_u8 * 3), ("hot_count", c_u32), ("cold_count", c_u32),
                ("hot_refs_offset", c_u32), ("cold_refs_offset", c_u32), ("token_pos", c_u32),
                ("_pad", c_u32 * 2)]


class FabricRegionsC(ctypes.Structure):
    _fields_ = [(n, c_u64) for n in (
        "weights_offset", "weights_size", "hot_pool_offset", "hot_pool_size", "cold_pool_offset",
        "cold_pool_size", "dict_offset", "dict_size", "looms_offset", "looms_size", "radix_offset",
        "radix_size", "obs_offset", "obs_size", "trace_offset", "trace_size", "total_size")]


class FabricGeometryC(ctypes.Structure):
    _fields_ = [("layers", c_u32), ("kv_heads", c_u32), ("head_dim", c_u32), ("dict_size", c_u32),
                ("hot_blocks", c_u64), ("cold_blocks", c_u64), ("separate_v", c_u32), ("_pad", c_u32),
                ("max_block_refs", c_u64)]


class FabricLayerC(ctypes.Structure):
    _fields_ = [("hot_k", c_void_p), ("hot_v", c_void_p), ("cold_k", c_void_p), ("cold_v", c_void_p),
                ("k_dict", c_void_p), ("v_dict", c_void_p), ("hot_pool_blocks", c_u64),
                ("cold_pool_blocks", c_u64)]


class ShapeC(ctypes.Structure):
    _fields_ = [("num_seqs", c_u32), ("num_queries", c_u32), ("q_heads", c_u32), ("kv_heads", c_u32),
                ("head_dim", c_u32), ("dict_size", c_u32), ("scale", c_float), ("flags", c_u32)]


class ViewsC(ctypes.Structure):
    _fields_ = [("q", c_void_p), ("q_latent", c_void_p), ("hot_k", c_void_p), ("hot_v", c_void_p),
                ("hot_pool_blocks", c_u64), ("hot_refs", c_void_p), ("cold_k", c_void_p),
                ("cold_v", c_void_p), ("cold_pool_blocks", c_u64), ("cold_refs", c_void_p),
                ("k_dict", c_void_p), ("v_dict", c_void_p), ("dict_head_stride", c_u64),
                ("out", c_void_p), ("part_m", c_void_p), ("part_l", c_void_p), ("part_o", c_void_p)]


assert ctypes.sizeof(SparseCodeC) == 16 and ctypes.sizeof(WeaverParamsC) == 48
assert ctypes.sizeof(LoomDescriptorC) == 32
assert ctypes.sizeof(FabricGeometryC) == 48 and ctypes.sizeof(FabricLayerC) == 64

# (name, restype, argtypes) for every entry point of include/weaver_cuda.h
SIGNATURES = [
    ("weaver_abi_version", c_int, []),
    ("weaver_last_error", ctypes.c_char_p, []),
    ("weaver_status_string", ctypes.c_char_p, [c_int]),
    ("weaver_model_dims_preset", c_int, [ctypes.c_char_p, ctypes.POINTER(ModelDimsC)]),
    ("weaver_params_from_loom", c_int, [ctypes.POINTER(ModelDimsC), ctypes.POINTER(LoomDescriptorC),
                                        ctypes.POINTER(WeaverParamsC)]),
    ("weaver_fabric_regions_compute", c_int, [ctypes.POINTER(ModelDimsC), ctypes.POINTER(FabricRegionsC)]),
    ("weaver_engine_create", c_int, [c_int, ctypes.POINTER(c_void_p)]),
    ("weaver_engine_destroy", None, [c_void_p]),
    ("weaver_engine_device_name", c_int, [c_void_p, ctypes.c_char_p, c_size_t]),
    ("weaver_engine_max_threads_per_block", c_int, [c_void_p, ctypes.POINTER(c_u64)]),
    ("weaver_decode_host", c_int, [c_void_p, c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                   c_void_p, c_size_t, c_void_p, c_size_t, c_void_p, c_size_t,
                                   ctypes.POINTER(WeaverParamsC), c_void_p, c_size_t]),
    ("weaver_decode_host_batch", c_int, [c_void_p, ctypes.POINTER(ShapeC), c_void_p, c_void_p,
                                         ctypes.POINTER(ViewsC)]),
    ("weaver_plan_create", c_int, [c_void_p, ctypes.POINTER(ShapeC), c_void_p, c_void_p,
                                   ctypes.POINTER(c_void_p)]),
    ("weaver_plan_destroy", None, [c_void_p]),
    ("weaver_run", c_int, [c_void_p, ctypes.POINTER(ViewsC), c_void_p]),
    ("weaver_plan_kernel_count", c_int, [c_void_p]),
    ("weaver_plan_status", c_int, [c_void_p]),
    ("weaver_plan_trace", c_int, [c_void_p, c_void_p, c_size_t, ctypes.POINTER(c_u32)]),
    ("weaver_merge_partials", c_int, [c_u32, c_u32, c_u32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    ("weaver_merge_partials_strided", c_int, [c_u32, c_u32, c_u32, c_void_p, c_void_p, c_void_p, c_u64, c_void_p,
                                              c_void_p]),
    ("weaver_combine_create", c_int, [c_void_p, c_u32, c_u32, c_u32, c_u32, ctypes.POINTER(c_void_p)]),
    ("weaver_combine_destroy", None, [c_void_p]),
    ("weaver_combine_ipc_handle", c_int, [c_void_p, c_void_p]),
    ("weaver_combine_open_peer", c_int, [c_void_p, c_u32, c_void_p]),
    ("weaver_combine_run", c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    ("weaver_combine_status", c_int, [c_void_p]),
    ("weaver_plan_attach_combine", c_int, [c_void_p, c_void_p]),
    ("weaver_wait_selftest", c_int, [c_u32, c_void_p, c_void_p, c_void_p]),
    ("weaver_block_entropy", c_int, [c_void_p, c_u64, c_u32, c_u32, c_void_p, c_void_p]),
    ("weaver_migrate_blocks", c_int, [c_void_p, c_void_p, c_u64, c_void_p, c_void_p, c_u32, c_u32, c_u32, c_void_p,
                                      c_void_p, c_u32, c_u64, c_void_p, c_void_p, c_u64, c_void_p, c_void_p]),
    ("weaver_hot_decode_noalloc", c_int, [c_u32, c_u32, c_u32, c_float, c_void_p, c_void_p, c_void_p, c_u64,
                                          c_void_p, c_u32, c_void_p, c_void_p, c_void_p]),
    ("weaver_distill", c_int, [c_void_p, c_u32, c_u32, c_u32, c_void_p, c_u32, c_u64, c_void_p, c_void_p]),
    ("weaver_device_fabric_create", c_int, [c_int, ctypes.POINTER(FabricGeometryC), ctypes.POINTER(c_void_p)]),
    ("weaver_device_fabric_destroy", None, [c_void_p]),
    ("weaver_device_fabric_layer", c_int, [c_void_p, c_u32, ctypes.POINTER(FabricLayerC)]),
    ("weaver_device_fabric_block_refs", c_int, [c_void_p, ctypes.POINTER(c_void_p), ctypes.POINTER(c_u64)]),
    ("weaver_device_fabric_upload_aether", c_int, [c_void_p, c_u32, c_void_p, c_u64, ctypes.POINTER(FabricRegionsC),
                                                   c_u32, c_void_p]),
    ("weaver_device_fabric_upload_refs", c_int, [c_void_p, c_void_p, c_u64, c_u64, c_void_p]),
    ("weaver_loom_page_tables", c_int, [c_void_p, c_void_p, c_u32, c_void_p, c_void_p, c_void_p, c_u64, c_void_p,
                                        c_u64, c_void_p]),
    ("weaver_multihead_attention", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_u32, c_u32, c_u32,
                                           c_u32, c_u32, c_void_p]),
    ("weaver_distill_stats", c_int, [c_void_p, c_u32, c_u32, c_u32, c_void_p, c_u32, c_u64, c_void_p, c_void_p,
                                     c_void_p]),
]

_lib = None


class WeaverError(RuntimeError):
    """A non-zero status from the C ABI (the reference's ``Err(String)``)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


def library_path() -> str:
    return _build.LIB


def lib() -> ctypes.CDLL:
    """Load (building first if needed) the CUDA library and bind its prototypes."""
    global _lib
    if _lib is None:
        if not os.path.exists(_build.LIB) or os.environ.get("WEAVER_REBUILD") == "1":
            _build.build()
        L = ctypes.CDLL(_build.LIB)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != WEAVER_OK:
        raise WeaverError(status, lib().weaver_last_error().decode(errors="replace"))
