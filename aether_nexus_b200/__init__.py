"""aether_nexus_b200 — B200 (sm_100a) Weaver decode attention.

A drop-in replacement for AetherNexus's Weaver decode path
(``nexus-core/src/weaver.rs`` + ``weaver_kernel.metal``): exact f16 GQA
attention over a paged hot KV pool, decompression-free attention over a cold
pool of 16-byte SparseCode dictionary codes, log-sum-exp merge.  The compute
lives in ``libweaver_cuda.so`` (hand-written CUDA for sm_100a, C ABI in
``include/weaver_cuda.h``); this package is its Python host API.
"""
from ._native import WeaverError, library_path
from .types import (BLOCK_SIZE, REF_MASK, SPARSE_CODE_DTYPE, SPARSITY_K, FabricRegions, LoomDescriptor,
                    ModelDims, Persona, WeaverParams, sparse_code_zero)
from .weaver import DecodeOutput, WeaverEngine, WeaverPlan, distill, merge_partials, merge_partials_packed

__all__ = [
    "BLOCK_SIZE", "REF_MASK", "SPARSE_CODE_DTYPE", "SPARSITY_K", "DecodeOutput", "FabricRegions",
    "LoomDescriptor", "ModelDims", "Persona", "WeaverEngine", "WeaverError", "WeaverParams", "WeaverPlan",
    "distill", "library_path", "merge_partials", "merge_partials_packed", "sparse_code_zero",
]
