"""Reference ABI types of the Weaver path, mirrored for Python callers.

* ``SPARSE_CODE_DTYPE`` — ``SparseCode`` (``nexus-core/src/types.rs:218-228``):
  4 x u16 atom index + 4 x f16 coefficient, 16 bytes.
* ``WeaverParams`` — ``types.rs:351-396`` (48 bytes, ``from_loom``).
* ``ModelDims`` presets — ``types.rs:150-204``.
* ``LoomDescriptor`` / ``Persona`` — ``types.rs:278-328``.
* ``FabricRegions.compute`` — ``nexus-core/src/fabric.rs:124-186``.
"""
from __future__ import annotations

import ctypes
import dataclasses
import enum

import numpy as np

from . import _native as N

BLOCK_SIZE = 16
SPARSITY_K = 4
REF_MASK = 0x7FFFFFFF

SPARSE_CODE_DTYPE = np.dtype([("indices", "<u2", (4,)), ("coeffs", "<f2", (4,))])
assert SPARSE_CODE_DTYPE.itemsize == 16


def sparse_code_zero() -> np.ndarray:
    """``SparseCode::zero()`` (types.rs:233-238)."""
    return np.zeros((), dtype=SPARSE_CODE_DTYPE)


class Persona(enum.IntEnum):
    PLANNER = 0
    CODER = 1
    CRITIC = 2
    REVIEWER = 3


@dataclasses.dataclass(frozen=True)
class ModelDims:
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    hidden_size: int
    intermediate_size: int
    vocab_size: int
    block_size: int = BLOCK_SIZE
    sparsity_k: int = SPARSITY_K
    dict_size: int = 512

    @property
    def gqa_group(self) -> int:
        return self.q_heads // self.kv_heads

    @classmethod
    def preset(cls, name: str) -> "ModelDims":
        c = N.ModelDimsC()
        N.check(N.lib().weaver_model_dims_preset(name.encode(), ctypes.byref(c)))
        return cls(c.layers, c.q_heads, c.kv_heads, c.head_dim, c.hidden_size, c.intermediate_size,
                   c.vocab_size, c.block_size, c.sparsity_k, c.dict_size)

    def to_c(self) -> N.ModelDimsC:
        return N.ModelDimsC(self.layers, self.q_heads, self.kv_heads, self.head_dim, self.hidden_size,
                            self.intermediate_size, self.vocab_size, self.block_size, self.sparsity_k,
                            self.dict_size, self.gqa_group)


# Preset names of types.rs:167-204 (Llama8B is the trait default).
LLAMA8B, GRANITE2B, QWEN05B, DEEPSEEK_R1_1_5B = "llama8b", "granite2b", "qwen05b", "deepseek_r1_1_5b"


@dataclasses.dataclass
class LoomDescriptor:
    persona: Persona = Persona.PLANNER
    hot_count: int = 0
    cold_count: int = 0
    hot_refs_offset: int = 0
    cold_refs_offset: int = 0
    token_pos: int = 0

    def to_c(self) -> N.LoomDescriptorC:
        c = N.LoomDescriptorC()
        c.persona = int(self.persona)
        c.hot_count, c.cold_count = self.hot_count, self.cold_count
        c.hot_refs_offset, c.cold_refs_offset = self.hot_refs_offset, self.cold_refs_offset
        c.token_pos = self.token_pos
        return c


@dataclasses.dataclass
class WeaverParams:
    q_heads: int
    kv_heads: int
    head_dim: int
    block_size: int
    gqa_group: int
    hot_count: int
    cold_count: int
    dict_size: int
    sparsity_k: int

    @classmethod
    def from_loom(cls, dims: ModelDims, loom: LoomDescriptor) -> "WeaverParams":
        c = N.WeaverParamsC()
        N.check(N.lib().weaver_params_from_loom(ctypes.byref(dims.to_c()), ctypes.byref(loom.to_c()),
                                                ctypes.byref(c)))
        return cls.from_c(c)

    @classmethod
    def from_c(cls, c: N.WeaverParamsC) -> "WeaverParams":
        return cls(c.q_heads, c.kv_heads, c.head_dim, c.block_size, c.gqa_group, c.hot_count,
                   c.cold_count, c.dict_size, c.sparsity_k)

    def to_c(self) -> N.WeaverParamsC:
        c = N.WeaverParamsC()
        for f in dataclasses.fields(self):
            setattr(c, f.name, int(getattr(self, f.name)))
        return c

    def as_dict(self) -> dict:
        return dataclasses.asdict(self)


@dataclasses.dataclass(frozen=True)
class FabricRegions:
    weights_offset: int
    weights_size: int
    hot_pool_offset: int
    hot_pool_size: int
    cold_pool_offset: int
    cold_pool_size: int
    dict_offset: int
    dict_size: int
    looms_offset: int
    looms_size: int
    radix_offset: int
    radix_size: int
    obs_offset: int
    obs_size: int
    trace_offset: int
    trace_size: int
    total_size: int

    @classmethod
    def compute(cls, dims: ModelDims) -> "FabricRegions":
        c = N.FabricRegionsC()
        N.check(N.lib().weaver_fabric_regions_compute(ctypes.byref(dims.to_c()), ctypes.byref(c)))
        return cls(*[getattr(c, f.name) for f in dataclasses.fields(cls)])

    # zero-copy sub-views of an in-memory .aether image (fabric.rs:347-384)
    def hot_pool(self, fabric: np.ndarray) -> np.ndarray:
        return fabric[self.hot_pool_offset:self.hot_pool_offset + self.hot_pool_size]

    def cold_pool(self, fabric: np.ndarray) -> np.ndarray:
        return fabric[self.cold_pool_offset:self.cold_pool_offset + self.cold_pool_size]

    def cold_pool_codes(self, fabric: np.ndarray) -> np.ndarray:
        return self.cold_pool(fabric).view(SPARSE_CODE_DTYPE)

    def dictionary(self, fabric: np.ndarray) -> np.ndarray:
        return fabric[self.dict_offset:self.dict_offset + self.dict_size]
