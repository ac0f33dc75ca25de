"""The C ABI library without a GPU: it loads, exports every entry point the
header declares, and the host-only helpers (types, ModelDims presets,
WeaverParams::from_loom, FabricRegions::compute) match the reference."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT
import aether_nexus_b200 as W
from aether_nexus_b200 import _native as N


def header_functions():
    with open(os.path.join(ROOT, "include", "weaver_cuda.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"WEAVER_EXPORT\s+[\w\s\*]*?\b(weaver_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    names = header_functions()
    assert len(names) >= 18
    for n in names:
        assert hasattr(lib, n), n
    assert {n for n, _, _ in N.SIGNATURES} == set(names)
    assert lib.weaver_abi_version() == 1


def test_status_strings_and_last_error():
    lib = N.lib()
    for s in range(9):
        assert lib.weaver_status_string(s)
    rc = lib.weaver_model_dims_preset(b"nope", ctypes.byref(N.ModelDimsC()))
    assert rc == 1
    assert b"nope" in lib.weaver_last_error()


def test_sparse_code_layout():
    """types.rs:521-560: 16 bytes, zero default, byte round trip."""
    assert W.SPARSE_CODE_DTYPE.itemsize == 16
    assert ctypes.sizeof(N.SparseCodeC) == 16
    z = W.sparse_code_zero()
    assert z.tobytes() == bytes(16)
    c = np.zeros((), W.SPARSE_CODE_DTYPE)
    c["indices"] = [1, 42, 255, 511]
    c["coeffs"] = [0.5, -0.25, 1.0, 0.0]
    raw = c.tobytes()
    back = np.frombuffer(raw, W.SPARSE_CODE_DTYPE)[0]
    assert list(back["indices"]) == [1, 42, 255, 511]
    assert list(back["coeffs"]) == [0.5, -0.25, 1.0, 0.0]
    assert raw[:8] == np.array([1, 42, 255, 511], "<u2").tobytes()


def test_weaver_params_and_loom():
    """types.rs:564-579, 380-395, 596-598."""
    assert ctypes.sizeof(N.WeaverParamsC) == 48
    assert ctypes.sizeof(N.LoomDescriptorC) == 32
    dims = W.ModelDims.preset("llama8b")
    assert dims.gqa_group == 4
    loom = W.LoomDescriptor(W.Persona.CODER, hot_count=100, cold_count=500)
    p = W.WeaverParams.from_loom(dims, loom)
    assert (p.q_heads, p.kv_heads, p.head_dim, p.block_size, p.gqa_group) == (32, 8, 128, 16, 4)
    assert (p.hot_count, p.cold_count, p.dict_size, p.sparsity_k) == (100, 500, 512, 4)


def test_model_dims_presets():
    """types.rs:150-204."""
    exp = {
        "llama8b": (32, 32, 8, 128, 4096, 14336, 128256),
        "granite2b": (40, 32, 8, 64, 2048, 8192, 49155),
        "qwen05b": (24, 14, 2, 64, 896, 4864, 151936),
        "deepseek_r1_1_5b": (28, 12, 2, 128, 1536, 8960, 151936),
    }
    for name, e in exp.items():
        d = W.ModelDims.preset(name)
        assert (d.layers, d.q_heads, d.kv_heads, d.head_dim, d.hidden_size, d.intermediate_size,
                d.vocab_size) == e
        assert (d.block_size, d.sparsity_k, d.dict_size) == (16, 4, 512)


def _fabric_regions_py(d):
    """Independent restatement of FabricRegions::compute (fabric.rs:124-186)."""
    def up(v, a):
        return (v + a - 1) // a * a
    h, inter, vocab, L = d.hidden_size, d.intermediate_size, d.vocab_size, d.layers
    kv, q, hd = d.kv_heads, d.q_heads, d.head_dim
    per_layer = 2 * (q * hd * h + kv * hd * h + kv * hd * h + q * hd * h + h * inter + h * inter + inter * h + h + h)
    est = int(float(L * per_layer + 2 * (vocab * h + h)) * 1.25)
    r = {}
    r["weights_offset"] = up(9 + 4 + 64, 16384)
    r["weights_size"] = up(est, 16384)
    r["hot_pool_offset"] = up(r["weights_offset"] + r["weights_size"], 16384)
    r["hot_pool_size"] = 8192 * 16 * kv * hd * 2
    r["cold_pool_offset"] = up(r["hot_pool_offset"] + r["hot_pool_size"], 16384)
    r["cold_pool_size"] = 32768 * 16 * kv * 16
    r["dict_offset"] = up(r["cold_pool_offset"] + r["cold_pool_size"], 16384)
    r["dict_size"] = kv * d.dict_size * hd * 2
    r["looms_offset"] = up(r["dict_offset"] + r["dict_size"], 4096)
    r["looms_size"] = 4 * 32
    r["radix_offset"] = up(r["looms_offset"] + r["looms_size"], 4096)
    r["radix_size"] = (8192 + 32768) * 12
    r["obs_offset"] = up(r["radix_offset"] + r["radix_size"], 16384)
    r["obs_size"] = 256 << 20
    r["trace_offset"] = up(r["obs_offset"] + r["obs_size"], 16384)
    r["trace_size"] = 128 << 20
    r["total_size"] = up(r["trace_offset"] + r["trace_size"] + 64, 16384)
    return r


@pytest.mark.parametrize("name", ["llama8b", "granite2b", "qwen05b", "deepseek_r1_1_5b"])
def test_fabric_regions(name):
    """fabric.rs:755-808 (alignment, no overlap) and the exact offsets."""
    d = W.ModelDims.preset(name)
    r = W.FabricRegions.compute(d)
    for k, v in _fabric_regions_py(d).items():
        assert getattr(r, k) == v, k
    for k in ("weights_offset", "hot_pool_offset", "cold_pool_offset", "dict_offset", "obs_offset",
              "trace_offset", "total_size"):
        assert getattr(r, k) % 16384 == 0, k
    assert r.weights_offset + r.weights_size <= r.hot_pool_offset
    assert r.hot_pool_offset + r.hot_pool_size <= r.cold_pool_offset
    assert r.cold_pool_offset + r.cold_pool_size <= r.dict_offset
    assert r.dict_offset + r.dict_size <= r.looms_offset
    assert r.looms_offset + r.looms_size <= r.radix_offset
    assert r.radix_offset + r.radix_size <= r.obs_offset
    assert r.obs_offset + r.obs_size <= r.trace_offset


def test_fabric_cold_pool_views_as_codes():
    """fabric.rs:843-864: a zeroed cold region reads as zero SparseCodes."""
    d = W.ModelDims.preset("qwen05b")
    r = W.FabricRegions.compute(d)
    img = np.zeros(r.dict_offset + r.dict_size, np.uint8)
    codes = r.cold_pool_codes(img)
    assert codes.size == 32768 * 16 * d.kv_heads
    assert (codes[0]["indices"] == 0).all()


def test_engine_without_gpu_fails_cleanly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(W.WeaverError) as e:
        W.WeaverEngine(0)
    assert e.value.status == 6  # WEAVER_ERR_NO_DEVICE
