"""The bench metric's definitions, pinned on CPU: the configurations' shapes
and the algorithmic byte and token counts that `bench.py` divides by its
step time (KV tokens/s = tokens per step / time; GB/s = compulsory bytes per
step / time).  No GPU."""
import math

import pytest

from aether_nexus_b200 import synth
from aether_nexus_b200.types import BLOCK_SIZE

# (q heads, kv heads, head dim, atoms, hot tokens, cold tokens, sequences, queries)
SHAPES = {
    "c1": (8, 8, 64, 512, 256, 1024, 1, 1),
    "c2": (32, 8, 128, 4096, 4096, 28672, 1, 1),
    "c3": (32, 8, 128, 4096, 2048, 16384, 64, 1),
    "c4": (32, 8, 128, 4096, 4096, 28672, 16, 8),
    "c5": (64, 8, 128, 8192, 8192, 131072, 1, 1),
}


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_configuration_shapes(name):
    c = synth.config(name)
    got = (c["q_heads"], c["kv_heads"], c["head_dim"], c["dict_size"], c["hot_tokens"], c["cold_tokens"],
           c["num_seqs"], c["num_queries"])
    assert got == SHAPES[name]
    assert c["scale"] == pytest.approx(1 / math.sqrt(c["head_dim"]))
    assert c["q_heads"] % c["kv_heads"] == 0


def test_c2_bytes_and_tokens_per_step():
    """c2: 4096 hot + 28672 cold tokens, 8 kv heads, d 128, 4096 atoms:
    hot K+V 16,777,216 B + K/V codes 7,340,032 B + K/V dictionaries
    16,777,216 B + q in / out 16,384 B = 40,910,848 B per step."""
    w = synth.make_workload("c2", seed=0)
    assert synth.kv_tokens(w) == 32768
    Hkv, d, A = 8, 128, 4096
    hot = 4096 * Hkv * d * 2 * 2
    codes = 28672 * Hkv * 16 * 2
    dicts = 2 * Hkv * A * d * 2
    qo = 32 * d * 2 * 2
    assert (hot, codes, dicts, qo) == (16777216, 7340032, 16777216, 16384)
    assert synth.bytes_algorithmic(w) == hot + codes + dicts + qo == 40910848


def test_byte_count_follows_the_page_tables():
    """Blocks referenced by the page tables are what is counted (16 tokens per
    block); a workload without cold blocks reads no dictionaries."""
    w = synth.make_workload("c1", seed=3)
    th = int(w["hot_indptr"][-1]) * BLOCK_SIZE
    tc = int(w["cold_indptr"][-1]) * BLOCK_SIZE
    assert (th, tc) == (256, 1024)
    Hkv, d, A = w["kv_heads"], w["head_dim"], w["dict_size"]
    qo = w["num_seqs"] * w["num_queries"] * w["q_heads"] * d * 2 * 2
    assert synth.bytes_algorithmic(w) == th * Hkv * d * 4 + tc * Hkv * 32 + 2 * Hkv * A * d * 2 + qo
    v = dict(w)
    v["cold_indptr"] = w["cold_indptr"] * 0
    assert synth.bytes_algorithmic(v) == th * Hkv * d * 4 + qo
    assert synth.kv_tokens(v) == th


def test_c3_step_decodes_32_layers():
    """c3 is measured as BASELINE states it: a step decodes all 32 layers,
    each with its own pools, codes and dictionaries behind the same page
    tables, so its tokens and compulsory bytes are 32 times one layer's."""
    assert synth.config("c3")["layers"] == 32
    for name in ("c1", "c2", "c4", "c5"):
        assert synth.config(name).get("layers", 1) == 1


def test_layer_like_keeps_shapes_and_page_tables():
    """Another layer generated on the device has the first layer's shapes,
    dtypes and page tables, different values, and valid atom indices."""
    import numpy as np
    import torch
    w = synth.make_workload("c1", seed=4)
    dw = synth.to_device(w, "cpu")
    lw = synth.layer_like(dw, seed=11, cfg="c1")
    for k, v in dw.items():
        if torch.is_tensor(v):
            assert lw[k].shape == v.shape and lw[k].dtype == v.dtype, k
    for k in ("hot_refs", "cold_refs", "hot_indptr", "cold_indptr"):
        assert lw[k] is dw[k]
    for k in ("q", "hot_k", "k_dict", "v_dict"):
        assert not torch.equal(lw[k], dw[k])
    idx = lw["k_codes"].numpy().view(np.uint16).reshape(-1, 8)[:, :4]
    assert idx.max() < w["dict_size"]
    co = lw["v_codes"].numpy().view(np.uint16).reshape(-1, 8)[:, 4:].view(np.float16).astype(np.float32)
    assert 0.3 < float(co.std()) < 0.7  # coefficients ~ N(0, 0.5)
