"""The full loop's multi-query attention (ops.metal:528-616, inference.rs:
552-562) on the GPU through weaver_multihead_attention, against the oracle
restatement (itself pinned bit for bit to the reference kernel) and the
committed fixtures.  Needs a B200."""
import os

import numpy as np
import pytest

from conftest import ROOT, assert_close, golden

pytestmark = pytest.mark.gpu

import importlib.util  # noqa: E402

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(ROOT, "tests", "golden", "make_golden.py"))
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)


@pytest.fixture(scope="module")
def engine():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    from aether_nexus_b200 import WeaverEngine
    e = WeaverEngine.new(None, 0)
    yield e
    e.close()


def _gpu(engine, q, k, v, T):
    import torch
    tq, tk, tv = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, k, v))
    out = torch.full(q.shape, float("nan"), dtype=torch.float16, device="cuda")
    engine.multihead_attention(tq, tk, tv, out, T)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("name", sorted(make_golden.MHA_CASES))
def test_mha_matches_reference_fixtures(engine, name):
    case = make_golden.MHA_CASES[name]
    q, k, v = make_golden.mha_inputs(case)
    assert_close(_gpu(engine, q, k, v, case["T"]), golden("mha.npz")[name], what=name)


CASES = {
    # speculative verify at c4's shape: 8 drafts over a 4096-token cache, 32 q / 8 kv heads
    "verify_c4": dict(T=4096, nq=8, Hq=32, Hkv=8, d=128),
    # decode over a cache whose length is not a multiple of 16, several chunks
    "decode_ragged": dict(T=4100, nq=1, Hq=32, Hkv=8, d=128),
    # a long cache (beyond the reference's 4096-entry score array)
    "decode_long": dict(T=20000, nq=1, Hq=64, Hkv=8, d=128),
    # a prompt chunk: 16 queries, rows of two 16-row tiles per kv head
    "prompt_chunk": dict(T=700, nq=16, Hq=8, Hkv=2, d=64),
    # odd GQA group (6) and queries that fill the whole cache
    "group6_full": dict(T=5, nq=5, Hq=12, Hkv=2, d=128),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_mha_matches_oracle(engine, oracle_mod, name):
    c = CASES[name]
    rng = np.random.default_rng(len(name) * 7919 + c["T"])
    q = rng.standard_normal((c["nq"], c["Hq"], c["d"]), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((c["T"] + 16, c["Hkv"], c["d"]), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((c["T"] + 16, c["Hkv"], c["d"]), dtype=np.float32).astype(np.float16)
    k[c["T"]:] = np.float16(np.inf)  # past the cache length: never read
    got = _gpu(engine, q, k, v, c["T"])
    ref = oracle_mod.mha(q, k, v, c["T"])
    assert_close(got, ref, what=name)
    assert np.array_equal(got, _gpu(engine, q, k, v, c["T"]))  # deterministic


def test_mha_refuses_bad_geometry(engine):
    import torch
    from aether_nexus_b200._native import WeaverError
    q = torch.zeros((4, 8, 128), dtype=torch.float16, device="cuda")
    kc = torch.zeros((16, 2, 128), dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    with pytest.raises(WeaverError):
        engine.multihead_attention(q, kc, kc, out, 3)  # total_kv_len < num_queries
    with pytest.raises(WeaverError):
        engine.multihead_attention(q[:, :, :96].contiguous(), kc[:, :, :96].contiguous(), kc[:, :, :96].contiguous(),
                                   out[:, :, :96].contiguous(), 8)  # head_dim 96
