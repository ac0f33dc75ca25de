"""Atom selection on the tensor cores (tcgen05 GEMM + exact re-scoring of the
candidates) against the CPU rule of distiller.rs:185-234, bit for bit, and
against the CUDA-core kernel.  Needs a B200."""
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    return torch


def _run(rows, kvh, dic, *, stride=None, stats=False):
    import torch
    from aether_nexus_b200 import distill
    from aether_nexus_b200.weaver import distill_stats
    r = torch.from_numpy(np.ascontiguousarray(rows)).cuda()
    d = torch.from_numpy(np.ascontiguousarray(dic)).cuda()
    out = torch.full((rows.shape[0], 8), -1, dtype=torch.int16, device="cuda")
    diag = None
    if stats:
        diag = torch.zeros(4, dtype=torch.int32, device="cuda")
        distill_stats(r, kvh, d, out, diag, dict_head_stride=stride)
    else:
        distill(r, kvh, d, out, dict_head_stride=stride)
    torch.cuda.synchronize()
    codes = out.cpu().numpy().view(np.uint16)
    if stats:
        dg = diag.cpu().numpy()
        return codes, float(dg[0:1].view(np.float32)[0]), int(dg[1]), int(dg[2])
    return codes


def _oracle(oracle_mod, rows, kvh, dic, stride=None):
    return oracle_mod.distill_rows(rows, kvh, dic, dict_head_stride=stride).view(np.uint16).reshape(-1, 8)


def _f16(rng, shape, std):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float16)


CASES = {
    # c2-shaped: 8 blocks x 16 tokens x 8 kv heads, 4096 atoms of d 128
    "c2": dict(n=1024, kvh=8, d=128, A=4096, x_std=1.0, d_std=1 / 11.3),
    "d64": dict(n=512, kvh=8, d=64, A=512, x_std=1.0, d_std=1 / 8),
    "ragged_atoms": dict(n=300, kvh=3, d=128, A=1000, x_std=0.5, d_std=0.3),
    "few_atoms": dict(n=64, kvh=2, d=64, A=5, x_std=1.0, d_std=1.0),
    "wide_values": dict(n=256, kvh=4, d=128, A=768, x_std=300.0, d_std=50.0),
}


@pytest.mark.parametrize("name", list(CASES))
def test_tensor_core_selection_bit_exact(torch_cuda, oracle_mod, name, monkeypatch):
    c = CASES[name]
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    rows = _f16(rng, (c["n"], c["d"]), c["x_std"])
    dic = _f16(rng, (c["kvh"], c["A"], c["d"]), c["d_std"])
    ref = _oracle(oracle_mod, rows, c["kvh"], dic)
    got, ratio, n_fb, status = _run(rows, c["kvh"], dic, stats=True)
    assert status == 0
    assert np.array_equal(got, ref), f"{name}: {int((got != ref).any(axis=1).sum())} rows differ"
    # the error bound holds with room to spare on every re-scored atom
    assert 0.0 <= ratio < 0.25, ratio
    assert np.array_equal(_run(rows, c["kvh"], dic), ref)
    monkeypatch.setenv("WEAVER_DISTILL_CUDA_CORES", "1")
    assert np.array_equal(_run(rows, c["kvh"], dic), ref)


def test_ties_fall_back_to_the_exact_scan(torch_cuda, oracle_mod):
    """Twelve identical best atoms: no list of 8 can hold every candidate, so
    the rows go to the exact full scan, which breaks the tie by index."""
    rng = np.random.default_rng(7)
    kvh, d, A, n = 2, 128, 700, 64
    rows = _f16(rng, (n, d), 1.0)
    dic = _f16(rng, (kvh, A, d), 0.1)
    for g in range(kvh):
        best = rows[g].astype(np.float32) / np.linalg.norm(rows[g].astype(np.float32))
        for a in (5, 17, 99, 100, 101, 250, 251, 400, 401, 402, 650, 699):
            dic[g, a] = best.astype(np.float16)
    ref = _oracle(oracle_mod, rows, kvh, dic)
    got, ratio, n_fb, status = _run(rows, kvh, dic, stats=True)
    assert status == 0 and n_fb >= 2
    assert np.array_equal(got, ref)
    assert [int(x) for x in got[0][:4]] == [5, 17, 99, 100]


def test_degenerate_inputs(torch_cuda, oracle_mod):
    """Zero dictionary (every score +-0: atoms 0..3), zero rows, subnormal
    rows, an infinite and a NaN entry (exact scan), shared dictionary."""
    rng = np.random.default_rng(11)
    kvh, d, A = 4, 128, 512
    zero_dic = np.zeros((kvh, A, d), np.float16)
    rows = _f16(rng, (64, d), 1.0)
    got, _, n_fb, status = _run(rows, kvh, zero_dic, stats=True)
    assert status == 0 and n_fb == 0
    assert np.array_equal(got, _oracle(oracle_mod, rows, kvh, zero_dic))

    dic = _f16(rng, (kvh, A, d), 0.2)
    rows = _f16(rng, (64, d), 1.0)
    rows[3] = 0
    rows[5] = (rows[5].astype(np.float32) * 1e-6).astype(np.float16)  # subnormal f16 values
    rows[6, :64] = (rows[6, :64].astype(np.float32) * 1e-6).astype(np.float16)
    rows[9, 7] = np.float16(np.inf)
    dic[1, 33, 4] = np.float16(np.nan)
    dic[2, 40] = (dic[2, 40].astype(np.float32) * 1e-5).astype(np.float16)
    got, _, n_fb, status = _run(rows, kvh, dic, stats=True)
    assert status == 0 and n_fb >= 1
    assert np.array_equal(got, _oracle(oracle_mod, rows, kvh, dic))

    shared = _f16(rng, (1, A, d), 0.2)
    assert np.array_equal(_run(rows, kvh, shared, stride=0), _oracle(oracle_mod, rows, kvh, shared, stride=0))
