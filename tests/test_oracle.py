"""The CPU oracle pinned against the reference's own known answers, the
reference kernel source itself (oracle/_ref, when built here) and the
committed golden fixtures.  No GPU."""
import json
import os

import numpy as np
import pytest

from conftest import ROOT, assert_close, digest, golden
from aether_nexus_b200 import synth

LITERAL_KEYS = ("q_exact", "q_latent", "hot_pool", "cold_pool", "loom_refs", "dictionary")

sys_golden = os.path.join(ROOT, "tests", "golden")
with open(os.path.join(sys_golden, "manifest.json")) as f:
    MANIFEST = json.load(f)

import importlib.util  # noqa: E402

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(sys_golden, "make_golden.py"))
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)


def test_f16_conversion_matches_ieee(oracle_mod):
    O = oracle_mod
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.h2f(int(b)) for b in bits], dtype=np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    rng = np.random.default_rng(0)
    xs = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504, 65519.99, 65520, -65520, 1e-8, 2.98e-8, 5.96e-8, 6.1e-5,
                  6.103515625e-05, np.inf, -np.inf], np.float32),
        # exact ties between binary16 neighbours
        (np.arange(1, 2000, dtype=np.float32) * 2 + 1) * np.float32(2 ** -11),
    ]).astype(np.float32)
    got = np.array([O.f2h(float(x)) for x in xs], dtype=np.uint16)
    assert np.array_equal(got, xs.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("kind,value", [("weaver_rs_test", 1.0), ("bench_rs", 0.0080221)])
def test_reference_known_answers(oracle_mod, kind, value):
    """weaver.rs:369-396 inputs give 1.0 everywhere; bench.rs:186-228 inputs
    give f16(0.0080221)."""
    w = make_golden.kat_inputs(kind)
    out = oracle_mod.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"])
    assert out.shape == (32 * 128,)
    assert np.all(out == np.float16(value))
    assert np.array_equal(out.view(np.uint16), golden("literal.npz")["kat_" + kind].view(np.uint16))


@pytest.mark.parametrize("name", sorted(make_golden.LITERAL_CASES))
def test_literal_restatement_matches_reference_kernel(oracle_mod, name):
    case = make_golden.LITERAL_CASES[name]
    w = make_golden.literal_inputs(case)
    assert digest([w[k] for k in LITERAL_KEYS]) == MANIFEST["literal"][name]["sha256"]
    out = oracle_mod.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"])
    assert np.array_equal(out.view(np.uint16), golden("literal.npz")[name].view(np.uint16))
    if oracle_mod.ref_available():
        ref = oracle_mod.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"], use_reference_kernel=True)
        assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))


def test_literal_out_of_range_ref_is_refused(oracle_mod):
    w = make_golden.literal_inputs(make_golden.LITERAL_CASES["lit_g4_seed0"])
    w["loom_refs"] = w["loom_refs"].copy()
    w["loom_refs"][-1] = 7  # cold pool has 2 blocks
    with pytest.raises(ValueError):
        oracle_mod.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"])


def _config_case(name):
    c = dict(make_golden.CONFIG_CASES[name])
    return synth.make_workload(c.pop("cfg"), c.pop("seed"), flag_refs=c.pop("flag_refs", False), **c)


@pytest.mark.parametrize("name", sorted(make_golden.CONFIG_CASES))
def test_config_oracle_matches_golden(oracle_mod, name):
    w = _config_case(name)
    assert digest([w[k] for k in make_golden.CONFIG_KEYS]) == MANIFEST["config"][name]["sha256"]
    out = oracle_mod.config_decode(w, precision="f64")
    assert np.array_equal(out.view(np.uint16), golden("config.npz")[name].view(np.uint16))
    out32 = oracle_mod.config_decode(w, precision="f32", threads=2)
    assert_close(out32, out, what=name)


def test_config_mode_with_literal_settings_equals_literal_mode(oracle_mod):
    """scale 1, V = K, one code set, supplied q_latent: the configuration-mode
    algorithm reduces to the reference kernel."""
    lw = synth.make_literal_workload(seed=11, q_heads=8, kv_heads=2, hot_count=3, cold_count=2)
    p = lw["params"]
    d, A, Hkv, Hq = p["head_dim"], p["dict_size"], p["kv_heads"], p["q_heads"]
    hot = lw["hot_pool"].reshape(-1, 16, Hkv, d)
    cold = lw["cold_pool"].reshape(-1, 16, Hkv)
    cw = dict(num_seqs=1, num_queries=1, q_heads=Hq, kv_heads=Hkv, head_dim=d, dict_size=A, scale=1.0,
              causal=0, q=lw["q_exact"].reshape(1, 1, Hq, d), q_latent=lw["q_latent"].reshape(1, 1, Hq, A),
              hot_k=hot, hot_v=hot, hot_refs=lw["loom_refs"][:3].copy(),
              hot_indptr=np.array([0, 3], np.uint32), k_codes=cold, v_codes=cold,
              cold_refs=lw["loom_refs"][3:].copy(), cold_indptr=np.array([0, 2], np.uint32),
              k_dict=None, v_dict=lw["dictionary"].reshape(Hkv, A, d))
    a = oracle_mod.config_decode(cw, precision="f64").reshape(-1)
    b = oracle_mod.literal_decode(*[lw[k] for k in LITERAL_KEYS], p)
    assert_close(a, b, atol=1e-4, rtol=2e-3)


def test_partials_recombine_to_full(oracle_mod):
    """Splitting a sequence's blocks in two and merging the (m, l, o)
    partials by log-sum-exp reproduces the single decode."""
    w = synth.make_workload("c1", seed=4)
    full = oracle_mod.config_decode(w, precision="f64").astype(np.float32)
    parts = []
    for half in range(2):
        v = dict(w)
        for side in ("hot", "cold"):
            n = int(w[f"{side}_indptr"][-1])
            lo, hi = (0, n // 2) if half == 0 else (n // 2, n)
            v[f"{side}_refs"] = w[f"{side}_refs"][lo:hi].copy()
            v[f"{side}_indptr"] = np.array([0, hi - lo], np.uint32)
        parts.append(oracle_mod.config_decode(v, precision="f64", partials=True)[1:])
    m = np.stack([p[0] for p in parts])
    l_ = np.stack([p[1] for p in parts])
    o = np.stack([p[2] for p in parts])
    M = m.max(0)
    f = np.exp(m - M)
    merged = (o * f[..., None]).sum(0) / (l_ * f).sum(0)[..., None]
    assert_close(merged, full, atol=1e-3, rtol=1e-3)


def test_distill_zero_dictionary_known_answer(oracle_mod):
    """distiller.rs:286-307: zero dictionary -> indices [0, 1, 2, 3]."""
    codes = oracle_mod.distill_rows(np.zeros((16 * 8, 128), np.float16), 8, np.zeros((8, 512, 128), np.float16))
    assert (codes["indices"] == np.array([0, 1, 2, 3], np.uint16)).all()
    assert (codes["coeffs"] == 0).all()
    assert np.array_equal(codes.view(np.uint16), golden("distill.npz")["kat_zero_dict"])


def _numpy_distill(rows, kvh, dic):
    """Independent restatement: sequential fp32 dot from -0.0, rank by
    (score desc, index asc), top 4, coefficient f16(score)."""
    out = []
    for i, x in enumerate(rows.astype(np.float32)):
        D = dic[i % kvh].astype(np.float32)
        prods = D * x[None, :]
        s = np.full(D.shape[0], -0.0, np.float32)
        for j in range(D.shape[1]):
            s = (s + prods[:, j]).astype(np.float32)
        order = sorted(range(len(s)), key=lambda a: (-float(s[a]), a))[:4]
        out.append((order, [np.float16(s[a]) for a in order]))
    return out


@pytest.mark.parametrize("seed", [0, 1])
def test_distill_matches_independent_rule_and_golden(oracle_mod, seed):
    rows, kvh, dic = make_golden.distill_inputs(seed)
    assert digest([rows, dic]) == MANIFEST["distill"][f"random_seed{seed}"]["sha256"]
    codes = oracle_mod.distill_rows(rows, kvh, dic)
    for c, (idx, co) in zip(codes, _numpy_distill(rows, kvh, dic)):
        assert list(c["indices"]) == idx
        assert np.array_equal(np.asarray(c["coeffs"], np.uint16), np.array(co, np.float16).view(np.uint16))
    assert np.array_equal(codes.view(np.uint16), golden("distill.npz")[f"random_seed{seed}"])
    # planted ties (atoms 3, 7, 50 equal): lower index first whenever they are selected
    for c in codes:
        sel = [int(i) for i in c["indices"]]
        tied = [i for i in sel if i in (3, 7, 50)]
        assert tied == sorted(tied)


def test_block_entropy_known_answers(oracle_mod):
    """distiller.rs:261-283."""
    assert oracle_mod.block_entropy(np.zeros(512, np.uint16)) == 0.0
    assert oracle_mod.block_entropy(np.full(512, np.float16(1.0))) < 1e-3
    v = np.array([0.0, 1.0, 2.0, 3.0], np.float16)
    assert abs(oracle_mod.block_entropy(v) - 1.25) < 1e-6


@pytest.mark.parametrize("name", sorted(make_golden.MHA_CASES))
def test_mha_restatement_matches_reference_kernel(oracle_mod, name):
    """oracle_mha (ops.metal:528-616 restated) equals the reference's own
    multihead_attention kernel bit for bit: against the committed fixture,
    and against the compiled kernel itself where oracle/_ref exists."""
    case = make_golden.MHA_CASES[name]
    q, k, v = make_golden.mha_inputs(case)
    assert digest([q, k, v]) == MANIFEST["mha"][name]["sha256"]
    got = oracle_mod.mha(q, k, v, case["T"])
    assert np.array_equal(got.view(np.uint16), golden("mha.npz")[name].view(np.uint16))
    if oracle_mod.ref_ops_available():
        ref = oracle_mod.mha(q, k, v, case["T"], reference_kernel=True)
        assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


def test_mha_causal_rule_and_refusals(oracle_mod):
    """Query i sees positions < T - nq + 1 + i (ops.metal:549): changing the
    cache at position T - nq + 1 + i changes rows > i only; T < nq is refused."""
    rng = np.random.default_rng(5)
    nq, Hq, Hkv, d, T = 4, 4, 2, 64, 20
    q = rng.standard_normal((nq, Hq, d), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((T, Hkv, d), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((T, Hkv, d), dtype=np.float32).astype(np.float16)
    base = oracle_mod.mha(q, k, v, T)
    k2, v2 = k.copy(), v.copy()
    k2[T - nq + 1 + 1] += np.float16(1.0)
    v2[T - nq + 1 + 1] += np.float16(1.0)
    moved = oracle_mod.mha(q, k2, v2, T)
    assert np.array_equal(moved[:2].view(np.uint16), base[:2].view(np.uint16))
    assert not np.array_equal(moved[2:].view(np.uint16), base[2:].view(np.uint16))
    with pytest.raises(ValueError):
        oracle_mod.mha(q, k, v, nq - 1)
