"""Parity of the CUDA path (through the C ABI) with the CPU oracle and the
reference's golden fixtures.  Needs a B200."""
import json
import os

import numpy as np
import pytest

from conftest import ROOT, assert_close, golden

pytestmark = pytest.mark.gpu

LITERAL_KEYS = ("q_exact", "q_latent", "hot_pool", "cold_pool", "loom_refs", "dictionary")

import importlib.util  # noqa: E402

_spec = importlib.util.spec_from_file_location("make_golden", os.path.join(ROOT, "tests", "golden", "make_golden.py"))
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    return torch


@pytest.fixture(scope="module")
def engine(torch_cuda):
    from aether_nexus_b200 import WeaverEngine
    e = WeaverEngine.new(None, 0)
    yield e
    e.close()


def run_plan(engine, w, *, partials=False, dict_head_stride=None, k_dict=None, v_dict=None, stream=None):
    import torch
    from aether_nexus_b200 import WeaverPlan, synth
    dw = synth.to_device(w)
    B, nq, Hq, d = w["q"].shape
    plan = WeaverPlan(engine, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"], head_dim=d,
                      dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                      cold_indptr=w["cold_indptr"], causal=bool(w["causal"]), partials=partials)
    out = torch.full((B, nq, Hq, d), float("nan"), dtype=torch.float16, device="cuda")
    kw = dict(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=dw["k_codes"],
              cold_v=dw["v_codes"], cold_refs=dw["cold_refs"],
              k_dict=dw["k_dict"] if k_dict is None else k_dict, v_dict=dw["v_dict"] if v_dict is None else v_dict,
              dict_head_stride=dict_head_stride)
    if partials:
        pm = torch.empty((B, nq, Hq), dtype=torch.float32, device="cuda")
        pl = torch.empty_like(pm)
        po = torch.empty((B, nq, Hq, d), dtype=torch.float32, device="cuda")
        plan.run(part_m=pm, part_l=pl, part_o=po, stream=stream, **kw)
        plan.status()
        return pm, pl, po
    plan.run(out=out, stream=stream, **kw)
    plan.status()
    return out.cpu().numpy()


def test_engine_pipeline(engine):
    """weaver.rs:334-356: the engine comes up on the device."""
    assert "B200" in engine.device_name() or engine.device_name()
    assert engine.max_threads_per_threadgroup() >= 32


@pytest.mark.parametrize("kind", ["weaver_rs_test", "bench_rs"])
def test_reference_known_answers_through_engine(engine, kind):
    """weaver.rs:359-420 and bench.rs:186-228 inputs through WeaverEngine.decode."""
    from aether_nexus_b200 import WeaverParams
    w = make_golden.kat_inputs(kind)
    out = engine.decode(*[w[k] for k in LITERAL_KEYS], WeaverParams(**w["params"])).data
    assert out.shape == (32 * 128,)
    ref = golden("literal.npz")["kat_" + kind]
    assert_close(out, ref, what=kind)
    if kind == "weaver_rs_test":
        assert np.all(out == np.float16(1.0))


@pytest.mark.parametrize("name", sorted(make_golden.LITERAL_CASES))
def test_literal_fixtures_through_engine(engine, name):
    """Outputs of the reference kernel itself (tests/golden/literal.npz)."""
    from aether_nexus_b200 import WeaverParams
    w = make_golden.literal_inputs(make_golden.LITERAL_CASES[name])
    for _ in range(2):  # second call reuses the engine's buffers and cached plan
        out = engine.decode(*[w[k] for k in LITERAL_KEYS], WeaverParams(**w["params"])).data
        assert_close(out, golden("literal.npz")[name], what=name)


def test_host_decode_rejects_out_of_range_refs(engine):
    from aether_nexus_b200 import WeaverError, WeaverParams
    w = make_golden.literal_inputs(make_golden.LITERAL_CASES["lit_g4_seed0"])
    w["loom_refs"] = w["loom_refs"].copy()
    w["loom_refs"][0] = 9  # hot pool has 3 blocks
    with pytest.raises(WeaverError) as e:
        engine.decode(*[w[k] for k in LITERAL_KEYS], WeaverParams(**w["params"]))
    assert e.value.status == 4


def _config_case(name):
    from aether_nexus_b200 import synth
    c = dict(make_golden.CONFIG_CASES[name])
    return synth.make_workload(c.pop("cfg"), c.pop("seed"), flag_refs=c.pop("flag_refs", False), **c)


@pytest.mark.parametrize("name", sorted(make_golden.CONFIG_CASES))
def test_config_fixtures(engine, name):
    w = _config_case(name)
    out = run_plan(engine, w)
    assert_close(out, golden("config.npz")[name], what=name)


@pytest.mark.parametrize("cfg,over", [
    ("c2", {}),
    ("c5", {}),
    ("c3", {}),   # the configured shape: 64 sequences, jittered lengths, shuffled 16-token pages
    ("c4", {}),   # the configured shape: 16 sequences x 8 causal drafts, 4096 hot + 28672 cold
    ("c3", dict(num_seqs=6, hot_tokens=512, cold_tokens=2048, spare_blocks=7)),
    ("c4", dict(num_seqs=2, hot_tokens=1024, cold_tokens=4096)),
])
def test_configs_against_oracle(engine, oracle_mod, cfg, over):
    from aether_nexus_b200 import synth
    w = synth.make_workload(cfg, seed=7, flag_refs=True, **over)
    out = run_plan(engine, w)
    ref = oracle_mod.config_decode(w, precision="f32", threads=0)
    assert_close(out, ref, what=cfg)


@pytest.mark.parametrize("case", [
    dict(hot_tokens=0, cold_tokens=512),                      # cold only
    dict(hot_tokens=512, cold_tokens=0),                      # hot only
    dict(hot_tokens=0, cold_tokens=0),                        # nothing to attend: zeros
    dict(hot_tokens=16, cold_tokens=16),                      # one block each
    dict(dict_size=300),                                      # atoms not a multiple of the tile
    dict(q_heads=16, kv_heads=8, head_dim=64),                # d = 64, G = 2
    dict(q_heads=64, kv_heads=8, head_dim=64, num_queries=8, causal=True, hot_tokens=64),  # R = 64
    dict(num_queries=3, causal=True, hot_tokens=16),          # causal with one hot block
    dict(q_heads=12, kv_heads=2, dict_size=640),              # G = 6 (DeepSeek-R1 1.5B shape)
])
def test_edge_cases(engine, oracle_mod, case):
    from aether_nexus_b200 import synth
    w = synth.make_workload("c1", seed=3, flag_refs=True, **case)
    out = run_plan(engine, w)
    ref = oracle_mod.config_decode(w, precision="f64")
    assert_close(out, ref, what=str(case))
    if case.get("hot_tokens") == 0 and case.get("cold_tokens") == 0:
        assert np.all(out == 0)


def test_shared_dictionary_head_stride_zero(engine, oracle_mod):
    import torch
    from aether_nexus_b200 import synth
    w = synth.make_workload("c1", seed=9, q_heads=8, kv_heads=4)
    w["k_dict"] = np.ascontiguousarray(np.broadcast_to(w["k_dict"][:1], w["k_dict"].shape))
    w["v_dict"] = np.ascontiguousarray(np.broadcast_to(w["v_dict"][:1], w["v_dict"].shape))
    kd = torch.from_numpy(w["k_dict"][0].copy()).cuda()
    vd = torch.from_numpy(w["v_dict"][0].copy()).cuda()
    out = run_plan(engine, w, dict_head_stride=0, k_dict=kd, v_dict=vd)
    assert_close(out, oracle_mod.config_decode(w, precision="f64"), what="shared dict")


def test_out_of_range_indices_are_flagged_not_read(engine, oracle_mod):
    """A bad block ref or atom index is skipped by the kernels' bounds checks
    and reported by the status call (no fault)."""
    from aether_nexus_b200 import WeaverError, synth
    w = synth.make_workload("c1", seed=5)
    w["hot_refs"] = w["hot_refs"].copy()
    w["hot_refs"][3] = 10_000
    with pytest.raises(WeaverError) as e:
        run_plan(engine, w)
    assert e.value.status == 4
    w = synth.make_workload("c1", seed=5)
    w["k_codes"] = w["k_codes"].copy()
    w["k_codes"]["indices"][0, 0, 0, 2] = 600  # dict_size is 512
    with pytest.raises(WeaverError) as e:
        run_plan(engine, w)
    assert e.value.status == 4
    # the plan recovers: a clean run afterwards passes
    w = synth.make_workload("c1", seed=5)
    assert_close(run_plan(engine, w), oracle_mod.config_decode(w, precision="f64"))


def test_split_kv_partials_merge(engine, oracle_mod):
    """The multi-GPU combine: two block ranges decoded separately with
    partial outputs, merged by weaver_merge_partials."""
    import torch
    from aether_nexus_b200 import merge_partials, synth
    w = synth.make_workload("c5", seed=2, hot_tokens=256, cold_tokens=2048, dict_size=1024)
    full = oracle_mod.config_decode(w, precision="f64")
    ms, ls, os_ = [], [], []
    for half in range(2):
        v = dict(w)
        for side in ("hot", "cold"):
            n = int(w[f"{side}_indptr"][-1])
            lo, hi = (0, n // 2) if half == 0 else (n // 2, n)
            v[f"{side}_refs"] = w[f"{side}_refs"][lo:hi].copy()
            v[f"{side}_indptr"] = np.array([0, hi - lo], np.uint32)
        pm, pl, po = run_plan(engine, v, partials=True)
        ms.append(pm.reshape(-1))
        ls.append(pl.reshape(-1))
        os_.append(po.reshape(-1, po.shape[-1]))
    out = torch.empty_like(os_[0], dtype=torch.float16)
    merge_partials(torch.stack(ms), torch.stack(ls), torch.stack(os_), out)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy().reshape(full.shape), full, what="split-kv merge")
    # the packed layout one all-gather produces: per part [m rows | l rows | o rows*d]
    from aether_nexus_b200 import merge_partials_packed
    rows, d = int(os_[0].shape[0]), int(os_[0].shape[1])
    gathered = torch.cat([torch.cat([m_, l2, o2.reshape(-1)]) for m_, l2, o2 in zip(ms, ls, os_)])
    out2 = torch.empty_like(out)
    merge_partials_packed(gathered, 2, rows, d, out2)
    torch.cuda.synchronize()
    assert torch.equal(out2, out)


def test_repeated_runs_and_streams(engine, oracle_mod):
    import torch
    from aether_nexus_b200 import synth
    w = synth.make_workload("c1", seed=8)
    ref = oracle_mod.config_decode(w, precision="f64")
    s = torch.cuda.Stream()
    for _ in range(3):
        assert_close(run_plan(engine, w, stream=s), ref)


def _distill_gpu(rows, kvh, dic):
    import torch
    from aether_nexus_b200 import distill
    r = torch.from_numpy(rows).cuda()
    d = torch.from_numpy(np.ascontiguousarray(dic)).cuda()
    out = torch.zeros((rows.shape[0], 8), dtype=torch.int16, device="cuda")
    distill(r, kvh, d, out)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


def test_distill_bit_exact(engine, oracle_mod):
    """GPU atom selection == distiller.rs rule, bit for bit."""
    for seed in (0, 1):
        rows, kvh, dic = make_golden.distill_inputs(seed)
        got = _distill_gpu(rows, kvh, dic)
        assert np.array_equal(got, golden("distill.npz")[f"random_seed{seed}"].reshape(got.shape))
        assert np.array_equal(got, _distill_gpu(rows, kvh, dic))  # deterministic
    got = _distill_gpu(np.zeros((128, 128), np.float16), 8, np.zeros((8, 512, 128), np.float16))
    assert np.array_equal(got, golden("distill.npz")["kat_zero_dict"].reshape(got.shape))
    rng = np.random.default_rng(3)
    rows = rng.standard_normal((16 * 8, 128), dtype=np.float32).astype(np.float16)
    dic = (rng.standard_normal((8, 4096, 128), dtype=np.float32) / 11).astype(np.float16)
    ref = oracle_mod.distill_rows(rows, 8, dic).view(np.uint16).reshape(-1, 8)
    assert np.array_equal(_distill_gpu(rows, 8, dic), ref)


@pytest.mark.parametrize("cfg,over", [("c2", {}), ("c1", {}), ("c3", dict(num_seqs=5, hot_tokens=256, cold_tokens=1024))])
def test_fused_step_matches_multikernel_path(engine, cfg, over, monkeypatch):
    """The single-kernel step and the multi-kernel pipeline agree (the plan
    picks the fused kernel whenever the geometry qualifies)."""
    from aether_nexus_b200 import synth
    w = synth.make_workload(cfg, seed=21, flag_refs=True, **over)
    monkeypatch.setenv("WEAVER_PREFER_FUSED", "1")
    fused = run_plan(engine, w)
    monkeypatch.setenv("WEAVER_DISABLE_FUSED", "1")
    multi = run_plan(engine, w)
    assert_close(fused, multi, atol=1e-3, rtol=5e-3, what=cfg)


@pytest.mark.parametrize("cfg,over", [
    ("c2", {}),
    ("c1", {}),
    ("c1", dict(q_heads=16, kv_heads=8, num_queries=2, causal=True, hot_tokens=48)),
    ("c3", dict(num_seqs=3, hot_tokens=256, cold_tokens=1024, spare_blocks=3)),
])
def test_head_partitioned_step_matches_general_fused_step(engine, oracle_mod, cfg, over, monkeypatch):
    """The head-partitioned kernel (chosen when one kv head's q_latent and
    per-atom weights fit in shared memory) agrees with the general fused
    kernel and with the oracle."""
    from aether_nexus_b200 import synth
    w = synth.make_workload(cfg, seed=23, flag_refs=True, **over)
    hp = run_plan(engine, w)
    monkeypatch.setenv("WEAVER_DISABLE_HP", "1")
    general = run_plan(engine, w)
    assert_close(hp, general, atol=1e-3, rtol=5e-3, what=cfg)
    assert_close(hp, oracle_mod.config_decode(w, precision="f32", threads=0), what=cfg)


def test_head_partitioned_partials_merge_across_shards(engine, oracle_mod):
    """The head-partitioned kernel's (m, l, o) partial outputs (what each rank
    of a split-KV run produces): two block shards of a c2-shaped sequence,
    merged, equal the full decode."""
    import torch
    from aether_nexus_b200 import merge_partials, split_kv, synth
    w = synth.make_workload("c2", seed=31, hot_tokens=1024, cold_tokens=6144)
    full = oracle_mod.config_decode(w, precision="f32", threads=0)
    ms, ls, os_ = [], [], []
    for rank in range(2):
        pm, pl, po = run_plan(engine, split_kv.shard_workload(w, rank, 2), partials=True)
        ms.append(pm.reshape(-1))
        ls.append(pl.reshape(-1))
        os_.append(po.reshape(-1, po.shape[-1]))
    out = torch.empty_like(os_[0], dtype=torch.float16)
    merge_partials(torch.stack(ms), torch.stack(ls), torch.stack(os_), out)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy().reshape(full.shape), full, what="hp split-kv merge")


@pytest.mark.parametrize("case", ["one_atom", "peaked", "wide_coeffs"])
def test_cold_accumulation_extremes(engine, oracle_mod, case):
    """The cold path's per-atom sums at their extremes: every V code on one
    atom (the largest possible sum of one atom's terms), sharply peaked scores
    (scale 1: a few tokens dominate the softmax, most weights underflow
    relative to them) and coefficients spanning many orders of magnitude."""
    from aether_nexus_b200 import synth
    over = dict(hot_tokens=512, cold_tokens=8192)
    if case == "peaked":
        over["scale"] = 1.0
    w = synth.make_workload("c2", seed=51, **over)
    if case == "one_atom":
        w["v_codes"] = w["v_codes"].copy()
        w["v_codes"]["indices"][:] = 7
    if case == "wide_coeffs":
        rng = np.random.default_rng(5)
        w["v_codes"] = w["v_codes"].copy()
        mag = np.float32(2.0) ** rng.integers(-14, 8, size=w["v_codes"]["coeffs"].shape).astype(np.float32)
        sign = np.where(rng.integers(0, 2, size=mag.shape) == 1, 1.0, -1.0).astype(np.float32)
        w["v_codes"]["coeffs"] = (mag * sign).astype(np.float16)
    out = run_plan(engine, w)
    assert_close(out, oracle_mod.config_decode(w, precision="f64"), what=case)


@pytest.mark.parametrize("cfg,over", [
    ("c4", dict(num_seqs=2, hot_tokens=1024, cold_tokens=2048)),
    ("c4", dict(num_seqs=1, num_queries=16, hot_tokens=300, cold_tokens=512, q_heads=32, kv_heads=8)),
    ("c1", dict(num_queries=4, q_heads=16, kv_heads=4, causal=True)),
    ("c5", dict(hot_tokens=1000, cold_tokens=1024, dict_size=1024)),
])
def test_hot_tensor_core_pass_matches_cuda_cores(engine, oracle_mod, cfg, over, monkeypatch):
    """At 8+ query rows per kv head the multi-kernel step's hot pass runs on
    mma.sync tiles (weaver_hot_mma.cu; c5's 8 rows fill half a tile); it
    agrees with the oracle and with the CUDA-core hot kernel
    (WEAVER_HOT_CUDA_CORES=1)."""
    from aether_nexus_b200 import synth
    monkeypatch.setenv("WEAVER_DISABLE_FUSED", "1")
    w = synth.make_workload(cfg, seed=31, flag_refs=True, **over)
    tc = run_plan(engine, w)
    assert_close(tc, oracle_mod.config_decode(w, precision="f32"), what=f"{cfg} tensor-core hot pass")
    monkeypatch.setenv("WEAVER_HOT_CUDA_CORES", "1")
    cc = run_plan(engine, w)
    assert_close(tc, cc, atol=1e-3, rtol=5e-3, what=f"{cfg} vs CUDA-core hot pass")


@pytest.mark.parametrize("over", [dict(num_seqs=2, hot_tokens=1024, cold_tokens=2048),
                                  dict(num_seqs=1, num_queries=16, hot_tokens=256, cold_tokens=1000)])
def test_cold_row_lane_passes_match(engine, oracle_mod, over, monkeypatch):
    """At 32+ query rows per kv head the cold score and scatter passes run one
    warp per token with a lane per query row (coalesced gathers and weight
    updates); they agree with the oracle and with the thread-per-token passes
    (WEAVER_COLD_PER_THREAD=1)."""
    from aether_nexus_b200 import synth
    monkeypatch.setenv("WEAVER_COLD_L2", "1")  # the L2 passes (not the shared-memory ones)
    w = synth.make_workload("c4", seed=37, flag_refs=True, **over)
    rows = run_plan(engine, w)
    assert_close(rows, oracle_mod.config_decode(w, precision="f32"), what="row-lane cold passes")
    monkeypatch.setenv("WEAVER_COLD_PER_THREAD", "1")
    assert_close(rows, run_plan(engine, w), atol=1e-3, rtol=5e-3, what="row-lane vs thread-per-token")


@pytest.mark.parametrize("cfg,over", [
    ("c5", dict(hot_tokens=512, cold_tokens=16384)),
    ("c4", dict(num_seqs=10, num_queries=4, hot_tokens=256, cold_tokens=2048)),
    ("c4", dict(num_seqs=2, num_queries=4, hot_tokens=512, cold_tokens=2000)),
    ("c3", dict(num_seqs=5, hot_tokens=256, cold_tokens=1024, spare_blocks=3)),
    ("c1", dict(q_heads=8, kv_heads=8)),
    ("c1", dict(q_heads=16, kv_heads=8)),
])
def test_cold_shared_memory_passes_match(engine, oracle_mod, cfg, over, monkeypatch):
    """The multi-kernel step's cold passes with the q_latent slice and the
    per-atom weight table in shared memory (weaver_cold_smem.cu): c5's 8192
    atoms x 8 rows in two 4-row slices, 16 rows (4 causal drafts x 4 q heads)
    in two 8-row slices with whole-sequence chunks (plain stores) and with
    split sequences (vector reductions), jittered batches, 1 and 2 rows.  They
    agree with the oracle and with the L2 gather / reduction passes
    (WEAVER_COLD_L2=1)."""
    from aether_nexus_b200 import synth
    monkeypatch.setenv("WEAVER_DISABLE_FUSED", "1")
    w = synth.make_workload(cfg, seed=43, flag_refs=True, **over)
    smem = run_plan(engine, w)
    assert_close(smem, oracle_mod.config_decode(w, precision="f32", threads=0), what=f"{cfg} shared-memory cold")
    monkeypatch.setenv("WEAVER_COLD_L2", "1")
    assert_close(smem, run_plan(engine, w), atol=1e-3, rtol=5e-3, what=f"{cfg} vs L2 cold passes")


@pytest.mark.parametrize("v_scale", [1024.0, 1.0 / 1024.0])
def test_cold_fixed_point_scatter_falls_back(engine, oracle_mod, v_scale, monkeypatch):
    """The shared-memory scatter accumulates in fixed point with a per-row
    scale guessed from the K coefficients; V coefficients 1024x larger (the
    integer sums would overflow) or 1024x smaller (too few bits) than the K
    ones make every CTA reject the integer table and redo the pass in fp32,
    and the result still matches the oracle and the L2 passes."""
    from aether_nexus_b200 import synth
    monkeypatch.setenv("WEAVER_DISABLE_FUSED", "1")
    w = synth.make_workload("c5", seed=53, hot_tokens=256, cold_tokens=8192, dict_size=2048)
    w["v_codes"] = w["v_codes"].copy()
    w["v_codes"]["coeffs"] = (w["v_codes"]["coeffs"].astype(np.float32) * np.float32(v_scale)).astype(np.float16)
    smem = run_plan(engine, w)
    assert_close(smem, oracle_mod.config_decode(w, precision="f64"), what=f"V coefficients x{v_scale}")
    monkeypatch.setenv("WEAVER_COLD_L2", "1")
    assert_close(smem, run_plan(engine, w), atol=1e-3, rtol=5e-3, what=f"x{v_scale} vs L2 passes")


def test_cold_shared_memory_passes_flag_bad_indices(engine, oracle_mod, monkeypatch):
    """A bad cold block reference or atom index in the shared-memory passes
    is skipped and reported, and the next clean run passes."""
    from aether_nexus_b200 import WeaverError, synth
    monkeypatch.setenv("WEAVER_DISABLE_FUSED", "1")
    base = synth.make_workload("c5", seed=47, hot_tokens=256, cold_tokens=4096, dict_size=2048)
    w = dict(base)
    w["cold_refs"] = base["cold_refs"].copy()
    w["cold_refs"][5] = 1_000_000
    with pytest.raises(WeaverError) as e:
        run_plan(engine, w)
    assert e.value.status == 4
    w = dict(base)
    w["v_codes"] = base["v_codes"].copy()
    w["v_codes"]["indices"][3, 2, 1, 0] = 4000
    with pytest.raises(WeaverError) as e:
        run_plan(engine, w)
    assert e.value.status == 4
    assert_close(run_plan(engine, base), oracle_mod.config_decode(base, precision="f64"), what="after bad indices")


@pytest.mark.parametrize("cfg,big", [("c4", False), ("c4", True), ("c5", False), ("c5", True)])
def test_contraction_tensor_core_matches(engine, oracle_mod, cfg, big, monkeypatch):
    """At 8+ query rows per kv head the cold contraction w . V_dict runs on
    mma.sync tiles with f16 weights, each 64-atom slice scaled by a power of
    two below 2^15 (c5: one sequence, so the atoms split over CTAs into
    several cold partials); with coefficients up to 2^14 (weights far beyond
    the f16 range) it still matches the oracle and the fp32 CUDA-core
    contraction."""
    from aether_nexus_b200 import synth
    monkeypatch.setenv("WEAVER_DISABLE_FUSED", "1")
    if cfg == "c4":
        w = synth.make_workload("c4", seed=41, num_seqs=2, hot_tokens=512, cold_tokens=2048)
    else:
        w = synth.make_workload("c5", seed=41, hot_tokens=256, cold_tokens=4096)
    if big:
        rng = np.random.default_rng(8)
        w["v_codes"] = w["v_codes"].copy()
        w["v_codes"]["indices"][..., 0] = 3  # every token's first V term on one atom: a large sum
        mag = np.float32(2.0) ** rng.integers(8, 15, size=w["v_codes"]["coeffs"].shape).astype(np.float32)
        w["v_codes"]["coeffs"] = mag.astype(np.float16)
    tc = run_plan(engine, w)
    assert_close(tc, oracle_mod.config_decode(w, precision="f64"), what=f"tensor-core contraction big={big}")
    monkeypatch.setenv("WEAVER_CONTRACT_CUDA_CORES", "1")
    assert_close(tc, run_plan(engine, w), atol=1e-3, rtol=5e-3, what="vs CUDA-core contraction")
