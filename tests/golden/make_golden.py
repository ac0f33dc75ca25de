"""Generate the golden fixtures in this directory.

Run from the repository root (needs the reference source to build
``oracle/_ref``):  ``python tests/golden/make_golden.py``

* ``literal.npz`` — outputs of the reference's own ``weaver_decode`` kernel
  (``nexus-core/src/weaver_kernel.metal:118-240`` compiled unmodified as host
  C++, ``oracle/Makefile`` target ``ref``) for seeded random inputs in the
  reference's geometry (head_dim 128, dict_size 512), plus the two known
  answers of the reference's own inputs (``weaver.rs:369-396``: every output
  1.0; ``bench.rs:186-228``: every output f16(0.00802)).
* ``config.npz`` — configuration-mode outputs of the fp64 C oracle for small
  seeded workloads (c1 in full and reduced c3/c4/c5 shapes).
* ``distill.npz`` — atom selections of the C restatement of
  ``distiller.rs:185-234`` (zero-dictionary known answer and random rows with
  planted ties).
* ``mha.npz`` — outputs of the reference's own ``multihead_attention`` kernel
  (``nexus-core/src/ops.metal:528-616``, the whole ``ops.metal`` compiled
  unmodified as host C++) for seeded random queries and caches
  (``python tests/golden/make_golden.py mha`` rewrites only this file).

Inputs are not stored: each case stores its generator arguments and a
SHA-256 of the generated input bytes, so a change in the generator is caught
instead of silently comparing different data.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
from aether_nexus_b200 import synth  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

LITERAL_CASES = {
    "lit_g4_seed0": dict(q_heads=8, kv_heads=2, hot_count=3, cold_count=2, seed=0),
    "lit_g1_seed1": dict(q_heads=4, kv_heads=4, hot_count=2, cold_count=3, seed=1),
    "lit_g8_seed2": dict(q_heads=16, kv_heads=2, hot_count=4, cold_count=4, seed=2),
    "lit_hot_only_seed3": dict(q_heads=8, kv_heads=2, hot_count=3, cold_count=0, seed=3),
    "lit_cold_only_seed4": dict(q_heads=8, kv_heads=2, hot_count=0, cold_count=3, seed=4),
}

CONFIG_CASES = {
    "c1": dict(cfg="c1", seed=0, flag_refs=True),
    "c3_small": dict(cfg="c3", seed=1, flag_refs=True, num_seqs=3, hot_tokens=96, cold_tokens=400,
                     spare_blocks=5),
    "c4_small": dict(cfg="c4", seed=2, num_seqs=2, hot_tokens=64, cold_tokens=256, dict_size=256),
    "c5_small": dict(cfg="c5", seed=3, hot_tokens=128, cold_tokens=512, dict_size=1024),
}

LITERAL_KEYS = ("q_exact", "q_latent", "hot_pool", "cold_pool", "loom_refs", "dictionary")
CONFIG_KEYS = ("q", "hot_k", "hot_v", "hot_refs", "hot_indptr", "k_codes", "v_codes", "cold_refs",
               "cold_indptr", "k_dict", "v_dict")


def digest(arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).view(np.uint8).tobytes())
    return h.hexdigest()


def literal_inputs(case: dict):
    return synth.make_literal_workload(**case)


def kat_inputs(kind: str):
    """The reference's own test (weaver.rs:369-396) and bench (bench.rs:186-228)
    inputs.  Their loom_refs (0..hot+cold) address cold blocks from index
    hot_count on; the reference reads its zero-initialised preallocated buffer
    there, so the cold pool here covers those blocks with zero codes."""
    qh, kvh, d, A = 32, 8, 128, 512
    hot, cold, val = (2, 1, 1.0) if kind == "weaver_rs_test" else (64, 16, 0.01)
    v = np.float16(val)
    return dict(
        params=dict(q_heads=qh, kv_heads=kvh, head_dim=d, block_size=16, gqa_group=qh // kvh, hot_count=hot,
                    cold_count=cold, dict_size=A, sparsity_k=4),
        q_exact=np.full(qh * d, v), q_latent=np.full(qh * A, v), hot_pool=np.full(hot * 16 * kvh * d, v),
        cold_pool=np.zeros((hot + cold) * 16 * kvh, dtype=synth.SPARSE_CODE_DTYPE),
        loom_refs=np.arange(hot + cold, dtype=np.uint32), dictionary=np.full(kvh * A * d, v))


def distill_inputs(seed: int):
    rng = np.random.default_rng(seed)
    kvh, d, A, n = 2, 64, 96, 40
    rows = (rng.standard_normal((n, d), dtype=np.float32) * 0.5).astype(np.float16)
    dic = (rng.standard_normal((kvh, A, d), dtype=np.float32) * 0.5).astype(np.float16)
    dic[:, 7] = dic[:, 3]    # planted exact ties: equal scores, distinct indices
    dic[:, 50] = dic[:, 3]
    dic[1, 11] = 0           # a zero atom
    return rows, kvh, dic


MHA_CASES = {
    "decode_g4": dict(T=37, nq=1, Hq=8, Hkv=2, d=64, seed=0),
    "verify_g4": dict(T=300, nq=8, Hq=16, Hkv=4, d=128, seed=1),
    "prompt_g1": dict(T=64, nq=16, Hq=4, Hkv=4, d=128, seed=2),
    "minimal_g8": dict(T=3, nq=3, Hq=16, Hkv=2, d=64, seed=3),
}


def mha_inputs(case: dict):
    """q [nq, Hq, d] and caches [T + 5, Hkv, d] (rows past T are never read)."""
    rng = np.random.default_rng(case["seed"])
    nq, Hq, Hkv, d, T = case["nq"], case["Hq"], case["Hkv"], case["d"], case["T"]
    q = rng.standard_normal((nq, Hq, d), dtype=np.float32).astype(np.float16)
    k = rng.standard_normal((T + 5, Hkv, d), dtype=np.float32).astype(np.float16)
    v = rng.standard_normal((T + 5, Hkv, d), dtype=np.float32).astype(np.float16)
    return q, k, v


def make_mha(manifest: dict) -> None:
    out = {}
    manifest["mha"] = {}
    for name, case in MHA_CASES.items():
        q, k, v = mha_inputs(case)
        ref = O.mha(q, k, v, case["T"], reference_kernel=True)
        assert np.array_equal(ref.view(np.uint16), O.mha(q, k, v, case["T"]).view(np.uint16)), name
        out[name] = ref
        manifest["mha"][name] = dict(args=case, sha256=digest([q, k, v]))
    np.savez_compressed(os.path.join(HERE, "mha.npz"), **out)


def main() -> None:
    if not (O.ref_available() and O.ref_ops_available()):
        O.build(with_ref=True)
    if sys.argv[1:] == ["mha"]:
        path = os.path.join(HERE, "manifest.json")
        with open(path) as f:
            manifest = json.load(f)
        make_mha(manifest)
        with open(path, "w") as f:
            json.dump(manifest, f, indent=1, sort_keys=True)
        print("wrote mha.npz")
        return
    lit, manifest = {}, {"literal": {}, "config": {}, "distill": {}}
    for name, case in LITERAL_CASES.items():
        w = literal_inputs(case)
        out = O.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"], use_reference_kernel=True)
        mine = O.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"])
        assert np.array_equal(out.view(np.uint16), mine.view(np.uint16)), name
        lit[name] = out
        manifest["literal"][name] = dict(args=case, sha256=digest([w[k] for k in LITERAL_KEYS]))
    for kind in ("weaver_rs_test", "bench_rs"):
        w = kat_inputs(kind)
        out = O.literal_decode(*[w[k] for k in LITERAL_KEYS], w["params"], use_reference_kernel=True)
        lit["kat_" + kind] = out
        manifest["literal"]["kat_" + kind] = dict(args=kind, sha256=digest([w[k] for k in LITERAL_KEYS]))
    np.savez_compressed(os.path.join(HERE, "literal.npz"), **lit)

    cfg_out = {}
    for name, case in CONFIG_CASES.items():
        c = dict(case)
        w = synth.make_workload(c.pop("cfg"), c.pop("seed"), flag_refs=c.pop("flag_refs", False), **c)
        cfg_out[name] = O.config_decode(w, precision="f64")
        manifest["config"][name] = dict(args=case, sha256=digest([w[k] for k in CONFIG_KEYS]))
    np.savez_compressed(os.path.join(HERE, "config.npz"), **cfg_out)

    dis = {}
    zero_rows = np.zeros((16 * 8, 128), np.float16)
    dis["kat_zero_dict"] = O.distill_rows(zero_rows, 8, np.zeros((8, 512, 128), np.float16)).view(np.uint16)
    manifest["distill"]["kat_zero_dict"] = dict(args="zero block, zero dictionary (distiller.rs:286-307)")
    for seed in (0, 1):
        rows, kvh, dic = distill_inputs(seed)
        dis[f"random_seed{seed}"] = O.distill_rows(rows, kvh, dic).view(np.uint16)
        manifest["distill"][f"random_seed{seed}"] = dict(args=seed, sha256=digest([rows, dic]))
    np.savez_compressed(os.path.join(HERE, "distill.npz"), **dis)
    make_mha(manifest)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1, sort_keys=True)
    print("wrote", sorted(lit), sorted(cfg_out), sorted(dis))


if __name__ == "__main__":
    main()
