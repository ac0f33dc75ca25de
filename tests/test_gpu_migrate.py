"""Hot -> cold migration on the GPU (distiller.rs:52-246 as device work):
block entropy against the oracle, block-list distillation bit-exact against
the oracle's atom selection, and a decode over the rewritten page tables
against the oracle.  Needs a B200."""
import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    return torch


def _workload(seed=5):
    """c1-shaped layer with spare cold blocks, every hot block but each
    sequence's newest scaled to std 0.3 (proxy ~0.09 < 0.15) except one that
    is zeroed (proxy 0: never a candidate) and one left at std 1."""
    from aether_nexus_b200 import synth
    w = synth.make_workload("c1", seed=seed, spare_blocks=16, shuffle_pages=True, num_seqs=2, hot_tokens=128,
                            cold_tokens=256)
    refs = w["hot_refs"] & np.uint32(0x7FFFFFFF)
    low = [int(b) for b in refs[:-1]]
    for b in low:
        w["hot_k"][b] = (w["hot_k"][b].astype(np.float32) * 0.3).astype(np.float16)
        w["hot_v"][b] = (w["hot_v"][b].astype(np.float32) * 0.3).astype(np.float16)
    w["hot_k"][low[0]] = 0
    w["hot_v"][low[0]] = 0
    w["hot_k"][low[1]] = (w["hot_k"][low[1]].astype(np.float32) / 0.3).astype(np.float16)
    return w


def test_block_entropy_matches_oracle(torch_cuda, oracle_mod):
    """distiller.rs:128-159: the variance proxy of every block, fp64
    accumulation.  The sums of f16 values are exact in fp64 at these
    magnitudes; the squared deviations round, so the f32 results may differ
    in the last place only."""
    from aether_nexus_b200 import migrate, synth
    w = _workload()
    dw = synth.to_device(w)
    got = migrate.block_entropy(dw["hot_k"], w["kv_heads"]).cpu().numpy()
    ref = np.array([oracle_mod.block_entropy(w["hot_k"][b]) for b in range(w["hot_k"].shape[0])], np.float32)
    np.testing.assert_allclose(got, ref, rtol=2.0 ** -23, atol=0)
    zero = int(w["hot_refs"][0] & 0x7FFFFFFF)
    assert got[zero] == 0.0
    # a pool of ragged size (not a multiple of the 8 blocks one CTA covers)
    got5 = migrate.block_entropy(dw["hot_k"][:5].contiguous(), w["kv_heads"]).cpu().numpy()
    np.testing.assert_array_equal(got5, got[:5])


def test_migrate_low_entropy_codes_and_decode(torch_cuda, oracle_mod):
    """One REM cycle: candidates chosen from the GPU proxy, K and V rows of
    each moved block encoded bit-exactly as the oracle's distill_block
    (distiller.rs:185-234) into free cold blocks, the other cold blocks
    untouched, and the decode over the new page tables equal to the oracle's
    on the migrated workload."""
    import torch
    from aether_nexus_b200 import WeaverEngine, WeaverPlan, migrate, synth
    w = _workload()
    dw = synth.to_device(w)
    Hkv, d = w["kv_heads"], w["head_dim"]
    used = set(int(x) for x in (w["cold_refs"] & np.uint32(0x7FFFFFFF)))
    free = [b for b in range(w["k_codes"].shape[0]) if b not in used]
    k_before = dw["k_codes"].cpu().numpy().copy()
    mig = migrate.migrate_low_entropy(hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=w["hot_refs"],
                                      hot_indptr=w["hot_indptr"], cold_refs=w["cold_refs"],
                                      cold_indptr=w["cold_indptr"], free_cold_blocks=free, k_dict=dw["k_dict"],
                                      v_dict=dw["v_dict"], cold_k=dw["k_codes"], cold_v=dw["v_codes"])
    torch.cuda.synchronize()
    refs = w["hot_refs"] & np.uint32(0x7FFFFFFF)
    zero = int(refs[0])
    assert zero not in set(mig.src_blocks.tolist())          # proxy 0 stays hot
    assert int(refs[1]) not in set(mig.src_blocks.tolist())  # proxy ~1 stays hot
    assert len(mig.src_blocks) >= 4
    k_after = dw["k_codes"].cpu().numpy()
    v_after = dw["v_codes"].cpu().numpy()
    for s, t in zip(mig.src_blocks.tolist(), mig.dst_blocks.tolist()):
        rk = oracle_mod.distill_rows(w["hot_k"][s].reshape(-1, d), Hkv, w["k_dict"])
        rv = oracle_mod.distill_rows(w["hot_v"][s].reshape(-1, d), Hkv, w["v_dict"])
        assert np.array_equal(k_after[t].reshape(-1).view(np.uint8), rk.view(np.uint8).reshape(-1)), (s, t)
        assert np.array_equal(v_after[t].reshape(-1).view(np.uint8), rv.view(np.uint8).reshape(-1)), (s, t)
    untouched = [b for b in range(k_after.shape[0]) if b not in set(mig.dst_blocks.tolist())]
    assert np.array_equal(k_after[untouched], k_before[untouched])
    # every block still referenced exactly once, block counts conserved
    assert len(mig.hot_refs) + len(mig.cold_refs) == len(w["hot_refs"]) + len(w["cold_refs"])
    assert int(mig.hot_indptr[-1]) == len(mig.hot_refs) and int(mig.cold_indptr[-1]) == len(mig.cold_refs)

    w2 = dict(w, hot_refs=mig.hot_refs, hot_indptr=mig.hot_indptr, cold_refs=mig.cold_refs,
              cold_indptr=mig.cold_indptr, k_codes=k_after.view(w["k_codes"].dtype).reshape(w["k_codes"].shape),
              v_codes=v_after.view(w["v_codes"].dtype).reshape(w["v_codes"].shape))
    ref = oracle_mod.config_decode(w2)
    eng = WeaverEngine.new(None, 0)
    try:
        B, nq, Hq, _ = w["q"].shape
        plan = WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=Hkv, head_dim=d,
                          dict_size=w["dict_size"], scale=w["scale"], hot_indptr=mig.hot_indptr,
                          cold_indptr=mig.cold_indptr, causal=bool(w["causal"]))
        out = torch.full((B, nq, Hq, d), float("nan"), dtype=torch.float16, device="cuda")
        plan.run(out=out, q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"],
                 hot_refs=torch.from_numpy(mig.hot_refs.view(np.int32)).cuda(), cold_k=dw["k_codes"],
                 cold_v=dw["v_codes"], cold_refs=torch.from_numpy(mig.cold_refs.view(np.int32)).cuda(),
                 k_dict=dw["k_dict"], v_dict=dw["v_dict"])
        plan.status()
        assert_close(out.cpu().numpy(), ref, what="decode after migration")
    finally:
        eng.close()


def test_migrate_blocks_flags_out_of_range(torch_cuda, oracle_mod):
    """An out-of-range source or destination block is skipped and reported
    in the flag; the valid entries of the same call are still written."""
    import torch
    from aether_nexus_b200 import migrate, synth
    w = _workload(seed=9)
    dw = synth.to_device(w)
    nb, nc = w["hot_k"].shape[0], w["k_codes"].shape[0]
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    src = torch.tensor([2, nb, 3], dtype=torch.int32, device="cuda")
    dst = torch.tensor([nc - 1, 0, nc], dtype=torch.int32, device="cuda")
    before = dw["k_codes"].cpu().numpy().copy()
    migrate.migrate_blocks(dw["hot_k"], dw["hot_v"], src, dst, dw["k_dict"], dw["v_dict"], dw["k_codes"],
                           dw["v_codes"], bad)
    torch.cuda.synchronize()
    assert int(bad.item()) == 1
    after = dw["k_codes"].cpu().numpy()
    ref = oracle_mod.distill_rows(w["hot_k"][2].reshape(-1, w["head_dim"]), w["kv_heads"], w["k_dict"])
    assert np.array_equal(after[nc - 1].reshape(-1).view(np.uint8), ref.view(np.uint8).reshape(-1))
    assert np.array_equal(after[:nc - 1], before[:nc - 1])
