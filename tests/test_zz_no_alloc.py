"""The allocation-free hot-pool decode (weaver_hot_decode_noalloc) against
the plan-based entry point on the same inputs.

It exists for callers that must not allocate device memory once they run (a
serving loop with a budget fixed at start-up, or a host whose device memory
belongs to another allocator), which therefore cannot create a plan.  Its
scratch is a fixed array inside the library, shared by every call, so the test
makes two calls in a row and checks both.  This file is collected last so a
run that stops at the first failure has run every other test first; it also
passes alone in a fresh process."""
import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("q_heads,kv_heads,head_dim,hot_tokens", [
    (32, 8, 128, 4096),   # the Llama-3-8B shape of the headline configuration
    (8, 8, 64, 272),      # G = 1, d = 64, a block count that is not a multiple of 4
    (16, 2, 128, 16),     # G = 8, one block
])
def test_noalloc_matches_plan_path_twice(oracle_mod, q_heads, kv_heads, head_dim, hot_tokens):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    from aether_nexus_b200 import WeaverEngine, WeaverPlan, synth
    from aether_nexus_b200.weaver import hot_decode_noalloc
    w = synth.make_workload("c1", seed=31, flag_refs=True, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
                            hot_tokens=hot_tokens, cold_tokens=0, shuffle_pages=True, spare_blocks=3)
    dw = synth.to_device(w)
    eng = WeaverEngine(0)
    plan = WeaverPlan(eng, num_seqs=1, num_queries=1, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
                      dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                      cold_indptr=w["cold_indptr"])
    ref = torch.empty((q_heads, head_dim), dtype=torch.float16, device="cuda")
    plan.run(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=None, cold_v=None,
             cold_refs=None, k_dict=None, v_dict=None, out=ref, cold_pool_blocks=0)
    plan.status()
    ref_np = ref.float().cpu().numpy()
    q = dw["q"].view(q_heads, head_dim)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(2):
        out = torch.full((q_heads, head_dim), float("nan"), dtype=torch.float16, device="cuda")
        hot_decode_noalloc(q, dw["hot_k"], dw["hot_v"], dw["hot_refs"], out, bad, scale=w["scale"])
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
    assert int(bad.item()) == 0
    full = oracle_mod.config_decode(w, precision="f64").reshape(q_heads, head_dim)
    for o in outs:
        assert_close(o, ref_np, what="noalloc vs plan")
        assert_close(o, full, what="noalloc vs oracle")
    plan.close()
    eng.close()


def test_noalloc_rejects_oversized_and_flags_bad_refs():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    from aether_nexus_b200 import synth
    from aether_nexus_b200.weaver import hot_decode_noalloc
    w = synth.make_workload("c1", seed=32, hot_tokens=64, cold_tokens=0)
    dw = synth.to_device(w)
    q = dw["q"].view(w["q_heads"], w["head_dim"])
    out = torch.empty_like(q)
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    from aether_nexus_b200 import _native as N
    # more blocks than the fixed maximum: refused by the C entry point before
    # any launch (the refs pointer is never read)
    st = N.lib().weaver_hot_decode_noalloc(w["q_heads"], w["kv_heads"], w["head_dim"], float(w["scale"]),
                                           q.data_ptr(), dw["hot_k"].data_ptr(), dw["hot_v"].data_ptr(),
                                           int(dw["hot_k"].shape[0]), dw["hot_refs"].data_ptr(), (1 << 24) + 1,
                                           out.data_ptr(), bad.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert st == 8
    with pytest.raises(ValueError):  # the wrapper refuses a count beyond the refs supplied
        hot_decode_noalloc(q, dw["hot_k"], dw["hot_v"], dw["hot_refs"], out, bad, scale=w["scale"],
                           n_blocks=int(dw["hot_refs"].numel()) + 1)
    refs = dw["hot_refs"].clone()
    refs[1] = 1 << 20  # beyond the pool: skipped and flagged, nothing read
    hot_decode_noalloc(q, dw["hot_k"], dw["hot_v"], refs, out, bad, scale=w["scale"])
    torch.cuda.synchronize()
    assert int(bad.item()) == 1
