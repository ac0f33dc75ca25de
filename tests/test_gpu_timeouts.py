"""Device-side waits give up on their own: every wait in the kernels (an
mbarrier phase, a dependency counter, a peer's (value, tag) word in the fused
split-KV merge) is bounded, records DEVERR_TIMEOUT and lets the kernel finish.
Here each kind of wait is pointed at a condition nothing will satisfy, with a
short limit (no fault, no hang: the wait itself ends), and the CUDA context is
shown to be usable afterwards by an ordinary decode checked against the
oracle.  Needs a B200."""
import ctypes

import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu

DEVERR_TIMEOUT = 4


def test_bounded_waits_expire_cleanly(oracle_mod):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    from aether_nexus_b200 import WeaverEngine, WeaverPlan, synth
    from aether_nexus_b200 import _native as N
    torch.cuda.set_device(0)
    mask = ctypes.c_uint32(0)
    waited = (ctypes.c_uint64 * 3)()
    status = (ctypes.c_uint32 * 6)()
    limit_us = 2000
    N.check(N.lib().weaver_wait_selftest(limit_us, ctypes.byref(mask), waited, status))
    assert mask.value == 0b111, f"waits that gave up: {mask.value:03b}"
    for i in range(3):
        assert limit_us * 1000 <= waited[i] < 200 * limit_us * 1000, (i, waited[i])
        assert status[2 * i] & DEVERR_TIMEOUT
        assert status[2 * i + 1] >> 31 == 1  # the first expired wait recorded its site
    sites = sorted(status[2 * i + 1] & 0xFF for i in range(3))
    assert sites == [26, 30, 31]
    # the context is intact: an ordinary step still matches the oracle
    w = synth.make_workload("c1", seed=61)
    dw = synth.to_device(w)
    eng = WeaverEngine(0)
    plan = WeaverPlan(eng, num_seqs=1, num_queries=1, q_heads=w["q_heads"], kv_heads=w["kv_heads"],
                      head_dim=w["head_dim"], dict_size=w["dict_size"], scale=w["scale"],
                      hot_indptr=w["hot_indptr"], cold_indptr=w["cold_indptr"])
    out = torch.empty(w["q"].shape, dtype=torch.float16, device="cuda")
    plan.run(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=dw["k_codes"],
             cold_v=dw["v_codes"], cold_refs=dw["cold_refs"], k_dict=dw["k_dict"], v_dict=dw["v_dict"], out=out)
    plan.status()
    assert_close(out.float().cpu().numpy(), oracle_mod.config_decode(w, precision="f64"), what="after timeouts")
    plan.close()
    eng.close()
