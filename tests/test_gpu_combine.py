"""The NVLink peer-memory split-KV combine (weaver_combine_*) on one GPU: a
world of one rank writes into its own receive buffer, signals itself and
merges; the result equals the packed merge of the same partials.  The
multi-rank path is exercised by bench.py --gpus N, which checks it against
the NCCL all-gather + merge before timing."""
import socket

import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_p2p_combine_world_one_equals_packed_merge(oracle_mod):
    import torch
    import torch.distributed as dist

    from aether_nexus_b200 import WeaverEngine, WeaverPlan, merge_partials_packed, synth
    from aether_nexus_b200.split_kv import P2PCombine

    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1)
    eng = WeaverEngine(0)
    comb = None
    try:
        w = synth.make_workload("c2", seed=41, hot_tokens=512, cold_tokens=2048)
        dw = synth.to_device(w)
        B, nq, Hq, d = w["q"].shape
        rows = B * nq * Hq
        plan = WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"], head_dim=d,
                          dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                          cold_indptr=w["cold_indptr"], partials=True)
        pk = torch.empty((rows * (d + 2),), dtype=torch.float32, device="cuda")
        plan.run(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=dw["k_codes"],
                 cold_v=dw["v_codes"], cold_refs=dw["cold_refs"], k_dict=dw["k_dict"], v_dict=dw["v_dict"],
                 part_m=pk[:rows], part_l=pk[rows:2 * rows], part_o=pk[2 * rows:].view(rows, d))
        plan.status()
        ref = torch.empty((rows, d), dtype=torch.float16, device="cuda")
        merge_partials_packed(pk, 1, rows, d, ref)
        torch.cuda.synchronize()
        comb = P2PCombine(eng, rows, d)
        for _ in range(3):  # epochs advance; the double buffer alternates
            out = torch.full((rows, d), float("nan"), dtype=torch.float16, device="cuda")
            comb.run(pk, out)
            comb.status()
            assert torch.equal(out, ref)
        full = oracle_mod.config_decode(w, precision="f32", threads=0)
        assert_close(out.cpu().numpy().reshape(full.shape), full, what="p2p combine")
        plan.close()
    finally:
        torch.cuda.synchronize()
        if comb is not None:
            comb.close()
        eng.close()
        dist.destroy_process_group()
