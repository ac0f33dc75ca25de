"""The NVLink peer-memory split-KV combine (weaver_combine_*): a world of one
rank (its own receive buffer, signalled by itself) against the packed merge of
the same partials, the combine fused into the step kernel on one rank, and two
ranks on two GPUs (skipped with fewer) against the oracle."""
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


def test_fused_combine_world_one_equals_plain_step(oracle_mod):
    """The split-KV merge fused into the step (weaver_plan_attach_combine) on
    one rank: the plan writes the merged output itself, over several steps
    (the step tag and the double buffer advance), equal to the same plan run
    without a combiner and to the oracle."""
    import torch
    import torch.distributed as dist

    from aether_nexus_b200 import WeaverEngine, WeaverPlan, synth
    from aether_nexus_b200.split_kv import P2PCombine

    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1)
    eng = WeaverEngine(0)
    comb = None
    try:
        w = synth.make_workload("c2", seed=43, hot_tokens=1024, cold_tokens=4096)
        dw = synth.to_device(w)
        B, nq, Hq, d = w["q"].shape
        plan = WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"], head_dim=d,
                          dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                          cold_indptr=w["cold_indptr"])
        kw = dict(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=dw["k_codes"],
                  cold_v=dw["v_codes"], cold_refs=dw["cold_refs"], k_dict=dw["k_dict"], v_dict=dw["v_dict"])
        ref = torch.empty((B, nq, Hq, d), dtype=torch.float16, device="cuda")
        plan.run(out=ref, **kw)
        plan.status()
        comb = P2PCombine(eng, B * nq * Hq, d)
        comb.attach(plan)
        for _ in range(3):
            out = torch.full_like(ref, float("nan"))
            plan.run(out=out, **kw)
            plan.status()
            assert torch.allclose(out.float(), ref.float(), atol=1e-3, rtol=1e-3)
        assert_close(out.cpu().numpy(), oracle_mod.config_decode(w, precision="f32", threads=0), what="fused combine")
        comb.detach()
        plan.close()
    finally:
        torch.cuda.synchronize()
        if comb is not None:
            comb.close()
        eng.close()
        dist.destroy_process_group()


def _two_rank_worker(rank, port, result_path):
    """One rank of the two-GPU split-KV test (spawned; GPU `rank`)."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from aether_nexus_b200 import WeaverEngine, WeaverPlan, split_kv, synth
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60))
    eng = WeaverEngine(rank)
    full = synth.make_workload("c2", seed=47, hot_tokens=2048, cold_tokens=8192)
    w = split_kv.shard_workload(full, rank, 2)
    dw = synth.to_device(w, f"cuda:{rank}")
    B, nq, Hq, d = w["q"].shape
    rows = B * nq * Hq
    kw = dict(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=dw["k_codes"],
              cold_v=dw["v_codes"], cold_refs=dw["cold_refs"], k_dict=dw["k_dict"], v_dict=dw["v_dict"])
    mk = lambda partials: WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"],  # noqa: E731
                                     head_dim=d, dict_size=w["dict_size"], scale=w["scale"],
                                     hot_indptr=w["hot_indptr"], cold_indptr=w["cold_indptr"], partials=partials)
    pk = torch.empty((rows * (d + 2),), dtype=torch.float32, device=f"cuda:{rank}")
    pplan = mk(True)
    fplan = mk(False)
    comb = split_kv.P2PCombine(eng, rows, d)
    outs = {}
    for step in range(3):
        pplan.run(part_m=pk[:rows], part_l=pk[rows:2 * rows], part_o=pk[2 * rows:].view(rows, d), **kw)
        o1 = torch.empty((rows, d), dtype=torch.float16, device=f"cuda:{rank}")
        comb.run(pk, o1)
        comb.status()
        outs.setdefault("kernel", []).append(o1.cpu())
    comb.attach(fplan)
    for step in range(3):
        o2 = torch.empty((B, nq, Hq, d), dtype=torch.float16, device=f"cuda:{rank}")
        fplan.run(out=o2, **kw)
        fplan.status()
        outs.setdefault("fused", []).append(o2.view(rows, d).cpu())
    torch.cuda.synchronize()
    dist.barrier()
    comb.detach()
    comb.close()
    if rank == 0:
        np.savez(result_path, **{f"{k}{i}": v.float().numpy() for k, vs in outs.items() for i, v in enumerate(vs)})
    dist.barrier()
    pplan.close()
    fplan.close()
    eng.close()
    dist.destroy_process_group()


def test_two_rank_split_kv_combines(oracle_mod, tmp_path):
    """Two ranks on two GPUs, one long context split by blocks: the combine
    kernel over peer memory and the combine fused into the step both give the
    oracle's full decode on every step (skipped with fewer than two GPUs)."""
    import torch
    import torch.multiprocessing as mp

    from aether_nexus_b200 import synth
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = str(tmp_path / "res.npz")
    mp.start_processes(_two_rank_worker, args=(_free_port(), path), nprocs=2, join=True, start_method="spawn")
    full = synth.make_workload("c2", seed=47, hot_tokens=2048, cold_tokens=8192)
    ref = oracle_mod.config_decode(full, precision="f32", threads=0).reshape(-1, full["head_dim"])
    res = np.load(path)
    for k in res.files:
        assert_close(res[k], ref, what=k)
