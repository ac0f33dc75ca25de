"""Split-KV across ranks without a GPU: block sharding, the log-sum-exp
combine, and a world-size-2 gloo run whose gathered partials (from the CPU
oracle, one shard per rank) reproduce the full decode."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, assert_close
from aether_nexus_b200 import split_kv, synth


@pytest.mark.parametrize("n,world", [(0, 2), (1, 2), (5, 2), (7, 3), (64, 8), (3, 8)])
def test_shard_ranges_cover_disjoint_tail_last(n, world):
    spans = [split_kv.shard_ranges(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (lo, hi), (lo2, _) in zip(spans, spans[1:]):
        assert lo <= hi == lo2
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1
    if n:
        assert sizes[-1] >= 1  # the last rank holds the sequence's tail


def _partials(oracle_mod, w):
    out, m, l_, o = oracle_mod.config_decode(w, precision="f64", partials=True)
    rows = m.size
    return m.reshape(rows), l_.reshape(rows), o.reshape(rows, -1)


@pytest.mark.parametrize("cfg,over,world", [
    ("c1", {}, 2),
    ("c1", dict(num_seqs=3, hot_tokens=80, cold_tokens=300), 3),
    ("c4", dict(num_seqs=2, hot_tokens=64, cold_tokens=256, dict_size=256), 2),  # causal, nq = 8
])
def test_sharded_partials_combine_to_full(oracle_mod, cfg, over, world):
    w = synth.make_workload(cfg, seed=5, **over)
    full = oracle_mod.config_decode(w, precision="f64")
    parts = [_partials(oracle_mod, split_kv.shard_workload(w, r, world)) for r in range(world)]
    m = np.stack([p[0] for p in parts])
    l_ = np.stack([p[1] for p in parts])
    o = np.stack([p[2] for p in parts])
    got = split_kv.combine_partials(m, l_, o)
    assert_close(got.reshape(full.shape), full, what=f"{cfg} x{world}")
    import torch
    got_t = split_kv.combine_partials(torch.from_numpy(m.astype(np.float32)), torch.from_numpy(l_.astype(np.float32)),
                                      torch.from_numpy(o.astype(np.float32)))
    assert_close(got_t.numpy().reshape(full.shape), full, what=f"{cfg} x{world} torch")


def test_combine_all_empty_rows_give_zeros():
    m = np.full((2, 3), -np.inf)
    l_ = np.zeros((2, 3))
    o = np.zeros((2, 3, 4))
    assert np.all(split_kv.combine_partials(m, l_, o) == 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result_path):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    import oracle as O
    from aether_nexus_b200 import split_kv as S
    from aether_nexus_b200 import synth as Y

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = Y.make_workload("c1", seed=12, num_seqs=2, hot_tokens=96, cold_tokens=400)
        out, m, l_, o = O.config_decode(S.shard_workload(w, rank, world), precision="f64", partials=True)
        rows = m.size
        pm = torch.from_numpy(m.reshape(rows).astype(np.float32))
        pl = torch.from_numpy(l_.reshape(rows).astype(np.float32))
        po = torch.from_numpy(o.reshape(rows, -1).astype(np.float32))
        merged = S.gather_and_combine(pm, pl, po)
        if rank == 0:
            np.save(result_path, merged.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_world2_split_kv_matches_full_decode(oracle_mod, tmp_path):
    import torch.multiprocessing as mp
    path = str(tmp_path / "merged.npy")
    mp.start_processes(_gloo_rank, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    w = synth.make_workload("c1", seed=12, num_seqs=2, hot_tokens=96, cold_tokens=400)
    full = oracle_mod.config_decode(w, precision="f64")
    assert_close(np.load(path).reshape(full.shape), full, what="gloo split-kv")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_shards_concatenate_to_full(oracle_mod, world):
    """Batched configs shard by kv head: every rank's heads are independent,
    so the shards' outputs side by side are the full output, bit for bit."""
    w = synth.make_workload("c3", seed=6, num_seqs=3, hot_tokens=64, cold_tokens=256, dict_size=256,
                            spare_blocks=2)
    full = oracle_mod.config_decode(w, precision="f64")
    outs = [oracle_mod.config_decode(split_kv.shard_heads(w, r, world), precision="f64") for r in range(world)]
    got = np.concatenate(outs, axis=2)
    assert np.array_equal(got.view(np.uint16), full.view(np.uint16))


def test_head_range_requires_even_split():
    with pytest.raises(ValueError):
        split_kv.head_range(8, 0, 3)
    assert [split_kv.head_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
