#!/usr/bin/env python3
"""Weaver decode-attention benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c2]

A step is one decode step of the configuration (default c2: Llama-3-8B
shaped, 32 q / 8 kv heads, d 128, 4096 hot + 28672 cold tokens, 4096-atom
K/V dictionaries, batch 1) over one set of synthetic inputs resident in HBM.
Steps rotate over enough copies of the inputs that every step reads data
that is not in L2 (copies x bytes > 3 x 126 MB).  Each copy's step is one
CUDA graph (the plan's kernels); K graph replays are timed with CUDA events.

N > 1 (torchrun): every rank holds its own c2-sized shard of one long
context (weak scaling); each step decodes the shard and merges the ranks'
(m, l, o) partials inside the same kernel, pushing them over NVLink peer
memory (WEAVER_COMBINE=p2p: partials then a separate peer-memory combine
kernel; WEAVER_COMBINE=nccl: an NCCL all-gather + merge kernel instead).
--config c3 (batched) at N > 1 shards by kv head instead (strong scaling,
8/N kv heads per GPU, no collective); --config c5 (long context) at N > 1
splits one context's blocks across the ranks (strong scaling, same combine).

--impl reference times the CPU implementation of the path (the C oracle in
oracle/, a restatement of nexus-core/src/weaver_kernel.metal; the reference
itself is Metal/Rust and cannot run here) on the host cores.

--op distill measures the migration's atom selection instead (the Distiller's
distill_block, nexus-core/src/distiller.rs:171-246): a step encodes --blocks
hot blocks of the configuration's shape, every (token, kv head) row of K and V
against its head's dictionary, through weaver_migrate_blocks (tcgen05 GEMM +
exact re-scoring); the CUDA-core kernel of the same rule and the CPU rule are
timed beside it.  Its line has a tensor-core roofline.

--op mha measures the full loop's exact multi-query attention
(ops.metal:528-616 through weaver_multihead_attention): a step is one call
over a --kv-len cache (default 32768 positions, 8 kv heads, d 128) with 8
causal queries of 32 heads (the speculative-verify batch); HBM roofline over
the cache bytes read.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-attn KV tokens/s per GPU (hot+cold) and HBM GB/s vs peak, 1/2/4/8 B200"
UNIT = "KV tokens/s"
L2_BYTES = 126 * 2 ** 20
REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
           0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """NVML sampling of SM clock and clock-event reasons during the timed region."""

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples = []
        self.reasons = 0
        self.err = None
        self._stop = threading.Event()
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            pr = torch.cuda.get_device_properties(device_index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
            fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self._reasons = fn
        except Exception as e:  # NVML missing: report it rather than guess
            self.err = f"{type(e).__name__}: {e}"
        self.thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self._reasons(self.h))
            except Exception as e:
                self.err = str(e)
                return
            time.sleep(self.period)

    def start(self):
        if self.err is None:
            self.thread.start()

    def stop(self):
        self._stop.set()
        if self.thread.is_alive():
            self.thread.join()

    def summary(self):
        if self.err is not None and not self.samples:
            return {"error": self.err}
        names = [n for bit, n in REASONS.items() if self.reasons & bit and bit != 0x1]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples)}


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------
# reference arm: the CPU implementation on the host cores
# ----------------------------------------------------------------------------

def _window(w: dict, frac: float) -> dict:
    """The first `frac` of every sequence's hot and cold blocks (at least one each)."""
    if frac >= 1.0:
        return w
    v = dict(w)
    for side in ("hot", "cold"):
        ip = w[f"{side}_indptr"]
        refs, new_ip = [], [0]
        for b in range(len(ip) - 1):
            n = int(ip[b + 1] - ip[b])
            k = min(n, max(1, int(round(n * frac)))) if n else 0
            refs.append(w[f"{side}_refs"][ip[b]:ip[b] + k])
            new_ip.append(new_ip[-1] + k)
        v[f"{side}_refs"] = np.concatenate(refs).astype(np.uint32)
        v[f"{side}_indptr"] = np.array(new_ip, np.uint32)
    return v


def run_reference(args, rank: int) -> None:
    if rank != 0:
        return
    import oracle
    from aether_nexus_b200 import synth

    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(with_ref=False)
    w = synth.make_workload(args.config, seed=1000)
    threads = cpu_threads()
    t0 = time.perf_counter()
    oracle.config_decode(w, precision="f32", threads=threads)
    t_full = time.perf_counter() - t0
    budget = 120.0
    frac = min(1.0, budget / max(1e-9, (args.steps + args.warmup) * t_full))
    ws = _window(w, frac)
    tokens = synth.kv_tokens(ws)
    for _ in range(args.warmup):
        oracle.config_decode(ws, precision="f32", threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.config_decode(ws, precision="f32", threads=threads)
    dt = time.perf_counter() - t0
    value = tokens * args.steps / dt
    sample = (f"{args.config} decode over the first {frac:.4f} of every sequence's hot and cold blocks "
              f"({tokens} of {synth.kv_tokens(w)} KV tokens, all query rows) per step; fp32 C oracle, "
              f"OpenMP over query rows")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": args.config, "kv_tokens_per_step": tokens},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------

def host_views_for(w: dict, pinned: dict):
    from aether_nexus_b200 import _native as N
    v = N.ViewsC()
    v.q = pinned["q"].data_ptr()
    v.hot_k, v.hot_v = pinned["hot_k"].data_ptr(), pinned["hot_v"].data_ptr()
    v.hot_pool_blocks = int(w["hot_k"].shape[0])
    v.hot_refs = pinned["hot_refs"].data_ptr()
    v.cold_k, v.cold_v = pinned["k_codes"].data_ptr(), pinned["v_codes"].data_ptr()
    v.cold_pool_blocks = int(w["k_codes"].shape[0])
    v.cold_refs = pinned["cold_refs"].data_ptr()
    v.k_dict, v.v_dict = pinned["k_dict"].data_ptr(), pinned["v_dict"].data_ptr()
    v.dict_head_stride = w["dict_size"] * w["head_dim"]
    return v


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import ctypes

    import torch

    from aether_nexus_b200 import WeaverEngine, WeaverError, WeaverPlan, merge_partials_packed, synth
    from aether_nexus_b200 import _native as N

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    # batched configs shard by kv head (strong scaling: every rank decodes all
    # sequences for its 8/N kv heads, its resident pools hold only those heads,
    # no collective); the others split one long context per rank (weak scaling)
    head_sharded = world > 1 and args.config == "c3"
    if head_sharded:
        from aether_nexus_b200 import synth as _s
        base_cfg = _s.config(args.config)
        if base_cfg["kv_heads"] % world:
            raise SystemExit(f"{base_cfg['kv_heads']} kv heads do not split over {world} GPUs")
        per = base_cfg["kv_heads"] // world
        G = base_cfg["q_heads"] // base_cfg["kv_heads"]
        w = synth.make_workload(args.config, seed=1000, kv_heads=per, q_heads=per * G)  # same page tables
    elif world > 1 and args.config == "c5":
        # one long context split across the ranks (strong scaling): every rank
        # takes its run of the same sequence's hot and cold blocks
        from aether_nexus_b200.split_kv import shard_workload
        w = shard_workload(synth.make_workload(args.config, seed=1000), rank, world)
    else:
        w = synth.make_workload(args.config, seed=1000 + rank)
    context_split = world > 1 and args.config == "c5"
    units = 1 if head_sharded else world  # KV tokens counted once per step across ranks
    B, nq, Hq, d = w["q"].shape
    # multi-layer configurations (c3: 32 layers): a step decodes every layer,
    # each with its own pools, codes and dictionaries behind the same page tables
    layers = int(synth.config(args.config).get("layers", 1))
    if args.layers:  # a subset of a multi-layer configuration's layers (profiling a small case)
        layers = min(layers, args.layers)
    tokens = layers * synth.kv_tokens(w)
    bytes_alg = layers * synth.bytes_algorithmic(w)
    partials = world > 1 and not head_sharded
    if partials and layers > 1:
        raise SystemExit("multi-layer configurations are sharded by kv head, not split")
    eng = WeaverEngine(local_rank)
    plan = WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"], head_dim=d,
                      dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                      cold_indptr=w["cold_indptr"], causal=bool(w["causal"]), partials=partials)
    base = synth.to_device(w, dev)
    copies = max(1, min(64, math.ceil(3 * L2_BYTES / bytes_alg)))
    if bytes_alg * copies > 40e9:
        copies = max(1, int(40e9 // bytes_alg))
    rows = B * nq * Hq
    out = torch.empty((B, nq, Hq, d), dtype=torch.float16, device=dev)
    # partials packed [m rows | l rows | o rows*d] so one all-gather moves them
    pk = torch.empty((rows * (d + 2),), dtype=torch.float32, device=dev)
    pm, pl, po = pk[:rows], pk[rows:2 * rows], pk[2 * rows:].view(rows, d)
    if partials:
        gk = torch.empty((world * pk.numel(),), dtype=torch.float32, device=dev)
    # sets[c][layer]: the device inputs of input copy c; views[c][layer] their views
    sets, views, outs = [], [], [out] + [torch.empty_like(out) for _ in range(layers - 1)]
    for c in range(copies):
        t = base if c == 0 else {k: (v.clone() if torch.is_tensor(v) else v) for k, v in base.items()}
        ls = [t] + [synth.layer_like(t, seed=7919 * (c + 1) + 104729 * layer + rank, cfg=args.config)
                    for layer in range(1, layers)]
        sets.append(ls)
        views.append([plan.views(q=u["q"], hot_k=u["hot_k"], hot_v=u["hot_v"], hot_refs=u["hot_refs"],
                                 cold_k=u["k_codes"], cold_v=u["v_codes"], cold_refs=u["cold_refs"],
                                 k_dict=u["k_dict"], v_dict=u["v_dict"], out=None if partials else outs[layer],
                                 part_m=pm if partials else None, part_l=pl if partials else None,
                                 part_o=po if partials else None) for layer, u in enumerate(ls)])

    def run_partials(c, s):
        for v in views[c]:
            plan.run_views(v, s)

    def nccl_collective(stream):
        dist.all_gather_into_tensor(gk, pk)
        merge_partials_packed(gk, world, rows, d, out.view(rows, d), stream=stream)

    # N > 1 combine: "fused" (default) = the merge over ranks inside the step
    # kernel (weaver_plan_attach_combine, one kernel per step); "p2p" = the
    # step's partials then the peer-memory combine kernel; "nccl" = NCCL
    # all-gather of the partials + merge kernel
    mode = os.environ.get("WEAVER_COMBINE", "fused") if partials else None
    combiner = fplan = None
    if mode in ("fused", "p2p"):
        from aether_nexus_b200.split_kv import P2PCombine
        combiner = P2PCombine(eng, rows, d)
    if mode == "fused":
        fplan = WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"], head_dim=d,
                           dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                           cold_indptr=w["cold_indptr"], causal=bool(w["causal"]))
        try:
            combiner.attach(fplan)
        except WeaverError:
            # a shard whose step is not the head-partitioned single kernel
            # (a kernel pipeline or the general fused step): its partials,
            # then the peer-memory combine kernel (every rank has the same
            # geometry, so every rank takes this branch)
            fplan.close()
            fplan = None
            mode = "p2p"
        else:
            fviews = [[fplan.views(q=u["q"], hot_k=u["hot_k"], hot_v=u["hot_v"], hot_refs=u["hot_refs"],
                                   cold_k=u["k_codes"], cold_v=u["v_codes"], cold_refs=u["cold_refs"],
                                   k_dict=u["k_dict"], v_dict=u["v_dict"], out=outs[layer])
                       for layer, u in enumerate(ls)] for ls in sets]

    def run_step(c, s):
        """One timed step on input copy c: the decode and, at N > 1, the combine."""
        if fplan is not None:
            for v in fviews[c]:
                fplan.run_views(v, s)
            return
        run_partials(c, s)
        if mode == "p2p":
            combiner.run(pk, out.view(rows, d), stream=s)
        elif mode == "nccl":
            nccl_collective(s)

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        run_partials(0, stream)
        if partials:
            nccl_collective(stream)  # warms the communicator before capture; the reference result
    stream.synchronize()
    plan.status()
    if combiner is not None:
        # the NVLink combine (kernel or fused) must reproduce the NCCL all-gather + merge
        ref = out.clone()
        with torch.cuda.stream(stream):
            run_step(0, stream)
        stream.synchronize()
        (fplan or plan).status()
        combiner.status()
        if not torch.allclose(out.float(), ref.float(), atol=1e-3, rtol=1e-3):
            raise RuntimeError(f"NVLink combine ({mode}) differs from the NCCL all-gather + merge")
    # one CUDA graph per input copy: the step (and at N > 1 its combine)
    graphs = []
    for c in range(copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            run_step(c, torch.cuda.current_stream())
        graphs.append(g)
    kernels_per_step = layers * plan.kernel_count + (1 if mode in ("p2p", "nccl") else 0)
    # also every copy's step in one graph (on one GPU, or with an NVLink
    # combine): consecutive steps then follow each other on the device (the
    # step and combine kernels are programmatic dependent launches) instead
    # of paying a graph launch each; every rank replays the same sequence
    round_graph = None
    if copies > 1 and mode != "nccl":
        round_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(round_graph, stream=stream):
            for c in range(copies):
                run_step(c, torch.cuda.current_stream())

    def step(i):
        graphs[i % copies].replay()

    def run_steps(i, n):
        """Steps i .. i + n - 1, step j on input copy j % copies."""
        while n > 0:
            if round_graph is not None and i % copies == 0 and n >= copies:
                round_graph.replay()
                i, n = i + copies, n - copies
            else:
                graphs[i % copies].replay()
                i, n = i + 1, n - 1

    # set-up, not warm-up: replay every captured graph once so that no graph's
    # first launch (its upload to the device) falls inside the timed region,
    # whatever --warmup is; every rank replays the same sequence
    for g in graphs:
        g.replay()
    if round_graph is not None:
        round_graph.replay()
    torch.cuda.synchronize()
    run_steps(0, args.warmup)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()

    def aligned_start():
        """Queue a ~50 us device spin so the host is ahead of the GPU when
        the timed region starts, and at N > 1 a small all-reduce after it,
        so every rank's start event is recorded right after a cross-rank
        rendezvous on the device rather than at its own host time."""
        torch.cuda._sleep(100_000)
        if dist:
            dist.all_reduce(torch.ones(1, device=dev))

    sampler = ClockSampler(local_rank)
    sampler.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    aligned_start()
    ev0.record()
    run_steps(args.warmup, args.steps)
    ev1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    plan.status()
    ms_step = ms / args.steps

    # at N > 1, the step kernel alone (no collective) over the same copies,
    # so the line can say what the combine adds per step
    phases = None
    if partials:
        # same graph structure as the timed steps: one graph per copy and
        # every copy's step in one graph, replayed in the same order
        solo = []
        for c in range(copies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run_partials(c, torch.cuda.current_stream())
            solo.append(g)
        solo_round = None
        if copies > 1:
            solo_round = torch.cuda.CUDAGraph()
            with torch.cuda.graph(solo_round, stream=stream):
                for c in range(copies):
                    run_partials(c, torch.cuda.current_stream())
            solo.append(solo_round)
        for g in solo:
            g.replay()
        torch.cuda.synchronize()
        torch.cuda._sleep(100_000)
        ev0.record()
        i, n = args.warmup, args.steps
        while n > 0:
            if solo_round is not None and i % copies == 0 and n >= copies:
                solo_round.replay()
                i, n = i + copies, n - copies
            else:
                solo[i % copies].replay()
                i, n = i + 1, n - 1
        ev1.record()
        torch.cuda.synchronize()
        t = torch.tensor([ev0.elapsed_time(ev1) / args.steps], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_only = float(t.item())
        phases = {"step_us": step_only * 1e3, "combine_us": (ms_step - step_only) * 1e3,
                  "how": "step_us: the decode-step graphs alone (no collective), CUDA events, max over ranks; "
                         "combine_us: ms_per_step minus step_us"}
        for g in solo:
            g.reset()
        solo.clear()
    if context_split:
        tokens = synth.kv_tokens(w)
        t_all = torch.tensor([tokens], device=dev, dtype=torch.float64)
        dist.all_reduce(t_all)  # the whole context's KV tokens, each counted once
        tokens_total = int(t_all.item())
    else:
        tokens_total = units * tokens
    value = tokens_total / (ms_step * 1e-3)

    # end to end through the reference-shaped C call with host buffers: every
    # input copied from pinned host memory, the output copied back, each call
    # synchronous (weaver.rs:139-237)
    pinned = {k: torch.from_numpy(np.ascontiguousarray(v).view(np.uint8) if v.dtype == synth.SPARSE_CODE_DTYPE
                                  else (v.view(np.int32) if v.dtype == np.uint32 else np.ascontiguousarray(v))
                                  ).pin_memory()
              for k, v in w.items() if isinstance(v, np.ndarray)}
    hv = host_views_for(w, pinned)
    out_h = torch.empty((rows * d,), dtype=torch.float16).pin_memory()
    pm_h = torch.empty((rows,), dtype=torch.float32).pin_memory()
    pl_h = torch.empty_like(pm_h).pin_memory()
    po_h = torch.empty((rows * d,), dtype=torch.float32).pin_memory()
    if partials:
        hv.part_m, hv.part_l, hv.part_o = pm_h.data_ptr(), pl_h.data_ptr(), po_h.data_ptr()
    else:
        hv.out = out_h.data_ptr()
    hip = np.ascontiguousarray(w["hot_indptr"], np.uint32)
    cip = np.ascontiguousarray(w["cold_indptr"], np.uint32)
    lib = N.lib()

    def host_call():
        # one call per layer; a multi-layer step's calls reuse layer 0's host
        # buffers (every call still copies all of its inputs in)
        for _ in range(layers):
            N.check(lib.weaver_decode_host_batch(eng.handle, ctypes.byref(plan.shape), hip.ctypes.data,
                                                 cip.ctypes.data, ctypes.byref(hv)))

    h2d = layers * sum(int(pinned[k].numel() * pinned[k].element_size()) for k in
                       ("q", "hot_k", "hot_v", "hot_refs", "k_codes", "v_codes", "cold_refs", "k_dict", "v_dict"))
    d2h = layers * ((rows * 4 * 2 + rows * d * 4) if partials else rows * d * 2)
    for _ in range(3):
        host_call()
    k_e2e = max(5, min(args.steps, 200))
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(k_e2e):
        host_call()
    dt = time.perf_counter() - t0
    if dist:
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    e2e_value = tokens_total * k_e2e / dt

    # resident pools: only the step's query goes in and its output comes out
    q_h = pinned["q"]
    out_res = torch.empty((rows * d,), dtype=torch.float16).pin_memory()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record()
    for i in range(args.steps):
        for u in sets[i % copies]:
            u["q"].copy_(q_h.view(u["q"].shape), non_blocking=True)
        step(i)
        for o_ in outs:
            out_res.copy_(o_.view(-1), non_blocking=True)
    ev1.record()
    torch.cuda.synchronize()
    ms_res = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms_res], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_res = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        if not os.path.exists(oracle.ORACLE_SO):
            oracle.build(with_ref=False)
        threads = cpu_threads()
        n, t0 = 0, time.perf_counter()
        while n < 1 or (time.perf_counter() - t0 < 10.0 and n < 50):
            oracle.config_decode(w, precision="f32", threads=threads)
            n += 1
        tc = (time.perf_counter() - t0) / n
        cpu = {"value": synth.kv_tokens(w) / tc, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{n} full {args.config} decode steps of one layer; fp32 C oracle (restatement of "
                         f"weaver_kernel.metal), OpenMP over query rows"}

    peak, peak_kind = peaks()
    achieved = bytes_alg / (ms_step * 1e-3) / 1e9
    traffic = None
    prof = os.path.join(ROOT, "profiles", f"decode_step_{args.config}.json")
    if world == 1 and os.path.exists(prof):
        # a one-GPU capture of this configuration's step; at N > 1 the step
        # also moves partials over NVLink, which that capture does not cover
        with open(prof) as f:
            traffic = json.load(f).get("dram_bytes_per_step")
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if (head_sharded or context_split) else "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": args.config, "layers": layers, "kv_tokens_per_step_per_gpu": tokens,
                       "bytes_alg_per_step_per_gpu": bytes_alg, "l2": f"inputs rotate over {copies} copies "
                       f"({copies * bytes_alg / 1e6:.0f} MB > 126 MB L2)",
                       "parallelism": (f"kv-head sharded x{world} (no collective)" if head_sharded else
                                       (f"split-KV x{world}" + (" of one context" if context_split else "") + ", " +
                                        ({"fused": "merge over ranks fused into the step kernel (NVLink peer stores)",
                                          "p2p": "NVLink peer-memory combine kernel"}.get(mode) if combiner is not None
                                         else "NCCL all-gather + merge"))) if world > 1
                       else "single GPU",
                       "per_gpu_value": value / world,
                       "kv_heads_per_gpu": w["kv_heads"]},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel": f"one decode step ({kernels_per_step} kernels in a CUDA graph)",
                         "peak_source": peak_kind},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "api": "weaver_decode_host_batch (all inputs copied from pinned host memory every step)"},
            "e2e_resident": {"value": tokens_total / (ms_res / args.steps * 1e-3), "unit": UNIT,
                             "h2d_bytes_per_step": layers * int(w["q"].nbytes),
                             "d2h_bytes_per_step": layers * rows * d * 2},
            "gpu_launches": args.steps * kernels_per_step,
            "clocks": sampler.summary(),
        }
        if phases is not None:
            line["phases"] = phases
        print(json.dumps(line), flush=True)
    # release every graph (they hold NCCL work at N > 1) before the process
    # group goes away, or its destruction waits for them forever
    torch.cuda.synchronize()
    for gr in graphs:
        gr.reset()
    graphs.clear()
    if round_graph is not None:
        round_graph.reset()
    g = gr = round_graph = None
    torch.cuda.synchronize()
    if dist:
        dist.barrier()  # every rank past its last combine before buffers go away
    if combiner is not None:
        combiner.status()
        combiner.detach()
        combiner.close()
    if fplan is not None:
        fplan.close()
    plan.close()
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_distill(args) -> None:
    """--op distill (see the module docstring)."""
    import torch
    import oracle
    from aether_nexus_b200 import migrate, synth

    cfg = synth.config(args.config)
    Hkv, d, A = cfg["kv_heads"], cfg["head_dim"], cfg["dict_size"]
    nb = args.blocks
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    hot_k = torch.randn((nb, 16, Hkv, d), generator=gen, device=dev).half()
    hot_v = torch.randn((nb, 16, Hkv, d), generator=gen, device=dev).half()
    k_dict = (torch.randn((Hkv, A, d), generator=gen, device=dev) * cfg["dict_std"]).half()
    v_dict = (torch.randn((Hkv, A, d), generator=gen, device=dev) * cfg["dict_std"]).half()
    cold_k = torch.zeros((nb, 16, Hkv, 16), dtype=torch.uint8, device=dev)
    cold_v = torch.zeros_like(cold_k)
    src = torch.arange(nb, dtype=torch.int32, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    rows = nb * 16 * Hkv * 2
    flops = rows * 2.0 * A * d

    def step():
        migrate.migrate_blocks(hot_k, hot_v, src, src, k_dict, v_dict, cold_k, cold_v, bad)

    def timed(n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            step()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    for _ in range(args.warmup):
        step()
    sampler = ClockSampler(0)
    sampler.start()
    ms = timed(args.steps)
    sampler.stop()
    tc_k = cold_k.clone()
    os.environ["WEAVER_DISTILL_CUDA_CORES"] = "1"
    try:
        step()
        ms_cc = timed(max(1, min(3, args.steps)))
        same = bool(torch.equal(cold_k, tc_k))
    finally:
        del os.environ["WEAVER_DISTILL_CUDA_CORES"]
    if not same or int(bad.item()):
        raise RuntimeError("tensor-core and CUDA-core atom selection differ")
    # the CPU rule on a sample of one block's K rows
    n_cpu = 16 * Hkv
    rows_h = hot_k[0].reshape(-1, d).cpu().numpy()
    dic_h = k_dict.cpu().numpy()
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(with_ref=False)
    t0 = time.perf_counter()
    ref = oracle.distill_rows(rows_h, Hkv, dic_h)
    t_cpu = time.perf_counter() - t0
    if not np.array_equal(ref.view(np.uint8).reshape(-1), tc_k[0].reshape(-1).cpu().numpy()):
        raise RuntimeError("GPU atom selection differs from the CPU rule")
    pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(ROOT, "MEASURED_PEAKS.json")) else {}
    peak, kind = (float(pk["bf16_tflops"]), "measured") if "bf16_tflops" in pk else (1590.0, "fallback")
    achieved = flops / (ms * 1e-3) / 1e12
    line = {"op": "distill", "metric": "atom selection rows/s (distill_block, K and V rows of hot blocks)",
            "value": rows / (ms * 1e-3), "unit": "rows/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{args.config} blocks: {nb} blocks x 16 tokens x {Hkv} kv heads x (K, V) = "
                                   f"{rows} rows against {A} atoms of d {d}",
                       "l2": f"hot blocks {2 * hot_k.numel() * 2 / 1e6:.0f} MB > 126 MB L2"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None, "peak_source": kind,
                         "kernel": "distill_tc_kernel (2 launches per step: K and V)"},
            "cuda_core": {"ms_per_step": ms_cc, "value": rows / (ms_cc * 1e-3), "unit": "rows/s",
                          "same_codes": same},
            "cpu_baseline": {"value": n_cpu / t_cpu, "unit": "rows/s", "cores": 1, "kind": "port",
                             "sample": f"{n_cpu} K rows of one block, C oracle (one thread)"},
            "gpu_launches": 2 * args.steps, "clocks": sampler.summary()}
    print(json.dumps(line), flush=True)


def run_mha(args) -> None:
    """--op mha (see the module docstring)."""
    import torch
    import oracle
    from aether_nexus_b200 import WeaverEngine

    T, nq, Hq, Hkv, d = args.kv_len, 8, 32, 8, 128
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(0)
    copies = max(1, math.ceil(3 * L2_BYTES / (2 * T * Hkv * d * 2)))
    caches = [(torch.randn((T, Hkv, d), generator=gen, device=dev).half(),
               torch.randn((T, Hkv, d), generator=gen, device=dev).half()) for _ in range(copies)]
    q = torch.randn((nq, Hq, d), generator=gen, device=dev).half()
    out = torch.empty_like(q)
    eng = WeaverEngine(0)
    bytes_step = 2 * T * Hkv * d * 2 + 2 * nq * Hq * d * 2
    for i in range(args.warmup):
        k, v = caches[i % copies]
        eng.multihead_attention(q, k, v, out, T)
    torch.cuda.synchronize()
    # the oracle on the first 2048 positions of the first cache, every query
    k0, v0 = caches[0]
    Ts = min(T, 2048)
    ref = oracle.mha(q.cpu().numpy(), k0[:Ts].cpu().numpy(), v0[:Ts].cpu().numpy(), Ts)
    eng.multihead_attention(q, k0, v0, out, Ts)
    torch.cuda.synchronize()
    got = out.cpu().numpy().astype(np.float32)
    if not np.all(np.abs(got - ref.astype(np.float32)) <= 2e-3 + 1e-2 * np.abs(ref.astype(np.float32))):
        raise RuntimeError("multi-query attention differs from the oracle")
    t0 = time.perf_counter()
    oracle.mha(q.cpu().numpy(), k0[:Ts].cpu().numpy(), v0[:Ts].cpu().numpy(), Ts)
    t_cpu = time.perf_counter() - t0
    sampler = ClockSampler(0)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        k, v = caches[i % copies]
        eng.multihead_attention(q, k, v, out, T)
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    peak, kind = peaks()
    achieved = bytes_step / (ms * 1e-3) / 1e9
    n_chunks_launch = 2  # the split-KV kernel and the merge over chunks
    line = {"op": "mha", "metric": "multi-query attention KV positions/s (ops.metal multihead_attention)",
            "value": T / (ms * 1e-3), "unit": "KV positions/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"T={T} cache x {Hkv} kv heads x d {d}, {nq} causal queries x {Hq} heads",
                       "l2": f"caches rotate over {copies} copies ({copies * 2 * T * Hkv * d * 2 / 1e6:.0f} MB > 126 MB L2)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_source": kind, "kernel": "mha_kernel + merge over chunks"},
            "cpu_baseline": {"value": Ts / t_cpu, "unit": "KV positions/s", "cores": 1, "kind": "port",
                             "sample": f"the first {Ts} positions, C oracle of ops.metal:528-616 (one thread)"},
            "gpu_launches": n_chunks_launch * args.steps, "clocks": sampler.summary()}
    eng.close()
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c4", "c5"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--op", choices=["decode", "distill", "mha"], default="decode")
    ap.add_argument("--kv-len", type=int, default=32768, help="cache positions of --op mha")
    ap.add_argument("--layers", type=int, default=0,
                    help="decode only the first L layers of a multi-layer config (c3) per step: a small profiling case")
    ap.add_argument("--blocks", type=int, default=4096, help="hot blocks per step of --op distill")
    args = ap.parse_args()
    if args.op == "distill":
        run_distill(args)
        return
    if args.op == "mha":
        run_mha(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
