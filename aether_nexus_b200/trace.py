"""Phase timeline of the single-kernel decode step on one GPU.

    python -m aether_nexus_b200.trace [config] [key=value ...]

Creates a plan for the configuration's synthetic workload with per-CTA
%globaltimer stamps enabled (``WEAVER_TRACE=1`` at plan creation), runs a few
steps with the L2 flushed before each, and prints, per stamped phase, the
minimum / median / 90th percentile / maximum over CTAs in microseconds from
the earliest CTA start.  A stamp is the CTA's last occurrence of that phase.
"""
from __future__ import annotations

import os
import sys

import numpy as np

NAMES = ["START", "QLAT_DONE", "SCORE_WAIT", "SCORE_DONE", "SCATTER_WAIT", "SCATTER_DONE", "CONTRACT_WAIT",
         "CONTRACT_DONE", "MERGE_WAIT", "MERGE_DONE", "HOT_DONE", "EXIT", "QT_LANDED", "CODES_LANDED",
         "QLAT_LANDED", "HOT_MERGE", "QT_LAST_LANDED", "SCORED", "WS_READY", "HOT_WIDE", "SCATTER_LOCAL", "VCODES",
         "PASS1", "HOT_SCORED"]


def main(argv: list[str]) -> None:
    os.environ["WEAVER_TRACE"] = "1"
    import torch
    from . import WeaverEngine, WeaverPlan, synth

    cfg = argv[0] if argv else "c2"
    over = {k: (float(v) if "." in v else int(v)) for k, v in (a.split("=") for a in argv[1:])}
    w = synth.make_workload(cfg, seed=1000, **over)
    dw = synth.to_device(w)
    eng = WeaverEngine(0)
    B, nq, Hq, d = w["q"].shape
    plan = WeaverPlan(eng, num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=w["kv_heads"], head_dim=d,
                      dict_size=w["dict_size"], scale=w["scale"], hot_indptr=w["hot_indptr"],
                      cold_indptr=w["cold_indptr"], causal=bool(w["causal"]))
    if plan.kernel_count != 1:
        raise SystemExit(f"{cfg}: the plan runs {plan.kernel_count} kernels; stamps exist for the single-kernel step")
    out = torch.empty((B, nq, Hq, d), dtype=torch.float16, device="cuda")
    kw = dict(q=dw["q"], hot_k=dw["hot_k"], hot_v=dw["hot_v"], hot_refs=dw["hot_refs"], cold_k=dw["k_codes"],
              cold_v=dw["v_codes"], cold_refs=dw["cold_refs"], k_dict=dw["k_dict"], v_dict=dw["v_dict"], out=out)
    flush = torch.empty(512 * 2 ** 20, dtype=torch.uint8, device="cuda")
    for _ in range(6):
        flush.zero_()
        plan.run(**kw)
        torch.cuda.synchronize()
    plan.status()
    t = plan.trace(2048).astype(np.int64)
    t0 = t[:, 0][t[:, 0] > 0].min()
    print(f"{cfg} {over}: {t.shape[0]} CTAs traced")
    rows = []
    for s, nm in enumerate(NAMES[: t.shape[1]]):
        v = t[:, s]
        v = v[v > 0]
        if v.size == 0:
            continue
        r = (v - t0) / 1000.0
        rows.append((np.median(r), f"{nm:16s} n={v.size:4d} min {r.min():7.2f} med {np.median(r):7.2f} "
                                   f"p90 {np.percentile(r, 90):7.2f} max {r.max():7.2f} us"))
    for _, line in sorted(rows):
        print(line)
    eng.close()


if __name__ == "__main__":
    main(sys.argv[1:])
