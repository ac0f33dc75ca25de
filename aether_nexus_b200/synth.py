"""Seeded synthetic workloads for the Weaver decode step (the configurations
the path is measured on; no external data exists for this path).

Distributions follow the configuration text: hot K/V and q ~ N(0, 1) f16;
SparseCode atom indices uniform in [0, A), coefficients ~ N(0, 0.5) (0.5 is
the standard deviation); K_dict / V_dict ~ N(0, 1) * dict_std.  Layouts are
the reference's: hot pool ``[blocks][16][Hkv][d]`` (fabric.rs:133-134), cold
pool ``[blocks][16][Hkv]`` SparseCode (fabric.rs:137-141), dictionaries
``[Hkv][A][d]`` (fabric.rs:144-145), with separate K and V pools / codes /
dictionaries for the model semantics.
"""
from __future__ import annotations

import math

import numpy as np

from .types import BLOCK_SIZE, SPARSE_CODE_DTYPE

CONFIGS = {
    # tiny, CPU-checkable
    "c1": dict(num_seqs=1, num_queries=1, q_heads=8, kv_heads=8, head_dim=64, dict_size=512,
               hot_tokens=256, cold_tokens=1024, dict_std=1 / 8, scale=1 / 8),
    # Llama-3-8B-shaped single layer, batch 1 (the headline)
    "c2": dict(num_seqs=1, num_queries=1, q_heads=32, kv_heads=8, head_dim=128, dict_size=4096,
               hot_tokens=4096, cold_tokens=28672, dict_std=1 / math.sqrt(128), scale=1 / math.sqrt(128)),
    # batched paged decode over 32 layers (every layer its own pools, codes and
    # dictionaries behind the same page tables; lengths jittered +-25%)
    "c3": dict(num_seqs=64, num_queries=1, q_heads=32, kv_heads=8, head_dim=128, dict_size=4096,
               hot_tokens=2048, cold_tokens=16384, dict_std=1 / math.sqrt(128), scale=1 / math.sqrt(128),
               jitter=0.25, shuffle_pages=True, layers=32),
    # speculative verify: 8 draft queries, causal among the drafts
    "c4": dict(num_seqs=16, num_queries=8, q_heads=32, kv_heads=8, head_dim=128, dict_size=4096,
               hot_tokens=4096, cold_tokens=28672, dict_std=1 / math.sqrt(128), scale=1 / math.sqrt(128),
               causal=True),
    # 70B-shaped long context
    "c5": dict(num_seqs=1, num_queries=1, q_heads=64, kv_heads=8, head_dim=128, dict_size=8192,
               hot_tokens=8192, cold_tokens=131072, dict_std=1 / math.sqrt(128), scale=1 / math.sqrt(128)),
}


def config(name: str, **overrides) -> dict:
    c = dict(CONFIGS[name])
    c.update(overrides)
    return c


def _f16(rng, shape, std=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float16)


def _codes(rng, n_blocks, kv_heads, A, coeff_std):
    c = np.empty((n_blocks, BLOCK_SIZE, kv_heads), dtype=SPARSE_CODE_DTYPE)
    c["indices"] = rng.integers(0, A, size=(n_blocks, BLOCK_SIZE, kv_heads, 4), dtype=np.uint16)
    c["coeffs"] = _f16(rng, (n_blocks, BLOCK_SIZE, kv_heads, 4), coeff_std)
    return c


def make_workload(cfg: dict | str, seed: int = 0, *, flag_refs: bool = False, **overrides) -> dict:
    """Generate one layer's decode-step inputs as numpy arrays.

    ``flag_refs`` sets bit 31 on a random half of the block references (the
    reference masks it, weaver_kernel.metal:145,174)."""
    if isinstance(cfg, str):
        cfg = config(cfg, **overrides)
    else:
        cfg = dict(cfg, **overrides)
    rng = np.random.default_rng(seed)
    B, nq = cfg["num_seqs"], cfg["num_queries"]
    Hq, Hkv, d, A = cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["dict_size"]
    jitter = cfg.get("jitter", 0.0)

    def lengths(mean):
        if jitter:
            t = mean * rng.uniform(1 - jitter, 1 + jitter, size=B)
        else:
            t = np.full(B, mean, dtype=np.float64)
        return np.maximum(np.round(t / BLOCK_SIZE).astype(np.int64), 0)

    hot_blocks = lengths(cfg["hot_tokens"])
    cold_blocks = lengths(cfg["cold_tokens"])
    if nq > 1:
        hot_blocks = np.maximum(hot_blocks, (nq + BLOCK_SIZE - 1) // BLOCK_SIZE)
    hot_indptr = np.concatenate([[0], np.cumsum(hot_blocks)]).astype(np.uint32)
    cold_indptr = np.concatenate([[0], np.cumsum(cold_blocks)]).astype(np.uint32)
    n_hot, n_cold = int(hot_indptr[-1]), int(cold_indptr[-1])
    extra = cfg.get("spare_blocks", 0)
    hot_pool_blocks, cold_pool_blocks = n_hot + extra, n_cold + extra
    if cfg.get("shuffle_pages"):
        hot_refs = rng.permutation(hot_pool_blocks)[:n_hot].astype(np.uint32)
        cold_refs = rng.permutation(cold_pool_blocks)[:n_cold].astype(np.uint32)
    else:
        hot_refs = np.arange(n_hot, dtype=np.uint32)
        cold_refs = np.arange(n_cold, dtype=np.uint32)
    if flag_refs:
        hot_refs |= (rng.integers(0, 2, n_hot, dtype=np.uint32) << np.uint32(31))
        cold_refs |= (rng.integers(0, 2, n_cold, dtype=np.uint32) << np.uint32(31))
    w = dict(
        num_seqs=B, num_queries=nq, q_heads=Hq, kv_heads=Hkv, head_dim=d, dict_size=A,
        scale=float(cfg["scale"]), causal=int(bool(cfg.get("causal", False))),
        q=_f16(rng, (B, nq, Hq, d)),
        hot_k=_f16(rng, (hot_pool_blocks, BLOCK_SIZE, Hkv, d)),
        hot_v=_f16(rng, (hot_pool_blocks, BLOCK_SIZE, Hkv, d)),
        hot_refs=hot_refs, hot_indptr=hot_indptr,
        k_codes=_codes(rng, cold_pool_blocks, Hkv, A, cfg.get("coeff_std", 0.5)),
        v_codes=_codes(rng, cold_pool_blocks, Hkv, A, cfg.get("coeff_std", 0.5)),
        cold_refs=cold_refs, cold_indptr=cold_indptr,
        k_dict=_f16(rng, (Hkv, A, d), cfg["dict_std"]),
        v_dict=_f16(rng, (Hkv, A, d), cfg["dict_std"]),
    )
    return w


def bytes_algorithmic(w: dict) -> int:
    """Compulsory bytes of one step, each counted once: hot K+V rows, K+V
    codes, K+V dictionaries, q in and o out (scratch excluded)."""
    Hkv, d, A = w["kv_heads"], w["head_dim"], w["dict_size"]
    th = int(w["hot_indptr"][-1]) * BLOCK_SIZE
    tc = int(w["cold_indptr"][-1]) * BLOCK_SIZE
    B, nq, Hq = w["num_seqs"], w["num_queries"], w["q_heads"]
    dict_bytes = 2 * Hkv * A * d * 2 if tc else 0
    return th * Hkv * d * 2 * 2 + tc * Hkv * 16 * 2 + dict_bytes + B * nq * Hq * d * 2 * 2


def kv_tokens(w: dict) -> int:
    return (int(w["hot_indptr"][-1]) + int(w["cold_indptr"][-1])) * BLOCK_SIZE


def to_device(w: dict, device="cuda"):
    """Copy a numpy workload to torch CUDA tensors (codes as raw 16-byte rows)."""
    import torch

    out = {}
    for k, v in w.items():
        if isinstance(v, np.ndarray):
            if v.dtype == SPARSE_CODE_DTYPE:
                t = torch.from_numpy(np.ascontiguousarray(v).view(np.uint8).reshape(v.shape + (16,)))
            elif v.dtype == np.uint32:
                t = torch.from_numpy(v.astype(np.int32, copy=False).view(np.int32))
            else:
                t = torch.from_numpy(np.ascontiguousarray(v))
            out[k] = t.to(device)
        else:
            out[k] = v
    return out


def make_literal_workload(*, q_heads=8, kv_heads=2, head_dim=128, dict_size=512, hot_count=3, cold_count=2,
                          seed=0, flag_refs=True, shuffle=True, qk_std=0.25):
    """Inputs of the reference's own decode call (weaver.rs:139-148) with
    random values: one hot_pool that serves as K and V, one cold code set,
    caller-supplied q_latent, loom_refs = [hot refs, cold refs]."""
    rng = np.random.default_rng(seed)
    G = q_heads // kv_heads
    hot_refs = (rng.permutation(hot_count) if shuffle else np.arange(hot_count)).astype(np.uint32)
    cold_refs = (rng.permutation(cold_count) if shuffle else np.arange(cold_count)).astype(np.uint32)
    refs = np.concatenate([hot_refs, cold_refs]).astype(np.uint32)
    if flag_refs:
        refs |= (rng.integers(0, 2, refs.size, dtype=np.uint32) << np.uint32(31))
    return dict(
        params=dict(q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim, block_size=BLOCK_SIZE, gqa_group=G,
                    hot_count=hot_count, cold_count=cold_count, dict_size=dict_size, sparsity_k=4),
        q_exact=_f16(rng, (q_heads * head_dim,), qk_std),
        q_latent=_f16(rng, (q_heads * dict_size,), 1.0),
        hot_pool=_f16(rng, (hot_count * BLOCK_SIZE * kv_heads * head_dim,), qk_std),
        cold_pool=_codes(rng, cold_count, kv_heads, dict_size, 0.5).reshape(-1),
        loom_refs=refs,
        dictionary=_f16(rng, (kv_heads * dict_size * head_dim,), qk_std),
    )


def layer_like(dw: dict, seed: int, cfg: dict | str | None = None) -> dict:
    """Another layer's inputs on the device: new q, hot K/V, K/V codes and
    dictionaries with the shapes and distributions of ``dw`` (a
    ``to_device`` workload), generated by a seeded torch generator on the
    device; the page tables are shared (every layer of a model has the same
    block table).  Used for the multi-layer configuration, whose 32 layers
    are too large to generate on the host."""
    import torch

    if isinstance(cfg, str):
        cfg = config(cfg)
    cfg = cfg or {}
    dev = dw["q"].device
    g = torch.Generator(device=dev)
    g.manual_seed(int(seed))
    A = int(dw["dict_size"])
    coeff_std = float(cfg.get("coeff_std", 0.5))
    dict_std = float(cfg.get("dict_std", 1.0 / math.sqrt(int(dw["head_dim"]))))

    def f16(shape, std=1.0):
        return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std).half()

    def codes(like):
        shp = tuple(like.shape[:-1])
        idx = torch.randint(0, A, shp + (4,), generator=g, device=dev, dtype=torch.int32).to(torch.int16)
        co = f16(shp + (4,), coeff_std).view(torch.int16)
        return torch.cat([idx, co], dim=-1).contiguous().view(torch.uint8)

    out = dict(dw)
    out["q"] = f16(tuple(dw["q"].shape))
    out["hot_k"] = f16(tuple(dw["hot_k"].shape))
    out["hot_v"] = f16(tuple(dw["hot_v"].shape))
    out["k_codes"] = codes(dw["k_codes"])
    out["v_codes"] = codes(dw["v_codes"])
    out["k_dict"] = f16(tuple(dw["k_dict"].shape), dict_std)
    out["v_dict"] = f16(tuple(dw["v_dict"].shape), dict_std)
    return out
