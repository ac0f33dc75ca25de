"""Hot -> cold migration on the GPU: the reference's Distiller REM cycle
(``nexus-core/src/distiller.rs:52-246``) as device work next to the decode.

The reference evaluates a variance proxy of every hot block's f16 values
(``evaluate_entropy`` / ``compute_block_entropy``, distiller.rs:97-159),
distills the blocks whose proxy lies in ``(0, threshold)`` into SparseCodes
(``distill_block``, distiller.rs:171-246: per (token, kv head) the top 4
dictionary atoms by dot product, coefficient = f16(dot)) and writes them into
the cold pool.  Here:

* :func:`block_entropy` runs the proxy for every hot-pool block in one kernel
  (``weaver_block_entropy``);
* :func:`migrate_blocks` encodes a list of hot blocks into chosen cold blocks
  (``weaver_migrate_blocks``: K rows against K_dict into the K codes, V rows
  against V_dict into the V codes), asynchronously on any stream, e.g. a side
  stream beside the decode steps;
* :func:`migrate_low_entropy` is the cycle for one batch of sequences: it
  picks the candidates among the blocks the hot page tables reference, keeps
  each sequence's newest ``keep_recent`` hot blocks hot (the causal tail of a
  multi-query step lives there), takes destination blocks from the caller's
  free list, launches the migration and returns the new page tables (the
  moved blocks leave the hot table and join the end of the cold table of
  their sequence; attention over a block set does not depend on its order).
  The caller then creates a plan for the new block counts.

Everything device-side goes through ``libweaver_cuda.so``; the candidate
choice and the page-table bookkeeping are host logic, as in the reference
(where the Fabric's page metadata lives on the host).
"""
from __future__ import annotations

import dataclasses

import numpy as np

from . import _native as N
from .types import BLOCK_SIZE
from .weaver import _dptr, _stream_handle

DEFAULT_THRESHOLD = 0.15  # MemoryConfig::distill_entropy_threshold default (types.rs:45-53)


def block_entropy(hot_pool, kv_heads: int, stream=None):
    """Variance proxy of every block of ``hot_pool`` ([blocks, 16, Hkv, d] f16
    CUDA tensor) as a float32 CUDA tensor ``[blocks]``."""
    import torch
    n, _, hkv, d = (int(x) for x in hot_pool.shape)
    if hkv != kv_heads:
        raise ValueError("hot_pool's kv-head dimension differs from kv_heads")
    out = torch.empty(n, dtype=torch.float32, device=hot_pool.device)
    N.check(N.lib().weaver_block_entropy(_dptr(hot_pool), n, kv_heads, d, _dptr(out), _stream_handle(stream)))
    return out


def migrate_blocks(hot_k, hot_v, src_blocks, dst_blocks, k_dict, v_dict, cold_k, cold_v, bad_flag, *,
                   dict_head_stride=None, stream=None) -> None:
    """Encode hot blocks ``src_blocks[i]`` into cold blocks ``dst_blocks[i]``
    (int32/uint32 CUDA tensors of equal length): K rows against ``k_dict``
    into ``cold_k``, V rows against ``v_dict`` into ``cold_v`` (16-byte code
    records, [blocks, 16, Hkv, 16] uint8).  ``bad_flag`` (one int32) gets 1
    OR-ed in for an out-of-range entry."""
    n = int(src_blocks.numel())
    if int(dst_blocks.numel()) != n:
        raise ValueError("src_blocks and dst_blocks differ in length")
    nb, _, hkv, d = (int(x) for x in hot_k.shape)
    A = int(k_dict.shape[-2])
    if dict_head_stride is None:
        dict_head_stride = A * d
    N.check(N.lib().weaver_migrate_blocks(_dptr(hot_k), _dptr(hot_v), nb, _dptr(src_blocks), _dptr(dst_blocks), n,
                                          hkv, d, _dptr(k_dict), _dptr(v_dict), A, dict_head_stride, _dptr(cold_k),
                                          _dptr(cold_v), int(cold_k.shape[0]), _dptr(bad_flag),
                                          _stream_handle(stream)))


@dataclasses.dataclass
class Migration:
    """What one cycle moved and the page tables after it (host arrays)."""
    src_blocks: np.ndarray   # hot-pool blocks that were encoded
    dst_blocks: np.ndarray   # cold-pool blocks that received their codes
    hot_refs: np.ndarray
    hot_indptr: np.ndarray
    cold_refs: np.ndarray
    cold_indptr: np.ndarray


def choose_candidates(entropy: np.ndarray, hot_refs: np.ndarray, hot_indptr: np.ndarray, threshold: float,
                      keep_recent: int = 1) -> list[list[int]]:
    """Per sequence, the positions in its hot page table whose block's proxy
    is in ``(0, threshold)`` (distiller.rs:115-121), leaving its newest
    ``keep_recent`` blocks out.  Block references carry a flag in bit 31
    that is ignored (weaver_kernel.metal:145)."""
    out = []
    refs = np.asarray(hot_refs, np.uint32) & np.uint32(0x7FFFFFFF)
    for b in range(len(hot_indptr) - 1):
        h0, h1 = int(hot_indptr[b]), int(hot_indptr[b + 1])
        pos = []
        for p in range(h0, max(h0, h1 - keep_recent)):
            blk = int(refs[p])
            if blk < len(entropy):
                e = float(entropy[blk])
                if 0.0 < e < threshold:
                    pos.append(p)
        out.append(pos)
    return out


def rewrite_page_tables(hot_refs, hot_indptr, cold_refs, cold_indptr, moved: list[list[int]],
                        dst_blocks: list[int]) -> tuple[np.ndarray, np.ndarray, np.ndarray, np.ndarray]:
    """Page tables after moving hot positions ``moved[b]`` of every sequence
    b to the end of its cold table, as cold blocks ``dst_blocks`` (in the order
    of ``moved`` flattened)."""
    hot_refs = np.asarray(hot_refs, np.uint32)
    cold_refs = np.asarray(cold_refs, np.uint32)
    nh, nc, hip, cip = [], [], [0], [0]
    k = 0
    for b in range(len(hot_indptr) - 1):
        h0, h1 = int(hot_indptr[b]), int(hot_indptr[b + 1])
        c0, c1 = int(cold_indptr[b]), int(cold_indptr[b + 1])
        mv = set(moved[b])
        keep = [int(hot_refs[p]) for p in range(h0, h1) if p not in mv]
        add = []
        for _ in moved[b]:
            add.append(int(dst_blocks[k]))
            k += 1
        nh.extend(keep)
        nc.extend([int(x) for x in cold_refs[c0:c1]] + add)
        hip.append(len(nh))
        cip.append(len(nc))
    return (np.asarray(nh, np.uint32), np.asarray(hip, np.uint32), np.asarray(nc, np.uint32),
            np.asarray(cip, np.uint32))


def migrate_low_entropy(*, hot_k, hot_v, hot_refs, hot_indptr, cold_refs, cold_indptr, free_cold_blocks, k_dict,
                        v_dict, cold_k, cold_v, threshold: float = DEFAULT_THRESHOLD, keep_recent: int = 1,
                        dict_head_stride=None, stream=None) -> Migration:
    """One REM cycle for a batch of sequences (see the module docstring).
    ``hot_refs``/``cold_refs``/``*_indptr`` are host arrays (the page tables),
    ``free_cold_blocks`` a host list of unused cold-pool blocks; the pools and
    dictionaries are CUDA tensors.  The entropy read-back synchronises
    ``stream``; the migration itself is left running on it."""
    import torch
    ent = block_entropy(hot_k, int(hot_k.shape[2]), stream=stream)
    (torch.cuda.current_stream() if stream is None else stream).synchronize()
    moved = choose_candidates(ent.cpu().numpy(), hot_refs, hot_indptr, threshold, keep_recent)
    flat = [p for seq in moved for p in seq]
    if len(flat) > len(free_cold_blocks):
        raise ValueError(f"{len(flat)} blocks to migrate but {len(free_cold_blocks)} free cold blocks")
    src = (np.asarray(hot_refs, np.uint32)[flat] & np.uint32(0x7FFFFFFF)).astype(np.int32) if flat else \
        np.zeros(0, np.int32)
    dst = np.asarray(list(free_cold_blocks)[:len(flat)], np.int32)
    if flat:
        dev = hot_k.device
        bad = torch.zeros(1, dtype=torch.int32, device=dev)
        s_t = torch.from_numpy(src).to(dev)
        d_t = torch.from_numpy(dst).to(dev)
        migrate_blocks(hot_k, hot_v, s_t, d_t, k_dict, v_dict, cold_k, cold_v, bad,
                       dict_head_stride=dict_head_stride, stream=stream)
    nh, hip, nc, cip = rewrite_page_tables(hot_refs, hot_indptr, cold_refs, cold_indptr, moved, dst.tolist())
    return Migration(src.astype(np.uint32), dst.astype(np.uint32), nh, hip, nc, cip)


__all__ = ["DEFAULT_THRESHOLD", "BLOCK_SIZE", "Migration", "block_entropy", "choose_candidates", "migrate_blocks",
           "migrate_low_entropy", "rewrite_page_tables"]
