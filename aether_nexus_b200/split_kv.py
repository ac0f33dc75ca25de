"""Multi-GPU decode (one process per GPU, one node): split-KV for long
contexts, kv-head sharding for batched steps.

A long context is partitioned by KV blocks: every rank attends to a
contiguous run of each sequence's hot blocks and of its cold blocks and
produces log-sum-exp partials ``(m, l, o)`` per query row
(``WEAVER_FLAG_PARTIALS``); the partials are gathered over the process
group (NCCL over NVLink on GPUs) and merged:
``M = max_r m_r``, ``L = sum_r l_r exp(m_r - M)``,
``out = sum_r o_r exp(m_r - M) / L``.  This is the reference's own
hot/cold log-sum-exp merge (``weaver_kernel.metal:224-239``) applied one level
up, across devices instead of across the hot and cold halves.

The causal rule of multi-query decode (``ops.metal:546-555``) masks only the
newest ``nq - 1`` positions, which sit in the last hot block(s): the last rank
keeps the sequence's hot tail and applies the rule; the other ranks' blocks are
all visible.
"""
from __future__ import annotations

import numpy as np


def shard_ranges(n_blocks: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block range ``[lo, hi)`` of ``rank`` among ``world`` ranks
    (sizes differ by at most one; later ranks take the larger shares, so the
    last rank always holds the tail when there is any block)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world {world}")
    base, extra = divmod(int(n_blocks), world)
    lo = rank * base + max(0, rank - (world - extra))
    hi = lo + base + (1 if rank >= world - extra else 0)
    return lo, hi


def shard_refs(indptr, refs, rank: int, world: int):
    """The rank's block references of every sequence: ``(indptr', refs')``
    where sequence ``b`` keeps blocks ``shard_ranges(len_b, rank, world)``."""
    indptr = np.asarray(indptr, dtype=np.uint32)
    refs = np.asarray(refs, dtype=np.uint32)
    out_ptr = [0]
    parts = []
    for b in range(len(indptr) - 1):
        n = int(indptr[b + 1] - indptr[b])
        lo, hi = shard_ranges(n, rank, world)
        parts.append(refs[indptr[b] + lo:indptr[b] + hi])
        out_ptr.append(out_ptr[-1] + (hi - lo))
    new_refs = np.concatenate(parts).astype(np.uint32) if parts else np.zeros(0, np.uint32)
    return np.asarray(out_ptr, dtype=np.uint32), new_refs


def shard_workload(w: dict, rank: int, world: int) -> dict:
    """A workload dict (``synth.make_workload`` layout) restricted to the
    rank's hot and cold blocks; pools and dictionaries are shared, so only
    the page tables change.  Ranks other than the last decode without the
    causal rule."""
    v = dict(w)
    for side in ("hot", "cold"):
        v[f"{side}_indptr"], v[f"{side}_refs"] = shard_refs(w[f"{side}_indptr"], w[f"{side}_refs"], rank, world)
    if rank != world - 1:
        v["causal"] = 0
    return v


def head_range(kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    """KV heads ``[g0, g1)`` of ``rank`` when a batched step is sharded by kv
    head (``kv_heads`` must divide evenly: every rank then runs the same
    geometry)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world {world}")
    if kv_heads % world:
        raise ValueError(f"{kv_heads} kv heads do not split evenly over {world} ranks")
    per = kv_heads // world
    return rank * per, (rank + 1) * per


def shard_heads(w: dict, rank: int, world: int) -> dict:
    """The rank's kv heads (and their GQA q heads) of a workload: pools,
    codes and dictionaries keep only those heads, page tables are unchanged.
    Heads are independent in attention, so the ranks' outputs concatenated
    along the head axis are the full output and no collective is needed
    (the resident pools of a GPU hold only its own heads)."""
    g0, g1 = head_range(w["kv_heads"], rank, world)
    G = w["q_heads"] // w["kv_heads"]
    v = dict(w)
    v["kv_heads"], v["q_heads"] = g1 - g0, (g1 - g0) * G
    for k in ("hot_k", "hot_v", "k_codes", "v_codes"):
        v[k] = np.ascontiguousarray(w[k][:, :, g0:g1])
    for k in ("k_dict", "v_dict"):
        if w.get(k) is not None:
            v[k] = np.ascontiguousarray(w[k][g0:g1])
    v["q"] = np.ascontiguousarray(w["q"][:, :, g0 * G:g1 * G])
    return v


def combine_partials(m, l, o):
    """Log-sum-exp merge of gathered partials: ``m, l [P, rows]``,
    ``o [P, rows, d]`` (numpy or torch) -> ``[rows, d]`` float32 output.
    Rows whose partials are all empty (``m = -inf``) give zeros."""
    try:
        import torch
        if isinstance(m, torch.Tensor):
            M = m.max(dim=0).values
            f = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m),
                            torch.exp(m - torch.where(torch.isinf(M), torch.zeros_like(M), M)))
            L = (l * f).sum(0)
            O = (o * f[..., None]).sum(0)
            return torch.where(L[..., None] > 0, O / torch.clamp(L, min=1e-30)[..., None], torch.zeros_like(O))
    except ImportError:
        pass
    m = np.asarray(m, np.float64)
    l_ = np.asarray(l, np.float64)
    o = np.asarray(o, np.float64)
    M = m.max(0)
    Ms = np.where(np.isinf(M), 0.0, M)
    with np.errstate(invalid="ignore", over="ignore"):
        f = np.where(np.isneginf(m), 0.0, np.exp(m - Ms))
    L = (l_ * f).sum(0)
    O = (o * f[..., None]).sum(0)
    out = np.zeros_like(O)
    nz = L > 0
    out[nz] = O[nz] / L[nz][..., None]
    return out.astype(np.float32)


def gather_and_combine(pm, pl, po, group=None, stream=None):
    """Gather every rank's partials over ``group`` (``torch.distributed``)
    and merge them: ``pm, pl [rows]``, ``po [rows, d]`` float32 tensors on the
    rank's device.  On CUDA the merge is the library's ``weaver_merge_partials``
    kernel and the result is f16 ``[rows, d]``; on CPU (gloo) it is
    ``combine_partials`` in float32."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rows, d = int(po.shape[0]), int(po.shape[1])
    if pm.is_cuda:
        # one collective: every rank's [m | l | o] packed, merged in place
        from .weaver import merge_partials_packed
        packed = torch.cat([pm.reshape(-1), pl.reshape(-1), po.reshape(-1)]).float()
        gathered = torch.empty((world * packed.numel(),), dtype=torch.float32, device=pm.device)
        dist.all_gather_into_tensor(gathered, packed, group=group)
        out = torch.empty((rows, d), dtype=torch.float16, device=pm.device)
        merge_partials_packed(gathered, world, rows, d, out, stream=stream)
        return out
    gm = torch.empty((world, rows), dtype=torch.float32)
    gl = torch.empty_like(gm)
    go = torch.empty((world, rows, d), dtype=torch.float32)
    dist.all_gather(list(gm.unbind(0)), pm.contiguous(), group=group)
    dist.all_gather(list(gl.unbind(0)), pl.contiguous(), group=group)
    dist.all_gather(list(go.unbind(0)), po.contiguous(), group=group)
    return combine_partials(gm, gl, go)


class P2PCombine:
    """Split-KV combine over NVLink peer memory in one kernel per step
    (``weaver_combine_*``): this rank's packed partials are written straight
    into every rank's receive buffer, and each rank merges once all have
    arrived.  Setup exchanges CUDA IPC handles over ``group`` (any backend);
    every rank must then call :meth:`run` once per step in the same order.
    :meth:`close` only after every rank finished its last run (a barrier)."""

    def __init__(self, engine, rows: int, head_dim: int, group=None):
        import ctypes

        import torch.distributed as dist

        from . import _native as N
        self._N = N
        self.rows, self.head_dim = int(rows), int(head_dim)
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        h = ctypes.c_void_p()
        N.check(N.lib().weaver_combine_create(engine.handle, self.world, self.rank, self.rows, self.head_dim,
                                              ctypes.byref(h)))
        self._h = h
        buf = (ctypes.c_uint8 * 64)()
        N.check(N.lib().weaver_combine_ipc_handle(self._h, buf))
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(buf), group=group)
        for p, hb in enumerate(handles):
            hbuf = (ctypes.c_uint8 * 64).from_buffer_copy(hb)
            N.check(N.lib().weaver_combine_open_peer(self._h, p, hbuf))

    def run(self, packed, out, stream=None) -> None:
        """``packed`` fp32 CUDA tensor ``[rows*(d+2)]`` ([m | l | o]), ``out``
        f16 ``[rows, d]``."""
        from .weaver import _dptr, _stream_handle
        if packed.numel() < self.rows * (self.head_dim + 2):
            raise ValueError("packed partials too short")
        self._N.check(self._N.lib().weaver_combine_run(self._h, _dptr(packed), _dptr(out), _stream_handle(stream)))

    def attach(self, plan) -> None:
        """Fuse this combine into ``plan``'s decode step
        (``weaver_plan_attach_combine``): the plan (this rank's shard, created
        without partials) then writes the output merged over all ranks, in one
        kernel per step.  ``plan=None`` is not accepted; use :meth:`detach`."""
        self._N.check(self._N.lib().weaver_plan_attach_combine(plan._h, self._h))
        self._attached = plan

    def detach(self) -> None:
        plan = getattr(self, "_attached", None)
        if plan is not None and getattr(plan, "_h", None):
            self._N.check(self._N.lib().weaver_plan_attach_combine(plan._h, None))
        self._attached = None

    def status(self) -> None:
        self._N.check(self._N.lib().weaver_combine_status(self._h))

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._N.lib().weaver_combine_destroy(self._h)
            self._h = None
