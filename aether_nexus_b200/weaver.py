"""Python mirror of the reference's Weaver host API over the CUDA library.

* ``WeaverEngine`` mirrors ``nexus-core/src/weaver.rs:27-322``: ``new`` /
  ``decode(q_exact, q_latent, hot_pool, cold_pool, loom_refs, dictionary,
  params) -> DecodeOutput`` / ``device_name`` / ``max_threads_per_threadgroup``,
  raising ``WeaverError`` where the reference returns ``Err(String)``.
* ``WeaverPlan`` is the device-resident batched path (pools stay in HBM as
  Fabric sub-views; one call launches one decode step on a CUDA stream).
* ``merge_partials`` / ``distill`` wrap the split-KV combine and the GPU atom
  selection (``nexus-core/src/distiller.rs:171-246``).

Every call goes through ``libweaver_cuda.so``; nothing here computes on the
CPU.  torch is used only to hand device pointers and streams across.
"""
from __future__ import annotations

import ctypes
import dataclasses

import numpy as np

from . import _native as N
from .types import SPARSE_CODE_DTYPE, WeaverParams


def _host_ptr(a):
    """(pointer, element count) of a contiguous numpy array or CPU torch tensor."""
    if a is None:
        return None, 0
    if hasattr(a, "data_ptr"):
        if not a.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return a.data_ptr(), a.numel()
    a = np.asarray(a)
    if not a.flags.c_contiguous:
        raise ValueError("array must be C-contiguous")
    n = a.size if a.dtype != SPARSE_CODE_DTYPE and a.dtype.itemsize != 16 else a.size
    return a.ctypes.data, n


@dataclasses.dataclass
class DecodeOutput:
    """``DecodeOutput`` (weaver.rs:59-62): the output token, q_heads*head_dim f16."""
    data: np.ndarray


class WeaverEngine:
    """``WeaverEngine`` (weaver.rs:31-56) on one CUDA device."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        N.check(N.lib().weaver_engine_create(int(device), ctypes.byref(h)))
        self._h = h
        self.device = int(device)

    @classmethod
    def new(cls, metallib_path: str | None = None, device: int = 0) -> "WeaverEngine":
        """``WeaverEngine::new`` (weaver.rs:85).  The path argument is accepted
        and ignored: the kernels are linked into the library."""
        return cls(device)

    def close(self) -> None:
        if getattr(self, "_h", None):
            N.lib().weaver_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def multihead_attention(self, q, k_cache, v_cache, out, total_kv_len: int, stream=None) -> None:
        """``Ops::multihead_attention`` (ops.rs:433-460, ops.metal:528-616) on
        CUDA tensors: ``q [nq, Hq, d]``, ``k_cache`` / ``v_cache`` ``[>= T, Hkv,
        d]``, ``out [nq, Hq, d]`` (f16).  Query i attends to positions
        ``< T - nq + 1 + i``."""
        nq, Hq, d = (int(x) for x in q.shape)
        Hkv = int(k_cache.shape[-2])
        if int(k_cache.shape[0]) < total_kv_len or int(v_cache.shape[0]) < total_kv_len:
            raise ValueError("cache shorter than total_kv_len")
        N.check(N.lib().weaver_multihead_attention(self._h, _dptr(q), _dptr(k_cache), _dptr(v_cache), _dptr(out),
                                                   int(total_kv_len), d, Hq, Hkv, nq, _stream_handle(stream)))

    def device_name(self) -> str:
        buf = ctypes.create_string_buffer(256)
        N.check(N.lib().weaver_engine_device_name(self._h, buf, 256))
        return buf.value.decode()

    def max_threads_per_threadgroup(self) -> int:
        v = ctypes.c_uint64()
        N.check(N.lib().weaver_engine_max_threads_per_block(self._h, ctypes.byref(v)))
        return v.value

    def decode(self, q_exact, q_latent, hot_pool, cold_pool, loom_refs, dictionary,
               params: WeaverParams, out=None) -> DecodeOutput:
        """``WeaverEngine::decode`` (weaver.rs:139-237).  Inputs are host arrays
        (numpy or CPU torch tensors; f16 as float16 or raw uint16 bits,
        ``cold_pool`` as 16-byte SparseCode records).  Blocks until done."""
        qp, qn = _host_ptr(q_exact)
        lp, ln = _host_ptr(q_latent)
        hp, hn = _host_ptr(hot_pool)
        cp, cn = _host_ptr(cold_pool)
        rp, rn = _host_ptr(loom_refs)
        dp, dn = _host_ptr(dictionary)
        n_out = params.q_heads * params.head_dim
        if out is None:
            out = np.empty(n_out, dtype=np.float16)
        op, on = _host_ptr(out)
        pc = params.to_c()
        N.check(N.lib().weaver_decode_host(self._h, qp, qn, lp, ln, hp, hn, cp, cn, rp, rn, dp, dn,
                                           ctypes.byref(pc), op, on))
        return DecodeOutput(out if isinstance(out, np.ndarray) else out)


def _dptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("device view must be a CUDA tensor")
    return t.data_ptr()


def _stream_handle(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class WeaverPlan:
    """A decode-step plan over device-resident pools (``weaver_plan_create``).

    ``hot_indptr`` / ``cold_indptr`` are the per-sequence block offsets into the
    concatenated block-reference arrays (the ``loom_refs`` split of
    weaver_kernel.metal:143,172, one segment per sequence)."""

    def __init__(self, engine: WeaverEngine, *, num_seqs: int, num_queries: int, q_heads: int,
                 kv_heads: int, head_dim: int, dict_size: int, scale: float, hot_indptr, cold_indptr,
                 causal: bool = False, qlatent_input: bool = False, partials: bool = False):
        self.engine = engine
        flags = (N.FLAG_CAUSAL if causal else 0) | (N.FLAG_QLATENT_INPUT if qlatent_input else 0) | \
            (N.FLAG_PARTIALS if partials else 0)
        self.shape = N.ShapeC(num_seqs, num_queries, q_heads, kv_heads, head_dim, dict_size, float(scale), flags)
        hip = np.ascontiguousarray(np.asarray(hot_indptr, dtype=np.uint32))
        cip = np.ascontiguousarray(np.asarray(cold_indptr, dtype=np.uint32))
        if hip.size != num_seqs + 1 or cip.size != num_seqs + 1:
            raise ValueError("indptr arrays need num_seqs + 1 entries")
        h = ctypes.c_void_p()
        N.check(N.lib().weaver_plan_create(engine.handle, ctypes.byref(self.shape), hip.ctypes.data,
                                           cip.ctypes.data, ctypes.byref(h)))
        self._h = h
        self.partials = partials

    def close(self) -> None:
        if getattr(self, "_h", None):
            N.lib().weaver_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def kernel_count(self) -> int:
        return N.lib().weaver_plan_kernel_count(self._h)

    def views(self, *, q, hot_k, hot_v, hot_refs, cold_k, cold_v, cold_refs, k_dict, v_dict, out=None,
              q_latent=None, part_m=None, part_l=None, part_o=None, dict_head_stride=None,
              hot_pool_blocks=None, cold_pool_blocks=None) -> N.ViewsC:
        """Build the C views struct from CUDA tensors (kept for repeated runs)."""
        v = N.ViewsC()
        v.q, v.q_latent = _dptr(q), _dptr(q_latent)
        v.hot_k, v.hot_v, v.hot_refs = _dptr(hot_k), _dptr(hot_v), _dptr(hot_refs)
        v.hot_pool_blocks = hot_pool_blocks if hot_pool_blocks is not None else int(hot_k.shape[0])
        v.cold_k, v.cold_v, v.cold_refs = _dptr(cold_k), _dptr(cold_v), _dptr(cold_refs)
        v.cold_pool_blocks = cold_pool_blocks if cold_pool_blocks is not None else int(cold_k.shape[0])
        v.k_dict, v.v_dict = _dptr(k_dict), _dptr(v_dict)
        if dict_head_stride is None:
            dict_head_stride = self.shape.dict_size * self.shape.head_dim
        v.dict_head_stride = dict_head_stride
        v.out, v.part_m, v.part_l, v.part_o = _dptr(out), _dptr(part_m), _dptr(part_l), _dptr(part_o)
        return v

    def run_views(self, views: N.ViewsC, stream=None) -> None:
        N.check(N.lib().weaver_run(self._h, ctypes.byref(views), _stream_handle(stream)))

    def run(self, stream=None, **tensors) -> None:
        """One decode step on ``stream`` (default: torch's current stream)."""
        self.run_views(self.views(**tensors), stream)

    def trace(self, n_ctas: int = 1024) -> np.ndarray:
        """Per-CTA phase timestamps (ns) of the last run; needs WEAVER_TRACE=1
        when the plan was created.  Shape [n_ctas, slots]."""
        buf = np.zeros(n_ctas * 16, dtype=np.uint64)
        slots = ctypes.c_uint32()
        N.check(N.lib().weaver_plan_trace(self._h, buf.ctypes.data, buf.size, ctypes.byref(slots)))
        t = buf[: (buf.size // slots.value) * slots.value].reshape(-1, slots.value)
        return t[: int((t[:, 0] > 0).sum())] if (t[:, 0] > 0).any() else t[:0]

    def status(self) -> None:
        """Synchronise and raise ``WeaverError`` if a kernel flagged a bad
        block reference / atom index or a timed-out wait."""
        N.check(N.lib().weaver_plan_status(self._h))


def merge_partials(m, l, o, out, stream=None) -> None:
    """Log-sum-exp merge of ``P`` partial results: ``m, l [P, rows]``,
    ``o [P, rows, d]`` fp32 CUDA tensors into ``out [rows, d]`` f16."""
    P, rows = int(m.shape[0]), int(m.shape[1])
    d = int(o.shape[-1])
    N.check(N.lib().weaver_merge_partials(P, rows, d, _dptr(m), _dptr(l), _dptr(o), _dptr(out),
                                          _stream_handle(stream)))


def merge_partials_packed(gathered, n_parts: int, rows: int, head_dim: int, out, stream=None) -> None:
    """Log-sum-exp merge of ``n_parts`` packed partials: ``gathered`` is a
    fp32 CUDA tensor of ``n_parts`` blocks ``[m rows | l rows | o rows*d]``
    (what one all-gather of every rank's packed buffer yields); ``out
    [rows, d]`` f16."""
    stride = rows * (head_dim + 2)
    if gathered.numel() < n_parts * stride:
        raise ValueError("gathered buffer shorter than n_parts packed partials")
    base = _dptr(gathered)
    N.check(N.lib().weaver_merge_partials_strided(n_parts, rows, head_dim, base, base + rows * 4,
                                                  base + 2 * rows * 4, stride, _dptr(out), _stream_handle(stream)))


def distill(rows, kv_heads: int, dictionary, out_codes, *, dict_head_stride=None, stream=None) -> None:
    """GPU atom selection (distiller.rs:185-234): ``rows [n, d]`` f16,
    ``dictionary [Hkv, A, d]`` f16, ``out_codes`` n x 16-byte CUDA buffer."""
    n, d = int(rows.shape[0]), int(rows.shape[1])
    A = int(dictionary.shape[-2])
    if dict_head_stride is None:
        dict_head_stride = A * d
    N.check(N.lib().weaver_distill(_dptr(rows), n, int(kv_heads), d, _dptr(dictionary), A, dict_head_stride,
                                   _dptr(out_codes), _stream_handle(stream)))


def distill_stats(rows, kv_heads: int, dictionary, out_codes, diag, *, dict_head_stride=None, stream=None) -> None:
    """``distill`` on the tensor-core path with its diagnostics in ``diag``
    (4 int32 CUDA words, zeroed by the caller): the largest |approximate -
    exact| / bound over re-scored atoms (float bits), the rows finished by the
    exact full scan, status and first expired wait."""
    n, d = int(rows.shape[0]), int(rows.shape[1])
    A = int(dictionary.shape[-2])
    if dict_head_stride is None:
        dict_head_stride = A * d
    N.check(N.lib().weaver_distill_stats(_dptr(rows), n, int(kv_heads), d, _dptr(dictionary), A, dict_head_stride,
                                         _dptr(out_codes), _dptr(diag), _stream_handle(stream)))


def hot_decode_noalloc(q, hot_k, hot_v, hot_refs, out, bad_ref_flag, *, scale: float, n_blocks=None,
                       stream=None) -> None:
    """Allocation-free exact attention of one decode step over the hot pool
    (``weaver_hot_decode_noalloc``): for callers that may not allocate device
    memory once running, so cannot create a plan.  ``q [Hq, d]``, ``hot_k`` /
    ``hot_v [blocks, 16, Hkv, d]`` f16, ``hot_refs`` int32/uint32 block refs,
    ``out [Hq, d]`` f16, ``bad_ref_flag`` one int32 the call ORs 1 into on an
    out-of-range ref.  Calls sharing a device must not overlap on the GPU."""
    Hq, d = int(q.shape[-2]), int(q.shape[-1])
    Hkv = int(hot_k.shape[2])
    n = int(hot_refs.shape[0]) if n_blocks is None else int(n_blocks)
    if n > int(hot_refs.numel()):
        raise ValueError(f"n_blocks {n} exceeds the {int(hot_refs.numel())} block references supplied")
    N.check(N.lib().weaver_hot_decode_noalloc(Hq, Hkv, d, float(scale), _dptr(q), _dptr(hot_k), _dptr(hot_v),
                                              int(hot_k.shape[0]), _dptr(hot_refs), n, _dptr(out),
                                              _dptr(bad_ref_flag), _stream_handle(stream)))
