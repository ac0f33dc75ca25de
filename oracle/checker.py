"""CPU checkers for the Weaver decode attention — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, and only as the checker: the product library
(``aether_nexus_b200``) never imports, loads or calls anything here.

Two libraries are wrapped:

* ``oracle/build/liboracle.so`` — the C restatement (``weaver_oracle.c``) of
  ``nexus-core/src/weaver_kernel.metal:118-240`` (literal and configuration
  mode), of the atom selection in ``nexus-core/src/distiller.rs:185-234`` and of
  the entropy proxy in ``nexus-core/src/distiller.rs:126-159`` and of the full
  loop's ``multihead_attention`` (``nexus-core/src/ops.metal:528-616``);
* ``oracle/_ref/libweaver_ref.so`` and ``oracle/_ref/libops_ref.so`` — the
  reference's own ``weaver_kernel.metal`` and ``ops.metal`` compiled unmodified
  as host C++ (``oracle/Makefile`` target ``ref``).  They exist only where the
  reference source was present when they were built.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(_HERE, "build", "liboracle.so")
REF_SO = os.path.join(_HERE, "_ref", "libweaver_ref.so")
REF_OPS_SO = os.path.join(_HERE, "_ref", "libops_ref.so")

SPARSE_CODE_DTYPE = np.dtype([("indices", "<u2", (4,)), ("coeffs", "<u2", (4,))])
assert SPARSE_CODE_DTYPE.itemsize == 16


def build(with_ref: bool | None = None) -> None:
    """Compile the checkers with ``make`` (the reference one only if present)."""
    targets = ["oracle"]
    ref_root = os.environ.get("WEAVER_REFERENCE_ROOT", "/root/reference")
    if with_ref is None:
        with_ref = os.path.exists(os.path.join(ref_root, "nexus-core", "src", "weaver_kernel.metal"))
    if with_ref:
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", _HERE, f"REF={ref_root}", *targets], check=True)


class _Params(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "q_heads", "kv_heads", "head_dim", "block_size", "gqa_group",
        "hot_count", "cold_count", "dict_size", "sparsity_k")] + [("pad", ctypes.c_uint32 * 3)]


class _Desc(ctypes.Structure):
    _fields_ = [
        ("num_seqs", ctypes.c_uint32), ("num_queries", ctypes.c_uint32),
        ("q_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32), ("dict_size", ctypes.c_uint32),
        ("scale", ctypes.c_float), ("causal", ctypes.c_uint32),
        ("q", ctypes.c_void_p), ("q_latent", ctypes.c_void_p),
        ("hot_k", ctypes.c_void_p), ("hot_v", ctypes.c_void_p),
        ("hot_pool_blocks", ctypes.c_uint64),
        ("hot_refs", ctypes.c_void_p), ("hot_indptr", ctypes.c_void_p),
        ("k_codes", ctypes.c_void_p), ("v_codes", ctypes.c_void_p),
        ("cold_pool_blocks", ctypes.c_uint64),
        ("cold_refs", ctypes.c_void_p), ("cold_indptr", ctypes.c_void_p),
        ("k_dict", ctypes.c_void_p), ("v_dict", ctypes.c_void_p),
        ("dict_head_stride", ctypes.c_uint64),
        ("out", ctypes.c_void_p), ("out_m", ctypes.c_void_p),
        ("out_l", ctypes.c_void_p), ("out_o", ctypes.c_void_p),
    ]


_lib = None
_ref = None
_ref_ops = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build(with_ref=False)
        _lib = ctypes.CDLL(ORACLE_SO)
        _lib.oracle_h2f.restype = ctypes.c_float
        _lib.oracle_h2f.argtypes = [ctypes.c_uint16]
        _lib.oracle_f2h.restype = ctypes.c_uint16
        _lib.oracle_f2h.argtypes = [ctypes.c_float]
        _lib.oracle_block_entropy.restype = ctypes.c_float
        _lib.oracle_block_entropy.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        _lib.oracle_config_decode_f32.argtypes = [ctypes.c_void_p, ctypes.c_int]
        _lib.oracle_config_decode_f64.argtypes = [ctypes.c_void_p]
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        _ref = ctypes.CDLL(REF_SO)
    return _ref


def _ptr(a):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _u16(a):
    return np.ascontiguousarray(np.asarray(a).view(np.uint16) if np.asarray(a).dtype == np.float16
                                else np.asarray(a, dtype=np.uint16))


def make_params(**kw) -> _Params:
    p = _Params()
    for k, v in kw.items():
        setattr(p, k, int(v))
    return p


def literal_decode(q_exact, q_latent, hot_pool, cold_pool, loom_refs, dictionary, params: dict,
                   *, use_reference_kernel: bool = False) -> np.ndarray:
    """One decode step with the reference's literal semantics.

    Arrays are numpy float16 (or raw uint16 bits) / SparseCode records /
    uint32, shaped as in ``weaver.rs:139-148``.  Returns ``[q_heads*head_dim]``
    float16.  ``use_reference_kernel`` runs the reference source itself.
    """
    p = make_params(**params)
    q_exact, q_latent, hot_pool, dictionary = map(_u16, (q_exact, q_latent, hot_pool, dictionary))
    cold_pool = np.ascontiguousarray(cold_pool).view(np.uint8)
    loom_refs = np.ascontiguousarray(loom_refs, dtype=np.uint32)
    out = np.zeros(p.q_heads * p.head_dim, dtype=np.uint16)
    if use_reference_kernel:
        rc = ref_lib().ref_weaver_decode(
            _ptr(q_exact), _ptr(q_latent), _ptr(hot_pool), _ptr(cold_pool), _ptr(loom_refs),
            _ptr(dictionary), ctypes.byref(p), _ptr(out))
    else:
        hot_blocks = hot_pool.size // (16 * p.kv_heads * p.head_dim)
        cold_blocks = cold_pool.size // (16 * p.kv_heads)
        rc = lib().oracle_literal_decode(
            _ptr(q_exact), _ptr(q_latent), _ptr(hot_pool), ctypes.c_uint64(hot_blocks),
            _ptr(cold_pool), ctypes.c_uint64(cold_blocks), _ptr(loom_refs), _ptr(dictionary),
            ctypes.byref(p), _ptr(out))
    if rc != 0:
        raise ValueError(f"oracle literal decode failed: {rc}")
    return out.view(np.float16)


def config_decode(w, *, precision: str = "f64", threads: int = 0, partials: bool = False):
    """Configuration-mode decode of a workload dict (see
    ``aether_nexus_b200.synth``).  Returns the f16 output ``[B, nq, Hq, d]``,
    plus ``(m, l, o)`` fp32 partials when ``partials``."""
    B, nq, Hq, d = w["q"].shape
    keep = {}

    def arr(name, dtype=None):
        a = w.get(name)
        if a is None:
            return None
        a = np.ascontiguousarray(a.view(np.uint16) if a.dtype == np.float16 else a)
        keep[name] = a
        return a

    D = _Desc()
    D.num_seqs, D.num_queries, D.q_heads = B, nq, Hq
    D.kv_heads, D.head_dim, D.dict_size = w["kv_heads"], d, w["dict_size"]
    D.scale = float(w["scale"])
    D.causal = int(w.get("causal", 0))
    for name in ("q", "q_latent", "hot_k", "hot_v", "hot_refs", "hot_indptr", "k_codes",
                 "v_codes", "cold_refs", "cold_indptr", "k_dict", "v_dict"):
        a = arr(name)
        setattr(D, name, None if a is None else a.ctypes.data)
    D.hot_pool_blocks = w["hot_k"].shape[0]
    D.cold_pool_blocks = w["k_codes"].shape[0]
    D.dict_head_stride = int(w.get("dict_head_stride", w["dict_size"] * d))
    out = np.zeros((B, nq, Hq, d), dtype=np.uint16)
    D.out = out.ctypes.data
    if partials:
        m = np.zeros((B, nq, Hq), np.float32)
        l_ = np.zeros((B, nq, Hq), np.float32)
        o = np.zeros((B, nq, Hq, d), np.float32)
        D.out_m, D.out_l, D.out_o = m.ctypes.data, l_.ctypes.data, o.ctypes.data
    if precision == "f64":
        rc = lib().oracle_config_decode_f64(ctypes.byref(D))
    else:
        rc = lib().oracle_config_decode_f32(ctypes.byref(D), int(threads))
    if rc != 0:
        raise ValueError(f"oracle config decode failed: {rc}")
    out = out.view(np.float16)
    return (out, m, l_, o) if partials else out


def distill_rows(rows, kv_heads: int, dictionary, *, dict_head_stride: int | None = None):
    """Atom selection of ``distiller.rs:185-234`` for ``rows [n, d]``; row i
    belongs to kv head ``i % kv_heads``.  Returns SparseCode records."""
    rows = _u16(rows)
    n, d = rows.shape
    dictionary = _u16(dictionary)
    A = dictionary.shape[-2]
    if dict_head_stride is None:
        dict_head_stride = A * d
    out = np.zeros(n, dtype=SPARSE_CODE_DTYPE)
    rc = lib().oracle_distill_rows(_ptr(rows), ctypes.c_uint32(n), ctypes.c_uint32(kv_heads),
                                   ctypes.c_uint32(d), _ptr(dictionary), ctypes.c_uint32(A),
                                   ctypes.c_uint64(dict_head_stride), _ptr(out))
    if rc != 0:
        raise ValueError(f"oracle distill failed: {rc}")
    return out


def block_entropy(values) -> float:
    v = _u16(values).ravel()
    return float(lib().oracle_block_entropy(_ptr(v), ctypes.c_uint64(v.size)))


def h2f(bits: int) -> float:
    return float(lib().oracle_h2f(bits))


def f2h(x: float) -> int:
    return int(lib().oracle_f2h(x))


def mha(q, k_cache, v_cache, total_kv_len: int, *, reference_kernel: bool = False):
    """ops.metal:528-616 for q [nq][Hq][d] and caches [>= total_kv_len][Hkv][d]
    (f16): the C restatement, or the reference kernel itself when
    ``reference_kernel``.  Returns f16 [nq][Hq][d]."""
    global _ref_ops
    q, kc, vc = _u16(q), _u16(k_cache), _u16(v_cache)
    nq, Hq, d = q.shape
    Hkv = kc.shape[-2]
    out = np.zeros((nq, Hq, d), np.uint16)
    args = (_ptr(q), _ptr(kc), _ptr(vc), _ptr(out), ctypes.c_uint32(total_kv_len), ctypes.c_uint32(d),
            ctypes.c_uint32(Hq), ctypes.c_uint32(Hkv), ctypes.c_uint32(nq))
    if reference_kernel:
        if _ref_ops is None:
            _ref_ops = ctypes.CDLL(REF_OPS_SO)
        rc = _ref_ops.ref_multihead_attention(*args)
    else:
        rc = lib().oracle_mha(*args)
    if rc != 0:
        raise ValueError(f"multi-head attention checker failed: {rc}")
    return out.view(np.float16)


def ref_ops_available() -> bool:
    return os.path.exists(REF_OPS_SO)
