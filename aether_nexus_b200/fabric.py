"""Device-resident Fabric (``weaver_device_fabric_*``): the Hot / Cold /
Dictionary regions of the reference's ``.aether`` file (fabric.rs:124-186,
347-420) uploaded once, with a layer dimension and optional separate V
regions, plus the block-reference array that LoomDescriptor offsets index
(types.rs:311-328).

Typical use::

    fab = DeviceFabric(layers=32, kv_heads=8, head_dim=128, dict_size=4096,
                       hot_blocks=..., cold_blocks=..., separate_v=True, max_block_refs=...)
    fab.upload_aether(layer, image_bytes, FabricRegions.compute(dims))   # K views
    fab.upload_refs(block_refs)
    hot_ip, cold_ip, hot_refs, cold_refs = fab.page_tables(looms)
    plan = WeaverPlan(engine, ..., hot_indptr=hot_ip, cold_indptr=cold_ip)
    plan.run_views(plan.views(q=q, out=out, hot_refs=hot_refs, cold_refs=cold_refs, **fab.layer_views(layer)))
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .weaver import _stream_handle


class DeviceFabric:
    def __init__(self, *, layers: int, kv_heads: int, head_dim: int, dict_size: int, hot_blocks: int,
                 cold_blocks: int, separate_v: bool = False, max_block_refs: int = 0, device: int = 0):
        g = N.FabricGeometryC(layers=layers, kv_heads=kv_heads, head_dim=head_dim, dict_size=dict_size,
                              hot_blocks=hot_blocks, cold_blocks=cold_blocks, separate_v=int(bool(separate_v)),
                              max_block_refs=max_block_refs)
        h = ctypes.c_void_p()
        N.check(N.lib().weaver_device_fabric_create(device, ctypes.byref(g), ctypes.byref(h)))
        self._h = h
        self.geometry = g

    def close(self) -> None:
        if getattr(self, "_h", None):
            N.lib().weaver_device_fabric_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def layer(self, layer: int) -> N.FabricLayerC:
        out = N.FabricLayerC()
        N.check(N.lib().weaver_device_fabric_layer(self._h, layer, ctypes.byref(out)))
        return out

    def layer_views(self, layer: int) -> dict:
        """Keyword arguments for ``WeaverPlan.views`` (raw device pointers)."""
        v = self.layer(layer)
        return dict(hot_k=v.hot_k, hot_v=v.hot_v, cold_k=v.cold_k, cold_v=v.cold_v, k_dict=v.k_dict,
                    v_dict=v.v_dict, hot_pool_blocks=int(v.hot_pool_blocks), cold_pool_blocks=int(v.cold_pool_blocks))

    def upload_aether(self, layer: int, image, regions, *, v: bool = False, stream=None) -> None:
        """Copy the Hot / Cold / Dictionary regions of an ``.aether`` image
        (bytes-like or uint8 array in host memory; ``regions`` a
        ``types.FabricRegions``) into the layer's K (or, ``v``, V) views."""
        img = np.frombuffer(image, dtype=np.uint8) if not isinstance(image, np.ndarray) else image
        img = np.ascontiguousarray(img.view(np.uint8).reshape(-1))
        rc = N.FabricRegionsC(*[int(getattr(regions, f[0])) for f in N.FabricRegionsC._fields_])
        N.check(N.lib().weaver_device_fabric_upload_aether(self._h, layer, img.ctypes.data, img.nbytes,
                                                           ctypes.byref(rc), int(bool(v)), _stream_handle(stream)))
        self._keep = img  # the copy is asynchronous on the stream

    def upload_refs(self, refs, offset: int = 0, stream=None) -> None:
        r = np.ascontiguousarray(np.asarray(refs, dtype=np.uint32))
        N.check(N.lib().weaver_device_fabric_upload_refs(self._h, r.ctypes.data, r.size, offset,
                                                         _stream_handle(stream)))
        self._keep_refs = r

    def page_tables(self, looms, stream=None):
        """LoomDescriptor list -> (hot_indptr, cold_indptr) host arrays and
        (hot_refs, cold_refs) int32 CUDA tensors for a plan."""
        import torch
        n = len(looms)
        arr = (N.LoomDescriptorC * max(1, n))()
        for i, L in enumerate(looms):
            arr[i] = L.to_c() if hasattr(L, "to_c") else L
        hot_count = sum(int(arr[i].hot_count) for i in range(n))
        cold_count = sum(int(arr[i].cold_count) for i in range(n))
        hip = np.zeros(n + 1, np.uint32)
        cip = np.zeros(n + 1, np.uint32)
        hot = torch.empty(max(1, hot_count), dtype=torch.int32, device="cuda")
        cold = torch.empty(max(1, cold_count), dtype=torch.int32, device="cuda")
        N.check(N.lib().weaver_loom_page_tables(self._h, arr, n, hip.ctypes.data, cip.ctypes.data, hot.data_ptr(),
                                                hot.numel(), cold.data_ptr(), cold.numel(), _stream_handle(stream)))
        return hip, cip, hot, cold


__all__ = ["DeviceFabric"]
