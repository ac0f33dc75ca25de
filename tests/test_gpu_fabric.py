"""Device-resident Fabric: .aether regions uploaded once per layer (K and
separate V views), LoomDescriptor offsets turned into a plan's page tables
(types.rs:311-328), and a decode over those views against the oracle.
Needs a B200."""
import numpy as np
import pytest

from conftest import assert_close

pytestmark = pytest.mark.gpu

HKV, D, A, HQ = 8, 128, 512, 32


@pytest.fixture(scope="module")
def engine():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device: GPU tests need a B200")
    from aether_nexus_b200 import WeaverEngine
    e = WeaverEngine.new(None, 0)
    yield e
    e.close()


def _align(x, a):
    return (x + a - 1) // a * a


def _image(rng, hot_blocks, cold_blocks):
    """An .aether-layout image: [header+weights | hot pool | cold pool | dictionary]
    at 16 KB alignment (fabric.rs:124-186 order), with the regions it fills."""
    from aether_nexus_b200.types import FabricRegions, SPARSE_CODE_DTYPE
    hot = (rng.standard_normal((hot_blocks, 16, HKV, D), dtype=np.float32)).astype(np.float16)
    cold = np.zeros((cold_blocks, 16, HKV), SPARSE_CODE_DTYPE)
    cold["indices"] = rng.integers(0, A, size=cold.shape + (4,), dtype=np.uint16)
    cold["coeffs"] = (rng.standard_normal(cold.shape + (4,), dtype=np.float32) * 0.5).astype(np.float16)
    dic = (rng.standard_normal((HKV, A, D), dtype=np.float32) / np.sqrt(D)).astype(np.float16)
    w_off, w_size = 0, 16384
    h_off = _align(w_off + w_size, 16384)
    c_off = _align(h_off + hot.nbytes, 16384)
    d_off = _align(c_off + cold.nbytes, 16384)
    total = _align(d_off + dic.nbytes, 16384)
    img = np.zeros(total, np.uint8)
    img[h_off:h_off + hot.nbytes] = hot.view(np.uint8).reshape(-1)
    img[c_off:c_off + cold.nbytes] = cold.view(np.uint8).reshape(-1)
    img[d_off:d_off + dic.nbytes] = dic.view(np.uint8).reshape(-1)
    regions = FabricRegions(w_off, w_size, h_off, hot.nbytes, c_off, cold.nbytes, d_off, dic.nbytes,
                            total, 0, total, 0, total, 0, total, 0, total)
    return img, regions, hot, cold, dic


def test_fabric_looms_decode_matches_oracle(engine, oracle_mod):
    import torch
    from aether_nexus_b200 import WeaverPlan
    from aether_nexus_b200.fabric import DeviceFabric
    from aether_nexus_b200.types import LoomDescriptor, Persona
    rng = np.random.default_rng(17)
    H, C = 24, 40
    img_k, reg_k, hot_k, cold_k, dic_k = _image(rng, H, C)
    img_v, reg_v, hot_v, cold_v, dic_v = _image(rng, H, C)
    fab = DeviceFabric(layers=2, kv_heads=HKV, head_dim=D, dict_size=A, hot_blocks=H, cold_blocks=C,
                       separate_v=True, max_block_refs=64)
    try:
        fab.upload_aether(1, img_k, reg_k)
        fab.upload_aether(1, img_v, reg_v, v=True)
        refs = np.zeros(64, np.uint32)
        refs[0:5] = rng.permutation(H)[:5]
        refs[10:17] = rng.permutation(C)[:7]
        refs[20:23] = rng.permutation(H)[:3] | (1 << 31)  # bit 31 is masked (weaver_kernel.metal:145)
        fab.upload_refs(refs)
        looms = [LoomDescriptor(Persona.PLANNER, hot_count=5, cold_count=7, hot_refs_offset=0, cold_refs_offset=10),
                 LoomDescriptor(Persona.CODER, hot_count=3, cold_count=0, hot_refs_offset=20, cold_refs_offset=30)]
        hip, cip, hot_t, cold_t = fab.page_tables(looms)
        assert hip.tolist() == [0, 5, 8] and cip.tolist() == [0, 7, 7]
        assert np.array_equal(hot_t.cpu().numpy().view(np.uint32), np.concatenate([refs[0:5], refs[20:23]]))
        assert np.array_equal(cold_t.cpu().numpy().view(np.uint32)[:7], refs[10:17])

        q = (rng.standard_normal((2, 1, HQ, D), dtype=np.float32)).astype(np.float16)
        scale = 1.0 / np.sqrt(D)
        plan = WeaverPlan(engine, num_seqs=2, num_queries=1, q_heads=HQ, kv_heads=HKV, head_dim=D, dict_size=A,
                          scale=scale, hot_indptr=hip, cold_indptr=cip)
        out = torch.full((2, 1, HQ, D), float("nan"), dtype=torch.float16, device="cuda")
        qt = torch.from_numpy(q).cuda()  # kept alive: the views hold raw pointers
        plan.run_views(plan.views(q=qt, out=out, hot_refs=hot_t, cold_refs=cold_t, **fab.layer_views(1)))
        plan.status()
        w = dict(num_seqs=2, num_queries=1, q_heads=HQ, kv_heads=HKV, head_dim=D, dict_size=A, scale=float(scale),
                 causal=0, q=q, hot_k=hot_k, hot_v=hot_v, hot_refs=hot_t.cpu().numpy().view(np.uint32)[:8],
                 hot_indptr=hip, k_codes=cold_k, v_codes=cold_v, cold_refs=cold_t.cpu().numpy().view(np.uint32)[:7],
                 cold_indptr=cip, k_dict=dic_k, v_dict=dic_v)
        assert_close(out.cpu().numpy(), oracle_mod.config_decode(w), what="fabric looms")
        # layer 0 was never uploaded: its views are distinct zeros
        l0, l1 = fab.layer(0), fab.layer(1)
        assert l0.hot_k != l1.hot_k and l1.hot_k != l1.hot_v
    finally:
        fab.close()


def test_fabric_refusals_and_shared_v(engine):
    from aether_nexus_b200._native import WeaverError
    from aether_nexus_b200.fabric import DeviceFabric
    from aether_nexus_b200.types import LoomDescriptor
    rng = np.random.default_rng(3)
    img, reg, *_ = _image(rng, 24, 40)
    fab = DeviceFabric(layers=1, kv_heads=HKV, head_dim=D, dict_size=A, hot_blocks=16, cold_blocks=40,
                       max_block_refs=8)
    try:
        v = fab.layer(0)
        assert v.hot_k == v.hot_v and v.cold_k == v.cold_v and v.k_dict == v.v_dict  # the reference's shared layout
        with pytest.raises(WeaverError):
            fab.upload_aether(0, img, reg)  # 24 hot blocks do not fit 16
        with pytest.raises(WeaverError):
            fab.upload_aether(0, img, reg, v=True)  # no separate V views
        with pytest.raises(WeaverError):
            fab.upload_refs(np.zeros(9, np.uint32))
        with pytest.raises(WeaverError):
            fab.page_tables([LoomDescriptor(hot_count=4, hot_refs_offset=6)])
    finally:
        fab.close()
