"""The domain-classified pool (l2d_pool_*), the counterpart of the reference's cudaMallocSided /
cudaFreeSided / cudaGetSidedPoolBase (utility/sidedgpu.cu:791-882).

* an allocation returns ceil(bytes / 4096) distinct free granules, every one classified on the
  requested side; the two sides never share a granule;
* the classification agrees with an independent address probe of the same chunk (mask and per-page
  attr through l2d_probe_addr_domains, then the reference's predictor per granule);
* granules are writable device memory at base + g * 4096;
* freeing returns them; a double free and a bad side are refused with L2D_ERR_INVALID.
"""
import ctypes as C

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import l2domain_b200 as L  # noqa: E402

GRAN = 4096


def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def test_sided_allocations_are_classified_and_disjoint():
    need_gpu()
    torch.cuda.set_device(0)
    g0 = L.malloc_sided(8 << 20, 0)
    g1 = L.malloc_sided(3 * GRAN + 1, 1)
    assert len(g0) == 2048 and len(g1) == 4
    assert len(set(g0)) == len(g0) and not set(g0) & set(g1)
    assert L.pool_sides(g0) == [0] * len(g0)
    assert L.pool_sides(g1) == [1] * len(g1)
    info = L.pool_info()
    assert info["mapped_bytes"] >= 1 << 30
    assert info["mask"] != 0 and info["mask"] & (GRAN - 1) == 0

    # Independent probe of the first 1 GiB chunk, then the predictor per granule.
    base = L.get_sided_pool_base()
    sm = L.get_map_smid2side(0)
    mask, attr = L.get_map_memory_attr(base, 1 << 30, sm, 0)
    assert mask == info["mask"]
    for g in g0[:256] + g1:
        if g * GRAN >= 1 << 30:
            continue
        addr = base + g * GRAN
        side = L.predict_addr_side(base, mask, attr, addr)
        assert side == L.pool_sides([g])[0], f"granule {g}"

    # The granules are device memory at base + g * 4096.
    lib = L.lib()
    for k, g in enumerate(g0[:4] + g1):
        L.device_view(base + g * GRAN, GRAN).fill_(k + 1)
    torch.cuda.synchronize()
    for k, g in enumerate(g0[:4] + g1):
        assert int(L.device_view(base + g * GRAN, GRAN).min()) == k + 1
    L.free_sided(g0)
    L.free_sided(g1)
    info2 = L.pool_info()
    assert info2["free_granules"][0] >= info["free_granules"][0] + len(g0)
    with pytest.raises(L.L2DError):
        L.free_sided(g1)
    assert lib.l2d_pool_alloc(0, GRAN, 2, None, (C.c_uint64 * 1)(), 1, C.byref(C.c_size_t())) == -1


def test_pool_reuses_freed_granules_then_releases():
    need_gpu()
    a = L.malloc_sided(1 << 20, 0)
    L.free_sided(a)
    b = L.malloc_sided(1 << 20, 0)
    assert sorted(a) == sorted(b)  # first-fit over the same free granules
    L.free_sided(b)
    L.pool_release()
    assert L.pool_info()["mapped_bytes"] == 0
