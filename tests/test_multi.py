"""CPU tests of the multi-device driver's host logic (C ABI): the row
partition agrees with the Python sharding helpers, and every argument check
of ww_corr_cost_stem3d_multi answers before any CUDA call."""
import ctypes

import pytest


@pytest.fixture(scope="module")
def ww():
    import whirlwind_trt_plugins_b200 as ww
    return ww


def test_multi_split_matches_shard_partition(ww):
    from whirlwind_trt_plugins_b200.shard import split_even, halo_rows
    for H in (1, 2, 3, 7, 23, 94, 180):
        for n in range(1, min(H, 9) + 1):
            covered = []
            for k in range(n):
                r0, r1, i0, i1 = ww.multi_split(n, H, k)
                assert (r0, r1) == split_even(H, n, k)
                assert (i0, i1) == halo_rows(H, r0, r1)
                covered += list(range(r0, r1))
            assert covered == list(range(H))


def test_multi_split_rejects_bad_arguments(ww):
    L = ww.lib()
    v = [ctypes.c_int() for _ in range(4)]
    refs = [ctypes.byref(x) for x in v]
    assert L.ww_multi_split(0, 10, 0, *refs) == 2
    assert L.ww_multi_split(3, 10, 3, *refs) == 2
    assert L.ww_multi_split(4, 3, 0, *refs) == 2      # fewer rows than parts
    assert L.ww_multi_split(2, 10, 0, None, *refs[1:]) == 4


def _arrays(n, value=0x1000):
    P = ctypes.c_void_p * n
    return P(*([value] * n))


def test_multi_driver_argument_checks(ww):
    L = ww.lib()
    f = L.ww_corr_cost_stem3d_multi
    devs = (ctypes.c_int * 2)(0, 0)
    a = _arrays(2)
    shape = (1, 16, 2, 10, 8, 8, 4, 0)  # B C G H W D Cout act
    assert f(2, None, 0, a, a, a, a, a, *shape, None) == 4
    assert f(2, devs, 0, None, a, a, a, a, *shape, None) == 4
    assert f(0, devs, 0, a, a, a, a, a, *shape, None) == 2
    assert f(2, devs, 7, a, a, a, a, a, *shape, None) == 2           # unknown mode
    assert f(2, devs, 0, a, a, a, a, a, 1, 16, 3, 10, 8, 8, 4, 0, None) == 2   # G does not divide C
    assert f(2, devs, 1, a, a, a, a, a, 1, 16, 2, 1, 8, 8, 4, 0, None) == 2    # rows: H < n
    holes = (ctypes.c_void_p * 2)(0x1000, None)
    assert f(2, devs, 1, a, holes, a, a, a, *shape, None) == 4
    bad_dev = (ctypes.c_int * 2)(0, -1)
    assert f(2, bad_dev, 0, a, a, a, a, a, *shape, None) == 2
    # nothing to compute: success without touching a device
    assert f(2, devs, 0, a, a, a, a, a, 0, 16, 2, 10, 8, 8, 4, 0, None) == 0
