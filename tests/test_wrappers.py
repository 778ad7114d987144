"""CPU tests of the Python wrappers' argument checks: a caller-supplied
``out`` of the wrong shape, or inputs that disagree with each other, raise
ValueError before the library is called.

There is no GPU here, so the wrappers get ``meta`` tensors (shapes without
storage) and the device check is relaxed for the test; a check that let the
call through would reach the C ABI with null pointers and raise WWError
(status 4) instead of ValueError."""
import pytest


@pytest.fixture()
def ww(monkeypatch):
    import whirlwind_trt_plugins_b200 as ww

    def dev(t, name, dtype=None):
        if dtype is not None and t.dtype != dtype:
            raise TypeError(f"{name} must be {dtype}")
        return t

    monkeypatch.setattr(ww, "_dev", dev)
    return ww


def meta(*shape, dtype=None):
    import torch
    return torch.empty(shape, dtype=dtype or torch.float16, device="meta")


def test_corr_volume_rejects_wrong_out(ww):
    L, R = meta(1, 16, 4, 8), meta(1, 16, 4, 8)
    with pytest.raises(ValueError, match="out must have shape"):
        ww.corr_volume(L, R, 4, 2, out=meta(1, 2, 4, 4, 7))
    with pytest.raises(ValueError, match="out must have shape"):
        ww.corr_volume(L, R, 4, 1, out=meta(1, 2, 4, 4, 8))
    # the right shape passes the check and reaches the library (null pointers)
    with pytest.raises(ww.WWError):
        ww.corr_volume(L, R, 4, 2, out=meta(1, 2, 4, 4, 8), stream=0)


def test_fused_rejects_wrong_out(ww):
    L, R = meta(1, 16, 4, 8), meta(1, 16, 4, 8)
    w, b = meta(8, 2, 3, 3, 3), meta(8)
    with pytest.raises(ValueError, match="out must have shape"):
        ww.corr_cost_stem3d(L, R, w, b, 4, 2, out=meta(1, 8, 4, 4, 4))


def test_band_checks_inputs_and_out(ww):
    L, R = meta(1, 16, 5, 8), meta(1, 16, 5, 8)
    w, b = meta(8, 2, 3, 3, 3), meta(8)
    with pytest.raises(ValueError, match="left_band/right_band"):
        ww.corr_cost_stem3d_band(L, meta(1, 16, 4, 8), w, b, 4, 2, 10, 0, 0, 4)
    with pytest.raises(ValueError, match="num_groups"):
        ww.corr_cost_stem3d_band(L, R, meta(8, 3, 3, 3, 3), b, 4, 2, 10, 0, 0, 4)
    with pytest.raises(ValueError, match="out must have shape"):
        ww.corr_cost_stem3d_band(L, R, w, b, 4, 2, 10, 0, 0, 4, out=meta(1, 8, 4, 5, 8))


def test_other_wrappers_reject_wrong_out(ww):
    with pytest.raises(ValueError, match="out must have shape"):
        ww.cost_stem3d(meta(1, 4, 6, 3, 8), meta(8, 4, 3, 3, 3), meta(8), out=meta(1, 8, 6, 3, 7))
    ws = [meta(n) for n in (108, 4, 432, 4, 108, 1)]
    with pytest.raises(ValueError, match="out must have shape"):
        ww.cost_stem3d_ref3(meta(1, 1, 6, 3, 8), *ws, out=meta(1, 1, 6, 3, 9))
    with pytest.raises(ValueError, match="out must have shape"):
        ww.corr_cost_stem3d_ref3(meta(1, 8, 3, 8), meta(1, 8, 3, 8), *ws, max_disp=6, out=meta(1, 1, 5, 3, 8))
    with pytest.raises(ValueError, match="out must have shape"):
        ww.disparity_regression(meta(1, 6, 3, 8), out=meta(1, 1, 3, 9))
