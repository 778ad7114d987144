"""Disparity regression on CPU: the oracle against its formula and its known
answers, and the DisparityRegression plugin mirror (shapes, formats,
fields).  The reference has no such op, so the oracle is the specification
(sum_d d * softmax_d(s * cost)); there is no reference output to pin it to."""
import numpy as np
import pytest


def _formula(cost, mode):
    x = cost.astype(np.float64) * (-1.0 if mode == 1 else 1.0)
    x = x - x.max(axis=1, keepdims=True)
    e = np.exp(x)
    d = np.arange(cost.shape[1], dtype=np.float64).reshape(1, -1, 1, 1)
    return ((e * d).sum(axis=1) / e.sum(axis=1))[:, None]


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_oracle_is_the_formula(orc, mode, dtype):
    rng = np.random.default_rng(11 + mode)
    cost = (rng.standard_normal((2, 13, 5, 7)) * 3).astype(dtype)
    got = orc.disparity_regression(cost, mode)
    assert got.shape == (2, 1, 5, 7) and got.dtype == np.float32
    assert np.allclose(got, _formula(cost, mode), rtol=1e-6, atol=1e-6)
    half = orc.disparity_regression(cost, mode, out_f16=True)
    assert half.dtype == np.float16
    assert np.array_equal(half, _formula(cost, mode).astype(np.float32).astype(np.float16))


def test_known_answers(orc):
    D = 9
    flat = np.zeros((1, D, 2, 3), np.float32)
    # equal costs: the mean disparity
    assert np.allclose(orc.disparity_regression(flat, 0), (D - 1) / 2)
    # one dominant similarity: its index; one dominant (lowest) cost: its index
    peak = flat.copy()
    peak[0, 6] = 80.0
    assert np.allclose(orc.disparity_regression(peak, 0), 6.0, atol=1e-9)
    low = flat.copy()
    low[0, 2] = -80.0
    assert np.allclose(orc.disparity_regression(low, 1), 2.0, atol=1e-9)
    # soft-argmin of c is soft-argmax of -c; a 5-D [B, 1, D, H, W] cost is the same op
    rng = np.random.default_rng(5)
    c = rng.standard_normal((2, D, 3, 4)).astype(np.float32)
    assert np.array_equal(orc.disparity_regression(c, 1), orc.disparity_regression(-c, 0))
    assert np.array_equal(orc.disparity_regression(c[:, None], 0), orc.disparity_regression(c, 0))
    # D = 1: disparity 0 everywhere
    assert np.array_equal(orc.disparity_regression(c[:, :1], 0), np.zeros((2, 1, 3, 4), np.float32))


def test_shift_invariance(orc):
    rng = np.random.default_rng(6)
    c = rng.standard_normal((1, 24, 4, 5))
    a = orc.disparity_regression(c.astype(np.float32), 0)
    b = orc.disparity_regression((c + 37.0).astype(np.float32), 0)
    assert np.allclose(a, b, rtol=1e-5, atol=1e-5)


def test_oracle_rejects_bad_arguments(orc):
    with pytest.raises(ValueError):
        orc.disparity_regression(np.zeros((1, 4, 2, 2), np.float32), mode=2)
    with pytest.raises(ValueError):
        orc.disparity_regression(np.zeros((1, 0, 2, 2), np.float32), mode=0)


@pytest.fixture(scope="module")
def pl():
    from whirlwind_trt_plugins_b200 import plugins
    return plugins


def test_plugin_shapes_formats_fields(pl):
    T = pl.TensorDesc
    cr = pl.get_plugin_creator("DisparityRegression", "1")
    assert cr.get_field_names() == ["mode"]
    p = cr.create_plugin({})
    assert p.mode == 0 and p.get_fields_to_serialize() == {"mode": 0}
    q = cr.create_plugin({"mode": 1}).clone()
    assert q.mode == 1 and q.get_plugin_name() == "DisparityRegression"
    assert p.get_output_shapes([T((2, 48, 30, 40), 1)]) == [(2, 1, 30, 40)]
    assert p.get_output_shapes([T((2, 1, 48, 30, 40), 0)]) == [(2, 1, 30, 40)]
    with pytest.raises(ValueError):
        p.get_output_shapes([T((2, 3, 48, 30, 40), 1)])
    assert p.get_output_data_types([1]) == [1] and p.get_output_data_types([0]) == [0]
    half_in, half_out, float_out = T((1, 8, 4, 4), 1), T((1, 1, 4, 4), 1), T((1, 1, 4, 4), 0)
    assert p.supports_format_combination(0, [half_in, half_out], 1, 1)
    assert p.supports_format_combination(1, [half_in, half_out], 1, 1)
    assert not p.supports_format_combination(1, [half_in, float_out], 1, 1)
    assert not p.supports_format_combination(0, [T((1, 8, 4, 4), 2), half_out], 1, 1)


def test_api_rejects_host_tensors():
    import torch
    import whirlwind_trt_plugins_b200 as ww
    with pytest.raises(TypeError):
        ww.disparity_regression(torch.zeros((1, 4, 2, 2)))
