"""ww_disparity_regression on the GPU against the CPU oracle (the op's
specification; the reference has no such op) and against a plain torch fp32
softmax at the bench's full size.

Tolerance (fp32 arithmetic with ex2.approx exponentials): an fp32 output is
within 1e-5 * max(|disp|, 1) of the oracle's exact value; an fp16 output is
within one fp16 ulp of it plus that bound (the fp16 rounding of a value
within the bound)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def env():
    import torch
    import whirlwind_trt_plugins_b200 as ww
    return torch, ww


def _cost(shape, scale, seed, dtype):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape) * scale).astype(dtype)


def _ulp16(x):
    x = np.abs(x).astype(np.float16)
    return (np.nextafter(x, np.float16(np.inf)) - x).astype(np.float64)


# (B, D, H, W): vector path (W % 4 == 0), ragged W (one pixel per thread),
# D not a multiple of the chunk of 8, D = 1, wide D
SHAPES = [(2, 48, 30, 40), (1, 24, 7, 37), (3, 7, 5, 12), (1, 1, 4, 8), (1, 192, 6, 20), (2, 64, 33, 161)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("in_t,out_t", [("f16", "f16"), ("f16", "f32"), ("f32", "f32"), ("f32", "f16")])
def test_matches_oracle(env, shape, mode, in_t, out_t):
    torch, ww = env
    import oracle
    np_in = np.float16 if in_t == "f16" else np.float32
    cost = _cost(shape, 3.0, hash((shape, mode)) % 1000, np_in)
    x = torch.from_numpy(cost).cuda()
    dt = torch.float16 if out_t == "f16" else torch.float32
    got = ww.disparity_regression(x, mode, dtype=dt)
    torch.cuda.synchronize()
    assert got.shape == (shape[0], 1, shape[2], shape[3]) and got.dtype == dt
    ref = oracle.disparity_regression(cost, mode).astype(np.float64)
    g = got.cpu().numpy().astype(np.float64)
    bound = RTOL * np.maximum(np.abs(ref), 1.0)
    if out_t == "f16":
        bound = bound + _ulp16(ref)
    assert np.all(np.abs(g - ref) <= bound), float(np.max(np.abs(g - ref) - bound))


@pytest.mark.parametrize("scale", [0.01, 30.0, 1000.0])
def test_value_ranges_fp32(env, scale):
    """Nearly flat, peaked and extreme fp32 costs."""
    torch, ww = env
    import oracle
    cost = _cost((2, 40, 9, 24), scale, 21, np.float32)
    got = ww.disparity_regression(torch.from_numpy(cost).cuda(), 1).cpu().numpy().astype(np.float64)
    ref = oracle.disparity_regression(cost, 1).astype(np.float64)
    assert np.all(np.abs(got - ref) <= RTOL * np.maximum(np.abs(ref), 1.0))


def test_five_d_input_and_plugin_enqueue(env):
    torch, ww = env
    from whirlwind_trt_plugins_b200 import plugins
    cost = torch.from_numpy(_cost((2, 1, 32, 12, 16), 2.0, 3, np.float16)).cuda()
    a = ww.disparity_regression(cost, ww.DISP_SOFTARGMIN)
    b = ww.disparity_regression(cost[:, 0].contiguous(), ww.DISP_SOFTARGMIN)
    p = plugins.get_plugin_creator("DisparityRegression").create_plugin({"mode": 1})
    c = torch.empty_like(a)
    assert p.enqueue([plugins.TensorDesc.of(cost)], [plugins.TensorDesc.of(c)], [cost], [c]) == 0
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, c)


def test_unaligned_output_takes_the_scalar_path(env):
    """An output that is not 8-byte aligned must not use the vector stores."""
    torch, ww = env
    import oracle
    cost = _cost((1, 16, 4, 8), 2.0, 4, np.float16)
    x = torch.from_numpy(cost).cuda()
    buf = torch.zeros(1 + 32, dtype=torch.float16, device="cuda")
    out = buf[1:].view(1, 1, 4, 8)
    ww.disparity_regression(x, 0, out=out)
    torch.cuda.synchronize()
    assert buf[0].item() == 0.0
    ref = oracle.disparity_regression(cost, 0).astype(np.float64)
    g = out.cpu().numpy().astype(np.float64)
    assert np.all(np.abs(g - ref) <= RTOL * np.maximum(np.abs(ref), 1.0) + _ulp16(ref))


def test_full_size_against_torch_fp32(env):
    """The bench workload ([64, 48, 94, 312] fp16, soft-argmin) against a plain
    torch fp32 softmax; the shift by a constant along D leaves it unchanged."""
    torch, ww = env
    g = torch.Generator(device="cuda").manual_seed(3)
    cost = (torch.randn((64, 48, 94, 312), generator=g, device="cuda") * 2.0).half()
    got = ww.disparity_regression(cost, ww.DISP_SOFTARGMIN, dtype=torch.float32)
    d = torch.arange(48, device="cuda", dtype=torch.float32).view(1, -1, 1, 1)
    ref = (torch.softmax(-cost.float(), dim=1) * d).sum(dim=1, keepdim=True)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-4)
    # fp16 values + 5 are exact in fp32: the shifted fp32 cost gives the same disparity
    shifted = ww.disparity_regression(cost.float() + 5.0, ww.DISP_SOFTARGMIN)
    assert torch.allclose(shifted, got, rtol=1e-4, atol=1e-4)
    assert ww.device_error() == 0


def test_argument_errors(env):
    torch, ww = env
    x = torch.zeros((1, 4, 2, 2), device="cuda")
    with pytest.raises(ValueError):
        ww.disparity_regression(x, mode=3)
    with pytest.raises(TypeError):
        ww.disparity_regression(x.to(torch.int32))
    L = ww.lib()
    assert L.ww_disparity_regression(None, None, 1, 1, 1, 4, 2, 2, 0, None) == 4  # null pointer
    assert L.ww_disparity_regression(x.data_ptr(), x.data_ptr(), 0, 0, 1, 0, 2, 2, 0, None) == 2  # D = 0
    assert L.ww_disparity_regression(x.data_ptr(), x.data_ptr(), 0, 0, 1, 4, 2, 2, 7, None) == 5  # mode
    assert L.ww_disparity_regression(x.data_ptr(), x.data_ptr(), 0, 0, 0, 4, 2, 2, 0, None) == 0  # B = 0
