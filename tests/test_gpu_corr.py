"""GPU parity of ww_corr_volume (CorrVolume) against the reference's own CUDA
kernels (golden fixtures and oracle/_ref live) and the CPU oracle.
Integer-exact bar: outputs must be bit-identical."""
import numpy as np
import pytest

from conftest import golden_files, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


@pytest.fixture(scope="module")
def ww():
    import whirlwind_trt_plugins_b200 as ww
    return ww


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16) if a.dtype == np.float16 else a.view(np.uint32)


def _run(ww, torch, L, R, D, G=1, offset=0):
    """Run the product kernel; `offset` shifts the device pointers by that many
    elements to exercise the unaligned path."""
    dev = torch.device("cuda:0")
    tl = torch.from_numpy(np.ascontiguousarray(L)).to(dev)
    tr = torch.from_numpy(np.ascontiguousarray(R)).to(dev)
    if offset:
        bl = torch.empty(tl.numel() + offset, dtype=tl.dtype, device=dev)
        br = torch.empty_like(bl)
        bl[offset:].copy_(tl.flatten())
        br[offset:].copy_(tr.flatten())
        tl = bl[offset:].view(tl.shape)
        tr = br[offset:].view(tr.shape)
    B, C, H, W = L.shape
    shape = (B, D, H, W) if G == 1 else (B, G, D, H, W)
    # canary-padded output: kernel writes must stay inside [pad, pad + n)
    n = int(np.prod(shape))
    pad = 64
    buf = torch.full((n + 2 * pad,), 7.0, dtype=tl.dtype, device=dev)
    out = buf[pad:pad + n].view(shape)
    ww.corr_volume(tl, tr, D, G, out=out)
    torch.cuda.synchronize()
    host = buf.cpu().numpy()
    assert np.all(host[:pad] == 7.0) and np.all(host[pad + n:] == 7.0), "write outside the output tensor"
    return out.cpu().numpy()


@pytest.mark.parametrize("name", [f for f in golden_files() if "corr" in f])
def test_corr_matches_reference_golden(ww, torch, name):
    g = load_golden(name)
    out = _run(ww, torch, g["left"], g["right"], int(g["D"]), int(g["G"]))
    assert out.shape == g["out"].shape
    assert np.array_equal(_bits(out), _bits(g["out"])), f"{name}: differs from the reference kernel"


def _ref_available():
    import os
    import oracle
    return os.path.exists(oracle.REF_SO)


# Volumes below ~800 outputs per SM take the one-thread-per-output path, the
# others the tiled kernel: 128-column tiles, or 64 / 32 columns for images that
# narrow ((2, 32, 96, 48, 64, 1) and (2, 16, 128, 24, 32, 2)).  The first entry
# is the reference's native CorrVolume shape.
@pytest.mark.parametrize("shape", [
    (1, 64, 32, 40, 48, 1),
    (1, 16, 32, 128, 48, 1), (1, 12, 32, 128, 48, 1), (2, 64, 16, 80, 24, 1), (1, 24, 12, 64, 64, 2),
    (1, 320, 16, 160, 48, 40), (2, 64, 12, 128, 32, 16), (1, 32, 7, 40, 30, 4), (1, 8, 3, 200, 36, 1),
    (2, 32, 96, 48, 64, 1), (2, 16, 128, 24, 32, 2),
    (1, 64, 6, 312, 48, 8), (1, 96, 5, 320, 64, 8),  # row-streaming kernels over two column tiles
])
def test_corr_matches_reference_live(ww, torch, orc, shape):
    if not _ref_available():
        pytest.skip("oracle/_ref/libww_ref.so not built")
    B, C, H, W, D, G = shape
    rng = np.random.default_rng(sum(shape))
    L = rng.standard_normal((B, C, H, W)).astype(np.float16)
    R = rng.standard_normal((B, C, H, W)).astype(np.float16)
    dev = torch.device("cuda:0")
    tl, tr = torch.from_numpy(L).to(dev), torch.from_numpy(R).to(dev)
    ref = torch.full((B, G, D, H, W), float("nan"), dtype=torch.float16, device=dev)
    rc = orc.ref_lib().wwref_corr_volume_grouped_f16(tl.data_ptr(), tr.data_ptr(), ref.data_ptr(), B, C, H, W, D,
                                                      G, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    out = _run(ww, torch, L, R, D, G)
    assert np.array_equal(_bits(out).reshape(-1), _bits(ref.cpu().numpy()).reshape(-1))


@pytest.mark.parametrize("cfg_id", [1, 2, 3, 4, 5])
def test_corr_configs_match_oracle(ww, torch, orc, cfg_id):
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[cfg_id]
    if cfg_id != 1:
        cfg = cfg.scaled(H=min(cfg.H, 12), B=min(cfg.B, 2))
    x = make_inputs(cfg)
    out = _run(ww, torch, x["left"], x["right"], cfg.D, cfg.G)
    if cfg.dtype == "f32":
        ref = orc.corr_f32(x["left"], x["right"], cfg.D, cfg.G)
    else:
        ref = orc.corr_f16(x["left"], x["right"], cfg.D, cfg.G)
    assert np.array_equal(_bits(out), _bits(ref))


@pytest.mark.parametrize("case", [
    dict(B=1, C=4, H=1, W=5, D=1, G=1),          # minimal
    dict(B=1, C=8, H=2, W=6, D=20, G=2),          # D > W
    dict(B=3, C=6, H=5, W=37, D=13, G=3),         # ragged W, odd D
    dict(B=1, C=40, H=3, W=131, D=70, G=5),       # several column tiles, several disparity bands
    dict(B=1, C=17, H=2, W=16, D=8, G=17),        # one channel per group
])
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_corr_edge_cases(ww, torch, orc, case, dtype):
    rng = np.random.default_rng(case["W"] * 7 + case["D"])
    shp = (case["B"], case["C"], case["H"], case["W"])
    L = rng.standard_normal(shp).astype(dtype)
    R = rng.standard_normal(shp).astype(dtype)
    out = _run(ww, torch, L, R, case["D"], case["G"])
    if dtype == np.float32:
        ref = orc.corr_f32(L, R, case["D"], case["G"])
    else:
        ref = orc.corr_f16(L, R, case["D"], case["G"])
    assert np.array_equal(_bits(out), _bits(ref))
    # w - d < 0 is exactly +0
    o = out.reshape(case["B"], case["G"], case["D"], case["H"], case["W"])
    for d in range(min(case["D"], case["W"])):
        assert not np.any(_bits(o[:, :, d, :, :d]))


@pytest.mark.parametrize("D", [40, 56])  # the 8 x 8 and the 4 x 8 row-streaming tiles
@pytest.mark.parametrize("G", [2, 6])    # Cg = 12 (divided) and 4 (multiplied), both under the naive rule
def test_corr_nonfinite_and_extreme_features(ww, torch, orc, D, G):
    """Infinite, NaN, signed-zero and near-overflow features under the naive
    scale rule: the row kernels' division takes its exact path for tiles
    holding a non-finite sum, and every finite output stays bit-identical to
    the oracle (NaN outputs compared as NaN, whatever their payload)."""
    rng = np.random.default_rng(D + G)
    L = rng.standard_normal((1, 24, 4, 96)).astype(np.float16)
    R = rng.standard_normal((1, 24, 4, 96)).astype(np.float16)
    L[0, 3, 1, 10] = np.inf
    R[0, 5, 2, 50] = -np.inf
    L[0, 14, 0, 70] = np.nan
    L[0, 7, 3, 20:28] = 60000.0
    R[0, 7, 3, 0:40] = -60000.0
    L[0, 9, :, 30:40] = -0.0
    R[0, 9, :, :] = 0.0
    out = _run(ww, torch, L, R, D, G)
    ref = orc.corr_f16(L, R, D, G)
    nan_o, nan_r = np.isnan(out), np.isnan(ref)
    assert np.array_equal(nan_o, nan_r)
    assert np.isinf(out).any() and nan_o.any()
    assert np.array_equal(_bits(np.where(nan_o, 0, out).astype(np.float16)),
                          _bits(np.where(nan_r, 0, ref).astype(np.float16)))


def test_corr_unaligned_pointers(ww, torch, orc):
    rng = np.random.default_rng(99)
    L = rng.standard_normal((1, 16, 4, 64)).astype(np.float16)
    R = rng.standard_normal((1, 16, 4, 64)).astype(np.float16)
    out = _run(ww, torch, L, R, 24, 2, offset=1)
    ref = orc.corr_f16(L, R, 24, 2)
    assert np.array_equal(_bits(out), _bits(ref))


def test_corr_rejects_bad_arguments(ww, torch):
    dev = torch.device("cuda:0")
    x = torch.zeros((1, 6, 2, 8), dtype=torch.float16, device=dev)
    with pytest.raises(ww.WWError):
        ww.corr_volume(x, x, 4, num_groups=4)


def test_int_division_matches_rounded_division_on_every_float(ww):
    """The naive rule's division by the group width is a multiply by the
    rounded reciprocal plus one correction fma (Markstein); for every divisor
    the library uses it for (1..1024) it equals the IEEE rounded division on
    all 2^32 fp32 inputs, NaN payloads aside."""
    import ctypes
    L = ww.lib()
    bad = {}
    for b in range(1, 1025):
        n = ctypes.c_ulonglong(0)
        assert L.ww_selftest_int_division(b, ctypes.byref(n)) == 0
        if n.value:
            bad[b] = n.value
    assert not bad, f"divisors with mismatches: {dict(list(bad.items())[:10])}"
