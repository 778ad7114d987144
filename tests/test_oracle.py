"""CPU tests of the oracle itself: conversions, known-answer tests, and
cross-checks against independent implementations (numpy, torch CPU conv3d).
No GPU needed."""
import numpy as np
import pytest


def test_f32_to_f16_matches_numpy(orc):
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10,
        rng.standard_normal(5000).astype(np.float32) * 1e-5,          # subnormal half range
        rng.standard_normal(5000).astype(np.float32) * 3e4,           # near the top
        np.array([0.0, -0.0, 65504, 65519.99, 65520, -65520, 1e9, -1e9, np.inf, -np.inf,
                  6.1035156e-05, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 1.0 + 2**-11,
                  1.0 + 3 * 2**-11, 2049.0, 2051.0], dtype=np.float32),
    ])
    # every float exactly halfway between two adjacent halves
    h = np.arange(0, 0x7bff, dtype=np.uint16).view(np.float16).astype(np.float32)
    mid = ((h[:-1].astype(np.float64) + h[1:].astype(np.float64)) / 2).astype(np.float32)
    vals = np.concatenate([vals, mid, -mid])
    got = orc.f32_to_f16(vals).view(np.uint16)
    want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_f16_to_f32_all_patterns(orc):
    L = orc.lib()
    bits = np.arange(65536, dtype=np.uint16)
    want = bits.view(np.float16).astype(np.float32)
    got = np.array([L.orc_f16_to_f32(int(b)) for b in bits[::7]], dtype=np.float32)
    w = want[::7]
    nan = np.isnan(w)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), w[~nan].view(np.uint32))


def test_corr_known_answer_ones(orc):
    B, C, H, W, D = 1, 8, 3, 12, 5
    L = np.ones((B, C, H, W), np.float16)
    out = orc.corr_f16(L, L, D).astype(np.float32)
    for d in range(D):
        assert np.all(out[0, d, :, d:] == 1.0)
        assert np.all(out[0, d, :, :d] == 0.0)
        assert not np.any(np.signbit(out[0, d, :, :d]))  # exact +0


def test_corr_one_hot_channel_is_shifted_copy(orc):
    rng = np.random.default_rng(3)
    B, C, H, W, D = 1, 4, 2, 16, 6
    L = np.zeros((B, C, H, W), np.float32)
    L[:, 2] = 1.0
    R = rng.standard_normal((B, C, H, W)).astype(np.float32)
    out = orc.corr_f32(L, R, D)
    for d in range(D):
        np.testing.assert_array_equal(out[0, d, :, d:], R[0, 2, :, :W - d] / np.float32(C))
        assert np.all(out[0, d, :, :d] == 0)


def test_corr_d_greater_than_w_gives_zero_columns(orc):
    rng = np.random.default_rng(4)
    L = rng.standard_normal((1, 4, 2, 5)).astype(np.float16)
    out = orc.corr_f16(L, L, 9).astype(np.float32)
    assert np.all(out[0, 5:] == 0)


def test_corr_grouped_matches_float64(orc):
    rng = np.random.default_rng(5)
    B, C, G, H, W, D = 2, 24, 3, 4, 20, 7
    L = rng.standard_normal((B, C, H, W)).astype(np.float32)
    R = rng.standard_normal((B, C, H, W)).astype(np.float32)
    out = orc.corr_f32(L, R, D, G)
    Cg = C // G
    ref = np.zeros((B, G, D, H, W))
    for d in range(D):
        prod = L[..., d:].astype(np.float64) * R[..., :W - d].astype(np.float64)
        ref[:, :, d, :, d:] = prod.reshape(B, G, Cg, H, W - d).mean(axis=2)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-6)


def test_corr_scale_modes_agree_for_power_of_two(orc):
    rng = np.random.default_rng(6)
    L = rng.standard_normal((1, 8, 3, 16)).astype(np.float16)
    R = rng.standard_normal((1, 8, 3, 16)).astype(np.float16)
    a = orc.corr_f16(L, R, 6, scale_mode=orc.SCALE_DIV).view(np.uint16)
    b = orc.corr_f16(L, R, 6, scale_mode=orc.SCALE_MULINV).view(np.uint16)
    assert np.array_equal(a, b)


def _torch_conv3d(vol, w, b, act):
    torch = pytest.importorskip("torch")
    x = torch.from_numpy(vol.astype(np.float64))
    wt = torch.from_numpy(w.astype(np.float64))
    y = torch.nn.functional.conv3d(x, wt, torch.from_numpy(b.astype(np.float64)), padding=1)
    y = torch.clamp(y, min=0.0)
    if act == 1:
        y = torch.clamp(y, max=6.0)
    return y.numpy()


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("acc_mode", [0, 1])
def test_stem_matches_torch_conv3d(orc, act, acc_mode):
    rng = np.random.default_rng(7)
    B, Cin, Cout, D, H, W = 2, 5, 3, 6, 5, 7
    vol = (rng.standard_normal((B, Cin, D, H, W)) * 0.5).astype(np.float16)
    w = (rng.standard_normal((Cout, Cin, 3, 3, 3)) * 0.2).astype(np.float16)
    b = (rng.standard_normal(Cout) * 0.2).astype(np.float16)
    got = orc.stem(vol, w, b, act=act, acc_mode=acc_mode).astype(np.float32)
    ref = _torch_conv3d(vol.astype(np.float32), w.astype(np.float32), b.astype(np.float32), act)
    np.testing.assert_allclose(got, ref, atol=2e-3, rtol=2e-3)


def test_stem_delta_weights_identity_relu(orc):
    rng = np.random.default_rng(8)
    B, C, D, H, W = 1, 4, 5, 4, 6
    vol = rng.standard_normal((B, C, D, H, W)).astype(np.float16)
    w = np.zeros((C, C, 3, 3, 3), np.float16)
    for o in range(C):
        w[o, o, 1, 1, 1] = 1.0
    b = np.zeros(C, np.float16)
    out = orc.stem(vol, w, b, act=0)
    np.testing.assert_array_equal(out, np.maximum(vol, 0).astype(np.float16))


def test_stem_ref3_matches_layerwise_torch(orc):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    D, H, W = 7, 6, 5
    x = (rng.standard_normal((1, 1, D, H, W)) * 2).astype(np.float16)
    w0 = (rng.standard_normal((4, 1, 3, 3, 3)) * 0.3).astype(np.float16)
    w1 = (rng.standard_normal((4, 4, 3, 3, 3)) * 0.2).astype(np.float16)
    w2 = (rng.standard_normal((1, 4, 3, 3, 3)) * 0.2).astype(np.float16)
    b0, b1 = (rng.standard_normal(4) * 0.2).astype(np.float16), (rng.standard_normal(4) * 0.2).astype(np.float16)
    b2 = np.array([0.5], np.float16)
    got = orc.stem_ref3(x, w0, b0, w1, b1, w2, b2).astype(np.float32)
    y = torch.from_numpy(x.astype(np.float32))
    for w, b in ((w0, b0), (w1, b1), (w2, b2)):
        y = torch.nn.functional.conv3d(y, torch.from_numpy(w.astype(np.float32)),
                                       torch.from_numpy(b.astype(np.float32)), padding=1)
        y = torch.clamp(y, 0, 6).half().float()
    np.testing.assert_allclose(got, y.numpy(), atol=4e-3, rtol=4e-3)


def test_corr_stem_band_equals_full(orc):
    rng = np.random.default_rng(10)
    B, C, G, H, W, D, Cout = 2, 16, 4, 9, 12, 8, 5
    L = rng.standard_normal((B, C, H, W)).astype(np.float16)
    R = rng.standard_normal((B, C, H, W)).astype(np.float16)
    w = (rng.standard_normal((Cout, G, 3, 3, 3)) * 0.1).astype(np.float16)
    b = (rng.standard_normal(Cout) * 0.1).astype(np.float16)
    full = orc.corr_stem(L, R, w, b, D, G)
    # the fused oracle equals corr -> stem composed
    vol = orc.corr_f16(L, R, D, G)
    comp = orc.stem(vol, w, b)
    assert np.array_equal(full.view(np.uint16), comp.view(np.uint16))
    # and computing row bands / batch slices separately stitches to the same tensor
    out = np.zeros_like(full)
    for (b0, b1) in ((0, 1), (1, 2)):
        for (h0, h1) in ((0, 4), (4, 5), (5, 9)):
            orc.corr_stem(L, R, w, b, D, G, batches=(b0, b1), rows=(h0, h1), out=out)
    assert np.array_equal(out.view(np.uint16), full.view(np.uint16))


def test_fold_bn_matches_numpy(orc):
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((6, 4, 3, 3, 3)) * 0.05).astype(np.float32)
    scale = rng.uniform(0.5, 1.5, 6).astype(np.float32)
    bias = (rng.standard_normal(6) * 0.1).astype(np.float32)
    w16, b16 = orc.fold_bn(w, scale, bias)
    assert np.array_equal(w16.view(np.uint16), (w * scale[:, None, None, None, None]).astype(np.float16).view(np.uint16))
    assert np.array_equal(b16.view(np.uint16), bias.astype(np.float16).view(np.uint16))


def test_ref_scale_mode_rules(orc):
    # fp32 always takes the naive kernel (division)
    assert orc.ref_scale_mode(False, 1, 16, 32, 128, 48) == orc.SCALE_DIV
    # fast path needs W % 8 == 0, D % 6 == 0 and >= SMs * 800 outputs
    assert orc.ref_scale_mode(True, 1, 16, 32, 128, 48) == orc.SCALE_MULINV
    assert orc.ref_scale_mode(True, 1, 16, 32, 124, 48) == orc.SCALE_DIV
    assert orc.ref_scale_mode(True, 1, 16, 32, 128, 64) == orc.SCALE_DIV
    assert orc.ref_scale_mode(True, 1, 16, 8, 64, 48) == orc.SCALE_DIV
    # large C: shared memory holds no tile at all -> naive
    assert orc.ref_scale_mode(True, 1, 4096, 32, 128, 48) == orc.SCALE_DIV
    # the group-wise composition is judged per (b, g) call with C = C/G
    assert orc.grouped_scale_mode(True, 1, 320, 40, 120, 160, 48) == orc.SCALE_MULINV
    assert orc.grouped_scale_mode(True, 4, 96, 8, 180, 320, 64) == orc.SCALE_DIV
