"""NV12 decode on CPU: the oracle's known answers and the Nv12Decode plugin
mirror (shapes, formats, fields) against the reference plugin's behaviour
(src/plugins/nv12_decode/nv12_decode.cpp:26-146).  The oracle's bit-level
parity with the reference kernel is pinned by the nv12_* golden fixtures
(tests/test_golden.py)."""
import numpy as np
import pytest


def _nv12(rng, H, W):
    return rng.integers(0, 256, size=(H * 3 // 2, W), dtype=np.uint8)


def test_grey_image_decodes_to_constant(orc):
    img = np.full((12, 8), 128, dtype=np.uint8)  # Y = U = V = 128
    out = orc.nv12_decode(img, 5, 7, out_f16=False)
    # 2 * 128 / 255 - 1 for R, G and B
    assert np.allclose(out, 2.0 * 128 / 255 - 1, atol=1e-6)


def test_identity_size_is_the_colour_transform(orc):
    rng = np.random.default_rng(3)
    H, W = 8, 12
    img = _nv12(rng, H, W)
    out = orc.nv12_decode(img, H, W, out_f16=False)[0]
    Y = img[:H].astype(np.float64)
    uv = img[H:].reshape(H // 2, W // 2, 2).astype(np.float64)
    # luma sampled at the pixel itself; chroma at (y + 0.5) / 2 - 0.5 bilinear
    assert out.shape == (3, H, W)
    cb = np.empty((H, W))
    cr = np.empty((H, W))
    for y in range(H):
        for x in range(W):
            yf, xf = (y + 0.5) * 0.5 - 0.5, (x + 0.5) * 0.5 - 0.5
            y0, x0 = int(np.floor(yf)), int(np.floor(xf))
            wy, wx = yf - y0, xf - x0
            def tap(yy, xx, c):
                return uv[min(max(yy, 0), H // 2 - 1), min(max(xx, 0), W // 2 - 1), c]
            for c, dst in ((0, cb), (1, cr)):
                dst[y, x] = ((1 - wy) * ((1 - wx) * tap(y0, x0, c) + wx * tap(y0, x0 + 1, c)) +
                             wy * ((1 - wx) * tap(y0 + 1, x0, c) + wx * tap(y0 + 1, x0 + 1, c))) - 128
    s = 2 / 255
    R = s * (Y + 1.402 * cr) - 1
    G = s * (Y - 0.344136 * cb - 0.714136 * cr) - 1
    B = s * (Y + 1.772 * cb) - 1
    assert np.allclose(out, np.stack([R, G, B]), atol=2e-6)


def test_batch_items_are_independent(orc):
    rng = np.random.default_rng(4)
    a, b = _nv12(rng, 10, 16), _nv12(rng, 10, 16)
    both = orc.nv12_decode(np.stack([a, b]), 7, 9)
    assert np.array_equal(both[0].view(np.uint16), orc.nv12_decode(a, 7, 9)[0].view(np.uint16))
    assert np.array_equal(both[1].view(np.uint16), orc.nv12_decode(b, 7, 9)[0].view(np.uint16))


def test_output_range(orc):
    rng = np.random.default_rng(5)
    out = orc.nv12_decode(_nv12(rng, 30, 40), 17, 23, out_f16=False)
    # random chroma is out of the RGB gamut: the transform's own bounds are
    # (0 - 1.772 * 128) * 2 / 255 - 1 = -2.78 and (255 + 1.772 * 127) * 2 / 255 - 1 = 2.77
    assert out.min() >= -2.78 and out.max() <= 2.77
    assert out.min() < -1 and out.max() > 1


def test_plugin_mirror(ww_plugins):
    pl = ww_plugins
    T = pl.TensorDesc
    p = pl.get_plugin_creator("Nv12Decode").create_plugin({})
    assert (p.out_h, p.out_w) == (224, 288)  # nv12_decode.cpp:143-145
    assert p.get_fields_to_serialize() == {"out_h": 224, "out_w": 288}
    q = pl.get_plugin_creator("Nv12Decode").create_plugin({"out_h": 120, "out_w": None})
    assert (q.out_h, q.out_w) == (120, 288)
    assert p.get_output_shapes([T((2, 180, 160), pl.DTYPE_INT8)]) == [(2, 3, 224, 288)]
    assert p.get_output_data_types([pl.DTYPE_INT8]) == [pl.DTYPE_FLOAT]  # declared fp32
    with pytest.raises(ValueError):
        p.get_output_shapes([T((2, 180, 160)), T((2, 180, 160))])
    i8, f16, f32 = T((1,), pl.DTYPE_INT8), T((1,), pl.DTYPE_HALF), T((1,), pl.DTYPE_FLOAT)
    assert p.supports_format_combination(0, [i8, f16], 1, 1)
    assert not p.supports_format_combination(0, [f32, f16], 1, 1)  # no fp32 input (nv12_decode.cpp:75-82)
    assert p.supports_format_combination(1, [i8, f16], 1, 1) and p.supports_format_combination(1, [i8, f32], 1, 1)
    assert not p.supports_format_combination(1, [i8, i8], 1, 1)
    assert not p.supports_format_combination(0, [T((1,), pl.DTYPE_INT8, 1), f16], 1, 1)


def test_enqueue_rejects_before_launch(ww_plugins):
    pl = ww_plugins
    T = pl.TensorDesc
    p = pl.Nv12DecodePlugin()
    # rank != 3 -> 1 (nv12_decode.cpp:97)
    assert p.enqueue([T((180, 160), pl.DTYPE_INT8)], [T((1, 3, 224, 288), pl.DTYPE_HALF)], [0x1000], [0x1000],
                     stream=0) == 1
    # output dtype not fp16/fp32 -> 1 (nv12_decode.cpp:113)
    assert p.enqueue([T((1, 180, 160), pl.DTYPE_INT8)], [T((1, 3, 224, 288), pl.DTYPE_INT8)], [0x1000],
                     [0x1000], stream=0) == 1


def test_c_abi_validates(ww_lib):
    L = ww_lib
    fake = 0x1000
    assert L.ww_nv12_decode(None, fake, 1, 1, 12, 8, 4, 4, None) == 4
    assert L.ww_nv12_decode(fake, fake, 2, 1, 12, 8, 4, 4, None) == 3
    assert L.ww_nv12_decode(fake, fake, 1, 1, 1, 8, 4, 4, None) == 2
    assert L.ww_nv12_decode(fake, fake, 1, 0, 12, 8, 4, 4, None) == 0  # empty batch: no-op


@pytest.fixture(scope="module")
def ww_plugins():
    from whirlwind_trt_plugins_b200 import plugins
    return plugins


@pytest.fixture(scope="module")
def ww_lib():
    import whirlwind_trt_plugins_b200 as ww
    return ww.lib()
