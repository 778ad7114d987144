"""ww_nv12_decode on the GPU against the reference kernel (golden fixtures and
oracle/_ref live, one image per call as the reference launcher takes it) and
against the CPU oracle for batches: bit-identical fp16 and fp32 outputs."""
import numpy as np
import pytest

from conftest import golden_files, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    import whirlwind_trt_plugins_b200 as ww
    return torch, ww


def _img(B, H, W, seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=(B, H * 3 // 2, W), dtype=np.uint8)


@pytest.mark.parametrize("name", [f for f in golden_files() if f.startswith("nv12")])
def test_matches_reference_golden(env, name):
    torch, ww = env
    g = load_golden(name)
    f16 = str(g["kind"]) == "nv12_16"
    x = torch.from_numpy(g["nv12"]).cuda()
    out = ww.nv12_decode(x, int(g["H_OUT"]), int(g["W_OUT"]), torch.float16 if f16 else torch.float32)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert got.shape == g["out"].shape
    view = np.uint16 if f16 else np.uint32
    assert np.array_equal(got.view(view), g["out"].view(view))


SHAPES = [(96, 128, 48, 64), (30, 40, 45, 61), (120, 160, 224, 288), (14, 22, 9, 13), (720, 1280, 224, 288),
          (64, 64, 64, 64), (2, 2, 1, 1)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("f16", [True, False])
def test_matches_reference_live(env, shape, f16):
    torch, ww = env
    import oracle
    R = oracle.ref_lib()
    Hi, Wi, Ho, Wo = shape
    x = torch.from_numpy(_img(1, Hi, Wi, 7)).cuda()
    dt = torch.float16 if f16 else torch.float32
    ref = torch.full((1, 3, Ho, Wo), float("nan"), dtype=dt, device="cuda")
    fn = R.wwref_nv12_decode_f16 if f16 else R.wwref_nv12_decode_f32
    assert fn(x.data_ptr(), ref.data_ptr(), Hi, Wi, Ho, Wo, torch.cuda.current_stream().cuda_stream) == 0
    out = ww.nv12_decode(x, Ho, Wo, dt)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16 if f16 else torch.int32), ref.view(torch.int16 if f16 else torch.int32))


@pytest.mark.parametrize("f16", [True, False])
def test_batches_match_oracle(env, orc, f16):
    torch, ww = env
    img = _img(3, 48, 80, 9)
    want = orc.nv12_decode(img, 37, 51, out_f16=f16)
    out = ww.nv12_decode(torch.from_numpy(img).cuda(), 37, 51, torch.float16 if f16 else torch.float32)
    got = out.cpu().numpy()
    view = np.uint16 if f16 else np.uint32
    assert np.array_equal(got.view(view), want.view(view))


def test_int8_input_and_unaligned_output(env, orc):
    torch, ww = env
    img = _img(2, 32, 48, 11)
    want = orc.nv12_decode(img, 20, 30)
    x = torch.from_numpy(img.view(np.int8)).cuda()  # TensorRT declares the bytes INT8
    flat = torch.empty(2 * 3 * 20 * 30 + 1, dtype=torch.float16, device="cuda")
    out = flat[1:].view(2, 3, 20, 30)  # 2-byte offset: the paired-store path is off
    ww.nv12_decode(x, 20, 30, out=out)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_plugin_enqueue(env, orc):
    torch, ww = env
    from whirlwind_trt_plugins_b200 import plugins as pl
    T = pl.TensorDesc
    img = _img(2, 60, 80, 13)
    x = torch.from_numpy(img.view(np.int8)).cuda()
    p = pl.get_plugin_creator("Nv12Decode").create_plugin({"out_h": 45, "out_w": 52})
    for dt, f16 in ((torch.float16, True), (torch.float32, False)):
        out = torch.empty((2, 3, 45, 52), dtype=dt, device="cuda")
        assert p.enqueue([T.of(x)], [T.of(out)], [x], [out]) == 0
        want = orc.nv12_decode(img, 45, 52, out_f16=f16)
        view = np.uint16 if f16 else np.uint32
        assert np.array_equal(out.cpu().numpy().view(view), want.view(view))
