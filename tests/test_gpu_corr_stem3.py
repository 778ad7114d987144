"""ww_corr_cost_stem3d_ref3 -- CorrVolume (G = 1) fused with the reference's
3-stage CostStem3D -- on the GPU: bit-identical to ww_corr_volume followed by
ww_cost_stem3d_ref3 (both rules of the reference's correlation scale, ragged
shapes, several batch items), to the reference's own two kernels run one after
the other at B = 1, through the CorrCostStem3D plugin with 8 inputs, and inside
a CUDA graph."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    import torch
    import whirlwind_trt_plugins_b200 as ww
    return torch, ww


def _weights(torch, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [(torch.randn((n,), generator=g, device="cuda") * s).half()
            for n, s in ((108, 0.2), (4, 0.1), (432, 0.2), (4, 0.1), (108, 0.2), (1, 0.1))]


def _features(torch, B, C, H, W, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn((B, C, H, W), generator=g, device="cuda").half(),
            torch.randn((B, C, H, W), generator=g, device="cuda").half())


# (B, C, H, W, D): the native shape with two channel counts, ragged H/W/D and
# C not a multiple of the 12-channel chunk, D > W, and two shapes on which the
# reference's correlation divides by C (the others multiply by 1/C).
SHAPES = [(1, 64, 32, 40, 48), (1, 128, 32, 40, 48), (2, 20, 19, 37, 13), (1, 8, 8, 8, 8), (3, 32, 12, 70, 30),
          (1, 16, 30, 20, 64), (4, 64, 64, 80, 48), (1, 32, 120, 160, 48)]


def test_shapes_cover_both_scale_rules():
    import oracle
    modes = {oracle.ref_scale_mode(True, B, C, H, W, D) for B, C, H, W, D in SHAPES}
    assert modes == {0, 1}


@pytest.mark.parametrize("shape", SHAPES)
def test_matches_the_unfused_pair(env, shape):
    torch, ww = env
    B, C, H, W, D = shape
    L, R = _features(torch, B, C, H, W, 100 + C)
    ws = _weights(torch, C)
    fused = ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=D)
    pair = ww.cost_stem3d_ref3(ww.corr_volume(L, R, D).unsqueeze(1), *ws)
    torch.cuda.synchronize()
    assert fused.shape == (B, 1, D, H, W)
    assert torch.equal(fused, pair)
    assert ww.device_error() == 0


@pytest.mark.parametrize("shape", [(1, 64, 32, 40, 48), (1, 20, 19, 37, 13), (1, 32, 120, 160, 48)])
def test_matches_the_reference_kernels(env, shape):
    torch, ww = env
    import oracle
    ref = oracle.ref_lib()
    B, C, H, W, D = shape
    L, R = _features(torch, B, C, H, W, 7)
    ws = _weights(torch, 8)
    vol = torch.empty((B, D, H, W), dtype=torch.float16, device="cuda")
    o_ref = torch.empty((B, 1, D, H, W), dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert ref.wwref_corr_volume_f16(L.data_ptr(), R.data_ptr(), vol.data_ptr(), B, C, H, W, D, s) == 0
    assert ref.wwref_cost_stem3d(vol.data_ptr(), o_ref.data_ptr(), *[w.data_ptr() for w in ws], B, D, H, W,
                                 s) == 0
    fused = ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=D)
    torch.cuda.synchronize()
    assert torch.equal(fused, o_ref)


def test_plugin_with_eight_inputs(env):
    torch, ww = env
    from whirlwind_trt_plugins_b200 import plugins
    B, C, H, W, D = 2, 24, 16, 24, 16
    L, R = _features(torch, B, C, H, W, 3)
    ws = _weights(torch, 4)
    p = plugins.get_plugin_creator("CorrCostStem3D").create_plugin({"max_disp": D})
    ins = [L, R] + ws
    descs = [plugins.TensorDesc.of(t) for t in ins]
    assert p.get_output_shapes(descs) == [(B, 1, D, H, W)]
    out = torch.empty((B, 1, D, H, W), dtype=torch.float16, device="cuda")
    assert p.enqueue(descs, ins, [out]) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=D))
    # num_groups > 1 has no 3-stage form
    q = plugins.get_plugin_creator("CorrCostStem3D").create_plugin({"max_disp": D, "num_groups": 2})
    assert q.enqueue(descs, ins, [out]) == 1
