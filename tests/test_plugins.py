"""The Python plugin mirror (whirlwind_trt_plugins_b200.plugins) against the
reference plugins' behaviour: creator names, versions, field defaults,
output shapes and types, format support, serialised fields, clone; and on a
GPU, enqueue through the plugin equals the direct call."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def pl():
    from whirlwind_trt_plugins_b200 import plugins
    return plugins


def test_registry_and_defaults(pl):
    assert ("CorrVolume", "1") in pl.registered_creators()
    assert ("CostStem3D", "1") in pl.registered_creators()
    cv = pl.get_plugin_creator("CorrVolume").create_plugin({})
    assert cv.get_plugin_name() == "CorrVolume" and cv.get_plugin_version() == "1"
    # max_disp defaults to 48 (corr_volume.cpp:138); an absent value falls back
    assert cv.max_disp == 48 and cv.num_groups == 1
    assert pl.get_plugin_creator("CorrVolume").create_plugin({"max_disp": 64, "num_groups": None}).max_disp == 64
    # the reference serialises exactly max_disp (corr_volume.cpp:113-123)
    assert cv.get_fields_to_serialize() == {"max_disp": 48}
    st = pl.get_plugin_creator("CostStem3D").create_plugin()
    assert st.get_fields_to_serialize() == {} and st.get_nb_outputs() == 1
    with pytest.raises(KeyError):
        pl.get_plugin_creator("CorrVolume", "2")


def test_clone_keeps_state_and_namespace(pl):
    p = pl.CorrVolumePlugin(max_disp=32, num_groups=8)
    p.namespace = "ns"
    q = p.clone()
    assert q is not p and q.max_disp == 32 and q.num_groups == 8 and q.namespace == "ns"


def test_output_shapes_types_formats(pl):
    T = pl.TensorDesc
    cv = pl.CorrVolumePlugin(max_disp=24)
    feats = [T((2, 32, 60, 80)), T((2, 32, 60, 80))]
    assert cv.get_output_shapes(feats) == [(2, 24, 60, 80)]
    assert pl.CorrVolumePlugin(24, 8).get_output_shapes(feats) == [(2, 8, 24, 60, 80)]
    assert cv.get_output_data_types([1, 1]) == [1]
    with pytest.raises(ValueError):
        cv.get_output_shapes(feats[:1])
    # fp16 only at position 0, LINEAR only, others follow position 0 (corr_volume.cpp:60-82)
    assert cv.supports_format_combination(0, [T((1,), 1)] * 3, 2, 1)
    assert not cv.supports_format_combination(0, [T((1,), 0)] * 3, 2, 1)
    assert not cv.supports_format_combination(0, [T((1,), 1, 1)] + [T((1,), 1)] * 2, 2, 1)
    st = pl.CostStem3DPlugin()
    seven = [T((1, 1, 48, 32, 40))] + [T((n,)) for n in (108, 4, 432, 4, 108, 1)]
    assert st.get_output_shapes(seven) == [(1, 1, 48, 32, 40)]
    three = [T((2, 40, 48, 30, 40)), T((32, 40, 3, 3, 3)), T((32,))]
    assert st.get_output_shapes(three) == [(2, 32, 48, 30, 40)]
    assert st.supports_format_combination(3, seven + [T((1, 1, 48, 32, 40))], 7, 1)
    fused = pl.CorrCostStem3DPlugin(48, 40, 0)
    ins = [T((1, 320, 120, 160)), T((1, 320, 120, 160)), T((32, 40, 3, 3, 3)), T((32,))]
    assert fused.get_output_shapes(ins) == [(1, 32, 48, 120, 160)]
    assert fused.get_fields_to_serialize() == {"max_disp": 48, "num_groups": 40, "act": 0}
    # 8 inputs: CorrVolume (G = 1) fused with the reference's 3-stage stem
    native = pl.CorrCostStem3DPlugin(48, 1, 0)
    eight = [T((1, 64, 32, 40)), T((1, 64, 32, 40))] + [T((n,)) for n in (108, 4, 432, 4, 108, 1)]
    assert native.get_output_shapes(eight) == [(1, 1, 48, 32, 40)]
    out = T((1, 1, 48, 32, 40))
    assert all(native.supports_format_combination(i, eight + [out], 8, 1) for i in range(9))
    assert not native.supports_format_combination(8, eight + [T((1, 1, 48, 32, 40), 0)], 8, 1)
    with pytest.raises(ValueError):
        native.get_output_shapes(eight[:5])


@pytest.mark.gpu
def test_enqueue_matches_direct_calls(pl):
    import torch
    import whirlwind_trt_plugins_b200 as ww
    T = pl.TensorDesc
    g = torch.Generator(device="cuda").manual_seed(5)
    l = torch.randn((1, 64, 20, 40), generator=g, device="cuda").half()
    r = torch.randn((1, 64, 20, 40), generator=g, device="cuda").half()
    cv = pl.get_plugin_creator("CorrVolume").create_plugin({"max_disp": 24})
    out = torch.empty((1, 24, 20, 40), dtype=torch.float16, device="cuda")
    assert cv.enqueue([T.of(l), T.of(r)], [l, r], [out]) == 0
    ref = ww.corr_volume(l, r, 24)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    w = (torch.randn((16, 8, 3, 3, 3), generator=g, device="cuda") * 0.1).half()
    b = (torch.randn((16,), generator=g, device="cuda") * 0.1).half()
    fused = pl.CorrCostStem3DPlugin(24, 8, 1)
    out2 = torch.empty((1, 16, 24, 20, 40), dtype=torch.float16, device="cuda")
    descs = [T.of(l), T.of(r), T.of(w), T.of(b)]
    assert fused.get_output_shapes(descs) == [tuple(out2.shape)]
    assert fused.enqueue(descs, [l, r, w, b], [out2]) == 0
    ref2 = ww.corr_cost_stem3d(l, r, w, b, 24, 8, 1)
    torch.cuda.synchronize()
    assert torch.equal(out2, ref2)
    # a rejected request returns 1 like IPluginV3OneRuntime::enqueue
    assert fused.enqueue([T.of(l), T.of(r), T((16, 4, 3, 3, 3)), T.of(b)], [l, r, w, b], [out2]) == 1
