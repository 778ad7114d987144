"""CPU tests of the C ABI: the library loads, exports every function that
include/*.h declares, and the TensorRT-free plugin layer behaves like the
reference's IPluginV3 methods (shapes, formats, fields, enqueue error paths
that return before any GPU work)."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

HDR_DIR = os.path.join(ROOT, "include")


class Desc(ctypes.Structure):
    _fields_ = [("nb_dims", ctypes.c_int32), ("dims", ctypes.c_int64 * 8),
                ("dtype", ctypes.c_int32), ("format", ctypes.c_int32)]


def desc(dims, dtype=1, fmt=0):
    d = Desc()
    d.nb_dims = len(dims)
    for i, v in enumerate(dims):
        d.dims[i] = v
    d.dtype, d.format = dtype, fmt
    return d


def descs(*ds):
    arr = (Desc * len(ds))()
    for i, d in enumerate(ds):
        arr[i] = d
    return arr


@pytest.fixture(scope="module")
def ww():
    import whirlwind_trt_plugins_b200 as ww
    return ww


def declared_functions():
    names = []
    for f in sorted(os.listdir(HDR_DIR)):
        if not f.endswith(".h"):
            continue
        txt = open(os.path.join(HDR_DIR, f)).read()
        txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(ww_\w+)\s*\(", txt, flags=re.M)
    return names


def test_exports_every_declared_symbol(ww):
    names = declared_functions()
    assert len(names) >= 20
    nm = os.popen(f"nm -D --defined-only {ww.LIB_PATH}").read()
    exported = set(re.findall(r"\sT\s(\w+)", nm))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert hasattr(ww.lib(), n)


def test_abi_version_and_status_strings(ww):
    L = ww.lib()
    assert L.ww_abi_version() == 2
    assert L.ww_status_string(0) == b"success"
    assert L.ww_status_string(2) == b"invalid tensor shape"
    assert L.ww_status_string(99) == b"unknown status"


def test_get_int_field_semantics(ww):
    L = ww.lib()
    L.ww_plugin_get_int_field.restype = ctypes.c_int
    v48, v7 = ctypes.c_int32(64), ctypes.c_int32(7)
    names = (ctypes.c_char_p * 3)(b"num_groups", b"max_disp", b"max_disp")
    vals = (ctypes.POINTER(ctypes.c_int32) * 3)(ctypes.pointer(v7), None, ctypes.pointer(v48))
    # first entry with non-null data wins; a null-data entry is skipped (plugin_fields.hpp:17-31)
    assert L.ww_plugin_get_int_field(3, names, vals, b"max_disp", 48) == 64
    assert L.ww_plugin_get_int_field(3, names, vals, b"num_groups", 1) == 7
    assert L.ww_plugin_get_int_field(3, names, vals, b"act", 0) == 0
    assert L.ww_plugin_get_int_field(0, None, None, b"max_disp", 48) == 48


def test_corr_volume_plugin_shapes_and_formats(ww):
    L = ww.lib()
    ins = descs(desc([2, 32, 60, 80]), desc([2, 32, 60, 80]))
    out = Desc()
    assert L.ww_plugin_corr_volume_output_dims(24, 1, 2, ins, ctypes.byref(out)) == 0
    assert out.nb_dims == 4 and list(out.dims[:4]) == [2, 24, 60, 80]
    assert L.ww_plugin_corr_volume_output_dims(24, 8, 2, ins, ctypes.byref(out)) == 0
    assert out.nb_dims == 5 and list(out.dims[:5]) == [2, 8, 24, 60, 80]
    assert L.ww_plugin_corr_volume_output_dims(24, 1, 1, ins, ctypes.byref(out)) == 1
    dt = (ctypes.c_int32 * 2)(1, 1)
    o = ctypes.c_int32(-1)
    assert L.ww_plugin_corr_volume_output_dtype(2, dt, ctypes.byref(o)) == 0 and o.value == 1
    # fp16 only at position 0; others must match position 0; LINEAR only
    f = L.ww_plugin_corr_volume_supports_format
    io = descs(desc([1], 1), desc([1], 1), desc([1], 1))
    assert f(0, io, 2, 1) == 1 and f(1, io, 2, 1) == 1 and f(2, io, 2, 1) == 1
    io32 = descs(desc([1], 0), desc([1], 0), desc([1], 0))
    assert f(0, io32, 2, 1) == 0
    mixed = descs(desc([1], 1), desc([1], 0), desc([1], 1))
    assert f(1, mixed, 2, 1) == 0
    nonlin = descs(desc([1], 1, fmt=1), desc([1], 1), desc([1], 1))
    assert f(0, nonlin, 2, 1) == 0
    assert f(3, io, 2, 1) == 0


def test_corr_volume_enqueue_rejects_before_launch(ww):
    L = ww.lib()
    ptrs = (ctypes.c_void_p * 2)(None, None)
    outs = (ctypes.c_void_p * 1)(None)
    # wrong rank -> 1 (corr_volume.cpp:93)
    assert L.ww_plugin_corr_volume_enqueue(24, 1, descs(desc([2, 32, 60])), ptrs, outs, None) == 1
    # unsupported dtype -> 1 (corr_volume.cpp:109)
    assert L.ww_plugin_corr_volume_enqueue(24, 1, descs(desc([1, 8, 4, 8], dtype=2)), ptrs, outs, None) == 1
    # null pointers -> 1
    assert L.ww_plugin_corr_volume_enqueue(24, 1, descs(desc([1, 8, 4, 8])), ptrs, outs, None) == 1


def test_kernel_entry_points_validate_arguments(ww):
    L = ww.lib()
    fake = ctypes.c_void_p(0x1000)
    # null pointers
    assert L.ww_corr_volume(None, fake, fake, 1, 1, 8, 4, 8, 4, 1, None) == 4
    # group count must divide C
    assert L.ww_corr_volume(fake, fake, fake, 1, 1, 8, 4, 8, 4, 3, None) == 2
    # dtype
    assert L.ww_corr_volume(fake, fake, fake, 7, 1, 8, 4, 8, 4, 1, None) == 3
    # empty work is a no-op success without touching the device
    assert L.ww_corr_volume(fake, fake, fake, 1, 0, 8, 4, 8, 4, 1, None) == 0
    # fused: band must cover the output rows plus a one-row halo
    assert L.ww_corr_cost_stem3d_band(fake, fake, fake, fake, fake, 1, 16, 2, 10, 8, 8, 4, 0,
                                      3, 4, 3, 4, None) == 2
    assert L.ww_corr_cost_stem3d(fake, fake, fake, fake, fake, 1, 16, 3, 10, 8, 8, 4, 0, None) == 2
    assert L.ww_corr_cost_stem3d(fake, fake, fake, fake, fake, 1, 16, 2, 10, 8, 8, 4, 5, None) == 2
    assert L.ww_cost_stem3d(None, fake, fake, fake, 1, 4, 4, 4, 4, 4, 0, None) == 4
    # CorrVolume (G = 1) fused with the 3-stage stem: null, negative size, empty batch
    ws = [fake] * 6
    assert L.ww_corr_cost_stem3d_ref3(None, fake, fake, *ws, 1, 64, 32, 40, 48, None) == 4
    assert L.ww_corr_cost_stem3d_ref3(fake, fake, fake, *ws, 1, 64, -1, 40, 48, None) == 2
    assert L.ww_corr_cost_stem3d_ref3(fake, fake, fake, *ws, 0, 64, 32, 40, 48, None) == 0
    # a correlation over no channels is invalid even when the output is empty
    assert L.ww_corr_cost_stem3d_ref3(fake, fake, fake, *ws, 0, 0, 32, 40, 48, None) == 2
    assert L.ww_corr_cost_stem3d_ref3(fake, fake, fake, *ws, 1, 0, 32, 40, 48, None) == 2
    # disparity regression: null, dtype, mode, D = 0, empty batch
    assert L.ww_disparity_regression(None, fake, 1, 1, 1, 8, 4, 4, 0, None) == 4
    assert L.ww_disparity_regression(fake, fake, 2, 1, 1, 8, 4, 4, 0, None) == 3
    assert L.ww_disparity_regression(fake, fake, 1, 1, 1, 8, 4, 4, 9, None) == 5
    assert L.ww_disparity_regression(fake, fake, 1, 1, 1, 0, 4, 4, 0, None) == 2
    assert L.ww_disparity_regression(fake, fake, 1, 1, 0, 8, 4, 4, 0, None) == 0


def test_cost_stem3d_plugin_shapes(ww):
    L = ww.lib()
    out = Desc()
    seven = descs(desc([1, 1, 48, 32, 40]), *[desc([n]) for n in (108, 4, 432, 4, 108, 1)])
    assert L.ww_plugin_cost_stem3d_output_dims(7, seven, ctypes.byref(out)) == 0
    assert list(out.dims[:5]) == [1, 1, 48, 32, 40]
    three = descs(desc([2, 40, 48, 30, 40]), desc([32, 40, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_cost_stem3d_output_dims(3, three, ctypes.byref(out)) == 0
    assert list(out.dims[:5]) == [2, 32, 48, 30, 40]
    assert L.ww_plugin_cost_stem3d_output_dims(6, seven, ctypes.byref(out)) == 1
    f = L.ww_plugin_cost_stem3d_supports_format
    assert f(0, seven, 7, 1) == 1
    bad = descs(desc([1], 0), *[desc([1]) for _ in range(7)])
    assert f(0, bad, 7, 1) == 0
    ptrs = (ctypes.c_void_p * 7)()
    outs = (ctypes.c_void_p * 1)()
    # rank != 5 -> 1 (cost_stem_3d.cpp:57)
    assert L.ww_plugin_cost_stem3d_enqueue(7, 0, descs(desc([1, 48, 32, 40])), ptrs, outs, None) == 1
    # 3-input form with mismatched Cin -> 1
    bad3 = descs(desc([1, 8, 4, 4, 4]), desc([4, 6, 3, 3, 3]), desc([4]))
    assert L.ww_plugin_cost_stem3d_enqueue(3, 0, bad3, ptrs, outs, None) == 1


def test_corr_cost_stem3d_plugin_shapes(ww):
    L = ww.lib()
    out = Desc()
    ins = descs(desc([1, 320, 120, 160]), desc([1, 320, 120, 160]), desc([32, 40, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_corr_cost_stem3d_output_dims(48, 40, 4, ins, ctypes.byref(out)) == 0
    assert out.nb_dims == 5 and list(out.dims[:5]) == [1, 32, 48, 120, 160]
    ptrs = (ctypes.c_void_p * 4)()
    outs = (ctypes.c_void_p * 1)()
    # weight groups must equal num_groups
    assert L.ww_plugin_corr_cost_stem3d_enqueue(4, 48, 8, 0, ins, ptrs, outs, None) == 1
    ins32 = descs(desc([1, 320, 120, 160], 0), desc([1, 320, 120, 160], 0), desc([32, 40, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_corr_cost_stem3d_enqueue(4, 48, 40, 0, ins32, ptrs, outs, None) == 1
    # right input of another shape, or a bias count that is not Cout
    bad_r = descs(desc([1, 320, 120, 160]), desc([1, 320, 119, 160]), desc([32, 40, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_corr_cost_stem3d_enqueue(4, 48, 40, 0, bad_r, ptrs, outs, None) == 1
    bad_b = descs(desc([1, 320, 120, 160]), desc([1, 320, 120, 160]), desc([32, 40, 3, 3, 3]), desc([16]))
    assert L.ww_plugin_corr_cost_stem3d_enqueue(4, 48, 40, 0, bad_b, ptrs, outs, None) == 1
    # the input count, not the rank of input 2, selects the form
    assert L.ww_plugin_corr_cost_stem3d_enqueue(5, 48, 40, 0, ins, ptrs, outs, None) == 1


def _ref3_descs(w_dims):
    """left, right [1, 64, 32, 40] and the six 3-stage weights with the given shapes."""
    return descs(desc([1, 64, 32, 40]), desc([1, 64, 32, 40]), *[desc(d) for d in w_dims])


def test_corr_cost_stem3d_plugin_eight_inputs_rank5_weights(ww):
    """The reference declares w0 as [4, 1, 3, 3, 3] (rank 5): with 8 inputs the
    plugin must take the 3-stage form whatever the weights' rank, and reject
    weights whose element counts are not 108/4/432/4/108/1."""
    L = ww.lib()
    out = Desc()
    rank5 = [[4, 1, 3, 3, 3], [4], [4, 4, 3, 3, 3], [4], [1, 4, 3, 3, 3], [1]]
    ins = _ref3_descs(rank5)
    assert L.ww_plugin_corr_cost_stem3d_output_dims(48, 1, 8, ins, ctypes.byref(out)) == 0
    assert list(out.dims[:5]) == [1, 1, 48, 32, 40]
    ptrs = (ctypes.c_void_p * 8)()
    outs = (ctypes.c_void_p * 1)()
    # correct counts reach the kernel entry point, which rejects the null pointers (1)
    assert L.ww_plugin_corr_cost_stem3d_enqueue(8, 48, 1, 0, ins, ptrs, outs, None) == 1
    # an empty batch with valid counts is a no-op success: the 3-stage entry
    # point was taken (the generic form would have read w0 as Cout = 4, G = 1)
    empty = _ref3_descs(rank5)
    empty[0].dims[0] = 0
    empty[1].dims[0] = 0
    fake = (ctypes.c_void_p * 8)(*([0x1000] * 8))
    fake_out = (ctypes.c_void_p * 1)(0x1000)
    assert L.ww_plugin_corr_cost_stem3d_enqueue(8, 48, 1, 0, empty, fake, fake_out, None) == 0
    # a wrong element count in any weight or bias is rejected before any launch
    for i in range(6):
        bad = [list(d) for d in rank5]
        bad[i][0] += 1
        assert L.ww_plugin_corr_cost_stem3d_enqueue(8, 48, 1, 0, _ref3_descs(bad), fake, fake_out, None) == 1
    # num_groups > 1 has no 3-stage form
    assert L.ww_plugin_corr_cost_stem3d_enqueue(8, 48, 2, 0, empty, fake, fake_out, None) == 1


def test_fold_bn_matches_oracle(ww, orc):
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((8, 5, 3, 3, 3)) * 0.05).astype(np.float32)
    s = rng.uniform(0.5, 1.5, 8).astype(np.float32)
    b = (rng.standard_normal(8) * 0.1).astype(np.float32)
    w1, b1 = ww.fold_bn(w, s, b)
    w2, b2 = orc.fold_bn(w, s, b)
    assert np.array_equal(w1.view(np.uint16), w2.view(np.uint16))
    assert np.array_equal(b1.view(np.uint16), b2.view(np.uint16))


def test_configs_fold_matches_library(ww):
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[2].scaled(H=2, W=8)
    x = make_inputs(cfg)
    w16, b16 = ww.fold_bn(x["w_raw"], x["scale"], x["bias_raw"])
    assert np.array_equal(w16.view(np.uint16), x["w"].view(np.uint16))
    assert np.array_equal(b16.view(np.uint16), x["b"].view(np.uint16))


def test_fused_limits_are_reported_and_enforced_at_build_time(ww):
    """The limits in the header: Cout <= 32, G <= 56 and shared memory for a
    16-disparity band (wide groups: C / G = 32 with G = 56 does not fit); any
    D (ranges one launch cannot hold run as disparity bands); the plugin's
    output_dims refuses a shape outside them, so an engine build fails
    instead of the enqueue."""
    L = ww.lib()
    for C, G, D, Cout in ((320, 40, 48, 32), (96, 8, 64, 16), (256, 32, 48, 32), (64, 16, 32, 16),
                          (64, 8, 80, 32), (32, 8, 160, 16), (448, 56, 48, 16), (320, 40, 48, 32),
                          (64, 8, 81, 32), (32, 8, 161, 16), (64, 8, 192, 32), (96, 8, 400, 16)):
        assert L.ww_corr_cost_stem3d_supported(C, G, D, Cout) == 0, (C, G, D, Cout)
    assert L.ww_corr_cost_stem3d_supported(512, 64, 48, 16) == 5  # G past 56
    assert L.ww_corr_cost_stem3d_supported(384, 48, 48, 32) == 0  # 16-disparity bands fit shared memory
    assert L.ww_corr_cost_stem3d_supported(1792, 56, 48, 32) == 5  # 32-channel groups: staging past shared memory
    assert L.ww_corr_cost_stem3d_supported(64, 8, 48, 33) == 5    # Cout past 32
    assert L.ww_corr_cost_stem3d_supported(64, 6, 48, 32) == 2    # G does not divide C
    assert L.ww_cost_stem3d_supported(40, 48, 32) == 0
    assert L.ww_cost_stem3d_supported(40, 96, 32) == 0   # two disparity bands
    assert L.ww_cost_stem3d_supported(64, 48, 32) == 5   # Cin past 56
    out = Desc()
    ok = descs(desc([1, 64, 20, 40]), desc([1, 64, 20, 40]), desc([32, 8, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_corr_cost_stem3d_output_dims(80, 8, 4, ok, ctypes.byref(out)) == 0
    assert L.ww_plugin_corr_cost_stem3d_output_dims(192, 8, 4, ok, ctypes.byref(out)) == 0  # disparity bands
    wide = descs(desc([1, 56 * 32, 20, 40]), desc([1, 56 * 32, 20, 40]), desc([32, 56, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_corr_cost_stem3d_output_dims(48, 56, 4, wide, ctypes.byref(out)) == 1  # past shared memory
    assert L.ww_plugin_corr_cost_stem3d_output_dims(48, 4, 4, ok, ctypes.byref(out)) == 1   # weights' G != num_groups
    big = descs(desc([1, 64, 20, 40, 96]), desc([32, 64, 3, 3, 3]), desc([32]))
    assert L.ww_plugin_cost_stem3d_output_dims(3, big, ctypes.byref(out)) == 1


def test_fused_corr_engine_knob(ww):
    """The fused op's correlation engine is a process-wide setting: tensor
    cores by default, CUDA cores on request; unknown values are refused and
    leave the setting alone."""
    assert ww.fused_corr_engine() == ww.CORR_ENGINE_TENSOR
    assert ww.set_fused_corr_engine(ww.CORR_ENGINE_CUDA_CORES) == ww.CORR_ENGINE_TENSOR
    try:
        assert ww.fused_corr_engine() == ww.CORR_ENGINE_CUDA_CORES
        assert ww.lib().ww_set_fused_corr_engine(7) == 2
        assert ww.fused_corr_engine() == ww.CORR_ENGINE_CUDA_CORES
        with pytest.raises(ww.WWError):
            ww.set_fused_corr_engine(-1)
    finally:
        assert ww.set_fused_corr_engine(ww.CORR_ENGINE_TENSOR) == ww.CORR_ENGINE_CUDA_CORES
    assert ww.fused_corr_engine() == ww.CORR_ENGINE_TENSOR
