"""The reference's own CUDA kernels, rebuilt for sm_100a (oracle/_ref), timed
beside this library's kernels on the same B200 and the same inputs: the
baseline the reference would give on this hardware.

* Group-wise correlation: the reference has no grouped kernel, so its
  composition is one launchCorrVolume<__half> per (b, g) (B = 1, C = C/G).
  Compared with ww_corr_volume (one launch, bit-identical output) and with
  the fused ww_corr_cost_stem3d, which also runs the G -> Cout stem the
  reference has no kernel for.
* The reference CostStem3D at its native shape [1, 1, 48, 32, 40] against
  ww_cost_stem3d_ref3 (bit-identical output), and the reference's
  CorrVolume -> CostStem3D pair at that shape against the fused
  ww_corr_cost_stem3d_ref3 (bit-identical output).
* The reference Nv12Decode (one launch per frame, as its launcher takes one
  image) on 8 720p frames -> 224 x 288 fp16 against one ww_nv12_decode call
  (bit-identical output).

Two figures per arm, both with CUDA events on the launching stream:
* device time: `inner` calls captured in one CUDA graph, the graph replayed
  `reps` times, the median replay divided by `inner` (what the GPU spends per
  call, host launch cost removed; inputs stay in L2 for both arms);
* call time: one eager call between two events, median of 50 after 10
  warm-ups (includes the host's launch path: ctypes for the reference,
  the Python API for this library).
The table is printed (pytest -s) and, when WW_REF_SPEED_OUT names a file,
written there as JSON.  The assertions check the outputs and that the library
is not slower than the reference composition on the device."""
import json
import os
import statistics

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _device_us(torch, fn, inner=20, reps=20):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # first-use host state outside the capture
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(inner):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3 / inner)
    del graph
    return statistics.median(ts)


def _median_us(torch, fn, warmup=10, reps=50):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    return statistics.median(ts)


@pytest.fixture(scope="module")
def env():
    import torch
    import oracle
    import whirlwind_trt_plugins_b200 as ww
    ref = oracle.ref_lib()
    return torch, ww, ref


RESULTS = {}


def _save():
    out = os.environ.get("WW_REF_SPEED_OUT")
    if out:
        with open(out, "w") as f:
            json.dump(RESULTS, f, indent=1)


@pytest.mark.parametrize("cfg_id", [2, 3, 5, 4])
def test_grouped_correlation_vs_reference_kernels(env, cfg_id):
    torch, ww, ref = env
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs_torch
    cfg = CONFIGS[cfg_id]
    x = make_inputs_torch(cfg, torch.device("cuda", 0))
    L, R = x["left"], x["right"]
    B, C, H, W = L.shape
    D, G = cfg.D, cfg.G
    vol_ref = torch.empty((B, G, D, H, W), dtype=torch.float16, device="cuda")
    vol = torch.empty_like(vol_ref)
    out = torch.empty((B, cfg.Cout, D, H, W), dtype=torch.float16, device="cuda")
    def run_ref():
        s = torch.cuda.current_stream().cuda_stream
        assert ref.wwref_corr_volume_grouped_f16(L.data_ptr(), R.data_ptr(), vol_ref.data_ptr(), B, C, H, W, D, G,
                                                 s) == 0

    def run_ours():
        ww.corr_volume(L, R, D, G, out=vol)

    def run_fused():
        ww.corr_cost_stem3d(L, R, x["w"], x["b"], D, G, act=cfg.act, out=out)

    inner, reps = (2, 5) if cfg_id == 4 else (10, 20)
    t_ref = _device_us(torch, run_ref, inner, reps)
    t_ours = _device_us(torch, run_ours, inner, reps)
    t_fused = _device_us(torch, run_fused, inner, reps)
    c_ref = _median_us(torch, run_ref, reps=10 if cfg_id == 4 else 50)
    c_ours = _median_us(torch, run_ours, reps=10 if cfg_id == 4 else 50)
    c_fused = _median_us(torch, run_fused, reps=10 if cfg_id == 4 else 50)
    torch.cuda.synchronize()
    assert torch.equal(vol, vol_ref)
    vox = B * D * H * W
    RESULTS[f"corr_c{cfg_id}"] = {
        "reference_per_bg_device_us": t_ref, "ww_corr_volume_device_us": t_ours,
        "ww_corr_cost_stem3d_device_us": t_fused,
        "reference_per_bg_call_us": c_ref, "ww_corr_volume_call_us": c_ours, "ww_corr_cost_stem3d_call_us": c_fused,
        "reference_launches": B * G, "voxels": vox,
        "reference_vox_per_s": vox / (t_ref * 1e-6), "fused_vox_per_s": vox / (t_fused * 1e-6)}
    print(f"\nconfig {cfg_id} device: reference CorrVolume x{B * G} launches {t_ref:9.1f} us | "
          f"ww_corr_volume {t_ours:8.1f} us | fused corr+stem {t_fused:8.1f} us;  per call: "
          f"{c_ref:.1f} | {c_ours:.1f} | {c_fused:.1f} us")
    _save()
    assert t_ours < t_ref


def test_native_stem_vs_reference_kernel(env):
    torch, ww, ref = env
    g = torch.Generator(device="cuda").manual_seed(7)
    vol = torch.randn((1, 1, 48, 32, 40), generator=g, device="cuda").half()
    ws = [(torch.randn((n,), generator=g, device="cuda") * s).half()
          for n, s in ((108, 0.2), (4, 0.1), (432, 0.2), (4, 0.1), (108, 0.2), (1, 0.1))]
    o_ref = torch.empty_like(vol)
    o = torch.empty_like(vol)
    def run_ref():
        s = torch.cuda.current_stream().cuda_stream
        assert ref.wwref_cost_stem3d(vol.data_ptr(), o_ref.data_ptr(), *[w.data_ptr() for w in ws], 1, 48, 32, 40,
                                     s) == 0

    def run_ours():
        ww.cost_stem3d_ref3(vol, *ws, out=o)

    t_ref = _device_us(torch, run_ref)
    t_ours = _device_us(torch, run_ours)
    c_ref = _median_us(torch, run_ref)
    c_ours = _median_us(torch, run_ours)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    RESULTS["stem3_native"] = {"reference_device_us": t_ref, "ww_cost_stem3d_ref3_device_us": t_ours,
                               "reference_call_us": c_ref, "ww_cost_stem3d_ref3_call_us": c_ours}
    print(f"\nnative CostStem3D [1,1,48,32,40] device: reference {t_ref:.2f} us | ww_cost_stem3d_ref3 {t_ours:.2f} us;"
          f"  per call: {c_ref:.2f} | {c_ours:.2f} us")
    _save()
    assert t_ours < t_ref


def test_native_corr_stem_vs_reference_pair(env):
    """The reference's own pair at its native shape (CorrVolume, then the
    3-stage CostStem3D on [1, 1, 48, 32, 40]; C = 64 features) against the
    fused ww_corr_cost_stem3d_ref3 and against this library's two-call pair."""
    torch, ww, ref = env
    g = torch.Generator(device="cuda").manual_seed(11)
    B, C, H, W, D = 1, 64, 32, 40, 48
    L = torch.randn((B, C, H, W), generator=g, device="cuda").half()
    R = torch.randn((B, C, H, W), generator=g, device="cuda").half()
    ws = [(torch.randn((n,), generator=g, device="cuda") * s).half()
          for n, s in ((108, 0.2), (4, 0.1), (432, 0.2), (4, 0.1), (108, 0.2), (1, 0.1))]
    vol_ref = torch.empty((B, D, H, W), dtype=torch.float16, device="cuda")
    o_ref = torch.empty((B, 1, D, H, W), dtype=torch.float16, device="cuda")
    vol = torch.empty((B, D, H, W), dtype=torch.float16, device="cuda")
    o_pair = torch.empty_like(o_ref)
    o = torch.empty_like(o_ref)

    def run_ref():
        s = torch.cuda.current_stream().cuda_stream
        assert ref.wwref_corr_volume_f16(L.data_ptr(), R.data_ptr(), vol_ref.data_ptr(), B, C, H, W, D, s) == 0
        assert ref.wwref_cost_stem3d(vol_ref.data_ptr(), o_ref.data_ptr(), *[w.data_ptr() for w in ws], B, D, H, W,
                                     s) == 0

    def run_pair():
        ww.corr_volume(L, R, D, out=vol)
        ww.cost_stem3d_ref3(vol.unsqueeze(1), *ws, out=o_pair)

    def run_fused():
        ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=D, out=o)

    t_ref, t_pair, t_fused = _device_us(torch, run_ref), _device_us(torch, run_pair), _device_us(torch, run_fused)
    c_ref, c_pair, c_fused = _median_us(torch, run_ref), _median_us(torch, run_pair), _median_us(torch, run_fused)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref) and torch.equal(o_pair, o_ref)
    RESULTS["corr_stem3_native"] = {"reference_pair_device_us": t_ref, "ww_pair_device_us": t_pair,
                                    "ww_fused_device_us": t_fused, "reference_pair_call_us": c_ref,
                                    "ww_pair_call_us": c_pair, "ww_fused_call_us": c_fused}
    print(f"\nnative CorrVolume -> CostStem3D (C = 64) device: reference pair {t_ref:.2f} us | ww pair {t_pair:.2f} us"
          f" | ww fused {t_fused:.2f} us;  per call: {c_ref:.2f} | {c_pair:.2f} | {c_fused:.2f} us")
    _save()
    assert t_fused < t_ref


def test_nv12_decode_vs_reference_kernel(env):
    torch, ww, ref = env
    B, H, W, OH, OW = 8, 720, 1280, 224, 288
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randint(0, 256, (B, H * 3 // 2, W), generator=g, device="cuda", dtype=torch.uint8)
    o_ref = torch.empty((B, 3, OH, OW), dtype=torch.float16, device="cuda")
    o = torch.empty_like(o_ref)
    frame_in, frame_out = H * 3 // 2 * W, 3 * OH * OW * 2

    def run_ref():
        s = torch.cuda.current_stream().cuda_stream
        for b in range(B):
            assert ref.wwref_nv12_decode_f16(x.data_ptr() + b * frame_in, o_ref.data_ptr() + b * frame_out, H, W,
                                             OH, OW, s) == 0

    def run_ours():
        ww.nv12_decode(x, OH, OW, out=o)

    t_ref = _device_us(torch, run_ref)
    t_ours = _device_us(torch, run_ours)
    c_ref = _median_us(torch, run_ref)
    c_ours = _median_us(torch, run_ours)
    torch.cuda.synchronize()
    assert torch.equal(o.view(torch.int16), o_ref.view(torch.int16))
    RESULTS["nv12_b8_720p"] = {"reference_device_us": t_ref, "reference_launches": B, "ww_nv12_decode_device_us": t_ours,
                               "reference_call_us": c_ref, "ww_nv12_decode_call_us": c_ours}
    print(f"\nNv12Decode 8 x 720p -> 224x288 device: reference x{B} launches {t_ref:.2f} us | ww_nv12_decode "
          f"{t_ours:.2f} us;  per call: {c_ref:.2f} | {c_ours:.2f} us")
    _save()
    assert t_ours < t_ref
