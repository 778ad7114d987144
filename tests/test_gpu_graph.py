"""Every entry point can be captured in a CUDA graph and replayed (no
allocation, no synchronisation, no host-side state that changes between
calls): a serving loop can replay the whole front end as one graph launch.
Replays must reproduce the eager results bit for bit."""
import pytest

pytestmark = pytest.mark.gpu


def test_front_end_captures_and_replays():
    import torch
    import whirlwind_trt_plugins_b200 as ww
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs_torch
    cfg = CONFIGS[5]
    x = make_inputs_torch(cfg, torch.device("cuda", 0))
    L, R, w, b = x["left"], x["right"], x["w"], x["b"]
    B, C, H, W = L.shape
    g = torch.Generator(device="cuda").manual_seed(2)
    frames = torch.randint(0, 256, (2, 96 * 3 // 2, 128), generator=g, device="cuda", dtype=torch.uint8)
    vol1 = torch.randn((1, 1, 16, 12, 20), generator=g, device="cuda").half()
    agg = torch.randn((2, 24, 10, 16), generator=g, device="cuda").half()
    ws = [(torch.randn((n,), generator=g, device="cuda") * 0.2).half() for n in (108, 4, 432, 4, 108, 1)]

    outs = {
        "fused": torch.empty((B, cfg.Cout, cfg.D, H, W), dtype=torch.float16, device="cuda"),
        "corr": torch.empty((B, cfg.G, cfg.D, H, W), dtype=torch.float16, device="cuda"),
        "nv12": torch.empty((2, 3, 60, 80), dtype=torch.float16, device="cuda"),
        "stem3": torch.empty_like(vol1),
        "disp": torch.empty((2, 1, 10, 16), dtype=torch.float16, device="cuda"),
        "corr_stem3": torch.empty((B, 1, cfg.D, H, W), dtype=torch.float16, device="cuda"),
    }

    def run():
        ww.corr_cost_stem3d(L, R, w, b, cfg.D, cfg.G, act=cfg.act, out=outs["fused"])
        ww.corr_volume(L, R, cfg.D, cfg.G, out=outs["corr"])
        ww.nv12_decode(frames, 60, 80, out=outs["nv12"])
        ww.cost_stem3d_ref3(vol1, *ws, out=outs["stem3"])
        ww.disparity_regression(agg, ww.DISP_SOFTARGMIN, out=outs["disp"])
        ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=cfg.D, out=outs["corr_stem3"])

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up outside the capture (first-use host state)
        run()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    eager = {k: v.clone() for k, v in outs.items()}
    for v in outs.values():
        v.zero_()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    for k in outs:
        assert torch.equal(outs[k], eager[k]), k
    assert ww.device_error() == 0
    del graph
