"""GPU tests of the multi-device driver ww_corr_cost_stem3d_multi through
the C ABI: batch split and row bands (halo rows copied between the parts'
band buffers) stitch to the single-call output bit for bit -- with several
parts on one device (always) and across two devices (when present) -- and
a halo copy made to fail on the host surfaces as a non-zero status."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


@pytest.fixture(scope="module")
def ww():
    import whirlwind_trt_plugins_b200 as ww
    return ww


def _inputs(torch, cfg, dev):
    from whirlwind_trt_plugins_b200.configs import make_inputs
    x = make_inputs(cfg)
    return {k: torch.from_numpy(np.ascontiguousarray(x[k])).to(dev) for k in ("left", "right", "w", "b")}


def _bands(torch, ww, x, H, devices):
    """Each part's band buffer: its own rows copied in, halo rows left zero
    (the driver must fill them)."""
    n = len(devices)
    Ls, Rs, ws, bs = [], [], [], []
    for k, d in enumerate(devices):
        r0, r1, i0, i1 = ww.multi_split(n, H, k)
        dev = torch.device("cuda", d)
        L = torch.zeros_like(x["left"][:, :, i0:i1]).to(dev)
        R = torch.zeros_like(x["right"][:, :, i0:i1]).to(dev)
        L[:, :, r0 - i0:r1 - i0].copy_(x["left"][:, :, r0:r1])
        R[:, :, r0 - i0:r1 - i0].copy_(x["right"][:, :, r0:r1])
        Ls.append(L)
        Rs.append(R)
        ws.append(x["w"].to(dev))
        bs.append(x["b"].to(dev))
    return Ls, Rs, ws, bs


def _rows_case(torch, ww, devices, n_streams_distinct=True):
    from whirlwind_trt_plugins_b200.configs import CONFIGS
    cfg = CONFIGS[3].scaled(B=1, H=23, W=40)
    x = _inputs(torch, cfg, torch.device("cuda", devices[0]))
    full = ww.corr_cost_stem3d(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G)
    Ls, Rs, ws, bs = _bands(torch, ww, x, cfg.H, devices)
    streams = [torch.cuda.Stream(torch.device("cuda", d)) for d in devices]
    outs = ww.corr_cost_stem3d_multi(Ls, Rs, ws, bs, cfg.D, cfg.G, ww.MULTI_ROWS, H=cfg.H, streams=streams)
    for d in set(devices):
        torch.cuda.synchronize(d)
    stitched = torch.cat([o.to(full.device) for o in outs], dim=3)
    assert torch.equal(stitched.view(torch.int16), full.view(torch.int16))
    # the driver filled the halo rows from the neighbours
    for k in range(len(devices)):
        r0, r1, i0, i1 = ww.multi_split(len(devices), cfg.H, k)
        assert torch.equal(Ls[k].to(full.device), x["left"][:, :, i0:i1])
    assert ww.device_error() == 0


@pytest.mark.parametrize("parts", [2, 3])
def test_rows_parts_on_one_device_stitch(ww, torch, parts):
    _rows_case(torch, ww, [0] * parts)


def test_batch_parts_on_one_device(ww, torch):
    from whirlwind_trt_plugins_b200.configs import CONFIGS
    cfg = CONFIGS[5].scaled(B=5, H=12, W=32)
    x = _inputs(torch, cfg, torch.device("cuda", 0))
    full = ww.corr_cost_stem3d(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G)
    n = 3
    from whirlwind_trt_plugins_b200.shard import split_even
    parts = [split_even(cfg.B, n, k) for k in range(n)]
    Ls = [x["left"][b0:b1].contiguous() for b0, b1 in parts]
    Rs = [x["right"][b0:b1].contiguous() for b0, b1 in parts]
    outs = ww.corr_cost_stem3d_multi(Ls, Rs, [x["w"]] * n, [x["b"]] * n, cfg.D, cfg.G, ww.MULTI_BATCH)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(outs, 0).view(torch.int16), full.view(torch.int16))


def test_injected_copy_failure_returns_error(ww, torch):
    """The second halo copy is made to fail on the host: the call reports a
    launch error (status 1) instead of computing with a missing halo row, and
    the next call, without injection, is correct again."""
    from whirlwind_trt_plugins_b200.configs import CONFIGS
    cfg = CONFIGS[3].scaled(B=1, H=10, W=16)
    x = _inputs(torch, cfg, torch.device("cuda", 0))
    Ls, Rs, ws, bs = _bands(torch, ww, x, cfg.H, [0, 0])
    assert ww.lib().ww_multi_inject_copy_failure(1) == 0
    with pytest.raises(ww.WWError) as ei:
        ww.corr_cost_stem3d_multi(Ls, Rs, ws, bs, cfg.D, cfg.G, ww.MULTI_ROWS, H=cfg.H)
    assert ei.value.status == 1
    torch.cuda.synchronize()
    _rows_case(torch, ww, [0, 0])


@pytest.mark.skipif("__import__('torch').cuda.device_count() < 2")
def test_rows_and_batch_across_two_devices(ww, torch):
    _rows_case(torch, ww, [0, 1])
    from whirlwind_trt_plugins_b200.configs import CONFIGS
    cfg = CONFIGS[5].scaled(B=4, H=12, W=32)
    x = _inputs(torch, cfg, torch.device("cuda", 0))
    full = ww.corr_cost_stem3d(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G)
    d1 = torch.device("cuda", 1)
    outs = ww.corr_cost_stem3d_multi([x["left"][:2].contiguous(), x["left"][2:].contiguous().to(d1)],
                                     [x["right"][:2].contiguous(), x["right"][2:].contiguous().to(d1)],
                                     [x["w"], x["w"].to(d1)], [x["b"], x["b"].to(d1)], cfg.D, cfg.G,
                                     ww.MULTI_BATCH)
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    assert torch.equal(torch.cat([outs[0], outs[1].to(full.device)], 0).view(torch.int16), full.view(torch.int16))
