"""GPU parity of the stems and of the fused front end.

* ww_cost_stem3d_ref3 (reference 7-input CostStem3D): bit-identical to the
  reference kernel (golden fixtures, live oracle/_ref at B = 1) and to the
  oracle for B > 1 (the reference kernel only writes batch 0).
* ww_cost_stem3d / ww_corr_cost_stem3d (tensor cores, fp32 accumulation in a
  different order than the oracle): |out - oracle| <= 2e-2 absolute (fp16
  tolerance of the north-star contract; values are already normalised by the
  channel count in the correlation).  The fused kernel's correlation runs on
  the tensor cores, so its volume can differ from CorrVolume's by one fp16
  ulp in rare values.
"""
import numpy as np
import pytest

from conftest import golden_files, load_golden

pytestmark = pytest.mark.gpu

ATOL_F16 = 2e-2


@pytest.fixture(scope="module")
def torch():
    import torch
    return torch


@pytest.fixture(scope="module")
def ww():
    import whirlwind_trt_plugins_b200 as ww
    return ww


def _t(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.device("cuda:0"))


def _u16(a):
    return np.ascontiguousarray(a).view(np.uint16)


# ------------------------------------------------------------------ ref3 stem

@pytest.mark.parametrize("name", [f for f in golden_files() if "stem3" in f])
def test_ref3_matches_reference_golden(ww, torch, name):
    g = load_golden(name)
    ws = [_t(torch, g[k]) for k in ("w0", "b0", "w1", "b1", "w2", "b2")]
    out = ww.cost_stem3d_ref3(_t(torch, g["vol"]), *ws).cpu().numpy()
    assert np.array_equal(_u16(out), _u16(g["out"]))


def _ref3_weights(rng):
    return [(rng.standard_normal(n) * s).astype(np.float16) for n, s in
            ((108, 0.3), (4, 0.2), (432, 0.2), (4, 0.2), (108, 0.2), (1, 0.2))]


@pytest.mark.parametrize("shape", [(1, 48, 32, 40), (3, 13, 9, 11), (2, 1, 1, 1), (1, 20, 33, 65)])
def test_ref3_matches_oracle_all_batches(ww, torch, orc, shape):
    B, D, H, W = shape
    rng = np.random.default_rng(D * 31 + W)
    x = (rng.standard_normal((B, 1, D, H, W)) * 2).astype(np.float16)
    ws = _ref3_weights(rng)
    out = ww.cost_stem3d_ref3(_t(torch, x), *[_t(torch, w) for w in ws]).cpu().numpy()
    ref = orc.stem_ref3(x, *ws)
    assert np.array_equal(_u16(out), _u16(ref))


def test_ref3_matches_reference_live_b1(ww, torch, orc):
    import os
    if not os.path.exists(orc.REF_SO):
        pytest.skip("oracle/_ref/libww_ref.so not built")
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((1, 1, 48, 32, 40)) * 2).astype(np.float16)
    ws = _ref3_weights(rng)
    tx, tws = _t(torch, x), [_t(torch, w) for w in ws]
    ref = torch.empty_like(tx)
    rc = orc.ref_lib().wwref_cost_stem3d(tx.data_ptr(), ref.data_ptr(), *[w.data_ptr() for w in tws], 1, 48, 32, 40,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    out = ww.cost_stem3d_ref3(tx, *tws)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


# ------------------------------------------------------ generalised stem (TC)

@pytest.mark.parametrize("case", [
    dict(B=1, Cin=40, Cout=32, D=48, H=5, W=16),
    dict(B=2, Cin=8, Cout=16, D=64, H=4, W=24),
    dict(B=1, Cin=32, Cout=32, D=48, H=3, W=8),
    dict(B=1, Cin=16, Cout=16, D=32, H=6, W=13),     # ragged W
    dict(B=1, Cin=5, Cout=7, D=20, H=4, W=9),        # padded channels, Cout, D
    dict(B=1, Cin=24, Cout=20, D=16, H=1, W=8),      # H = 1
    dict(B=1, Cin=12, Cout=32, D=80, H=3, W=17),     # five M-blocks along D
])
@pytest.mark.parametrize("act", [0, 1])
def test_stem_tc_matches_oracle(ww, torch, orc, case, act):
    B, Cin, Cout, D, H, W = (case[k] for k in ("B", "Cin", "Cout", "D", "H", "W"))
    rng = np.random.default_rng(Cin * 100 + Cout + D)
    vol = (rng.standard_normal((B, Cin, D, H, W)) * 0.5).astype(np.float16)
    w = (rng.standard_normal((Cout, Cin, 3, 3, 3)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(Cout) * 0.1).astype(np.float16)
    out = ww.cost_stem3d(_t(torch, vol), _t(torch, w), _t(torch, b), act=act).cpu().numpy().astype(np.float32)
    ref = orc.stem(vol, w, b, act=act, acc_mode=orc.ACC_F64).astype(np.float32)
    err = np.abs(out - ref).max()
    assert err <= ATOL_F16, f"max abs err {err}"
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("case", [
    dict(B=2, Cin=40, Cout=32, D=48, H=6, W=40),
    dict(B=1, Cin=12, Cout=16, D=64, H=5, W=32),     # a partial octet
    dict(B=1, Cin=8, Cout=16, D=200, H=3, W=16),     # disparity bands
    dict(B=1, Cin=24, Cout=16, D=200, H=3, W=16),    # 160-plane band: no room for the staging ring
])
def test_stem_volume_gather_paths_agree(ww, torch, case):
    """The volume form's gathers -- TMA-staged boxes or, where shared memory
    has no room for the staging ring (the 160-plane band of the last case),
    16-byte loads, both with a register transpose (W % 8 == 0, 16-byte
    aligned volume), and 2-byte loads (any other volume) -- fill the same
    volume rows, so the outputs are equal bit for bit; the 2-byte path is
    reached by passing a volume that starts one element into its storage."""
    B, Cin, Cout, D, H, W = (case[k] for k in ("B", "Cin", "Cout", "D", "H", "W"))
    g = torch.Generator().manual_seed(Cin + D)
    n = B * Cin * D * H * W
    flat = (torch.randn(n + 8, generator=g) * 0.5).half().cuda()
    shifted = flat[1:n + 1].view(B, Cin, D, H, W)
    aligned = shifted.clone()
    assert aligned.data_ptr() % 16 == 0 and shifted.data_ptr() % 16 != 0
    w = (torch.randn(Cout, Cin, 3, 3, 3, generator=g) * 0.05).half().cuda()
    b = (torch.randn(Cout, generator=g) * 0.1).half().cuda()
    assert torch.equal(ww.cost_stem3d(aligned, w, b), ww.cost_stem3d(shifted, w, b))
    assert ww.device_error() == 0


# ------------------------------------------------------------ fused front end

def _fused(ww, torch, x, cfg, act=0):
    return ww.corr_cost_stem3d(_t(torch, x["left"]), _t(torch, x["right"]), _t(torch, x["w"]), _t(torch, x["b"]),
                               cfg.D, cfg.G, act=act)


@pytest.mark.parametrize("cfg_id", [2, 3, 4, 5])
def test_fused_configs_match_oracle(ww, torch, orc, cfg_id):
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[cfg_id]
    cfg = cfg.scaled(B=min(cfg.B, 2), H=min(cfg.H, 10), W=min(cfg.W, 64))
    x = make_inputs(cfg)
    out = _fused(ww, torch, x, cfg).cpu().numpy().astype(np.float32)
    ref = orc.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, acc_mode=orc.ACC_F64)
    err = np.abs(out - ref.astype(np.float32)).max()
    assert err <= ATOL_F16, f"max abs err {err}"


def test_fused_matches_unfused_composition(ww, torch, orc):
    """corr -> stem through HBM and the fused kernel agree: the fused kernel's
    correlation runs on the tensor cores (its fp32 sums are added in another
    order than CorrVolume's sequential fma chain), so a volume value may differ
    by one fp16 ulp; the stem outputs stay within the fp16 tolerance and
    almost all are bit-identical."""
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[2].scaled(H=9, W=40)
    x = make_inputs(cfg)
    tl, tr, tw, tb = (_t(torch, x[k]) for k in ("left", "right", "w", "b"))
    fused = ww.corr_cost_stem3d(tl, tr, tw, tb, cfg.D, cfg.G)
    vol = ww.corr_volume(tl, tr, cfg.D, cfg.G)
    unfused = ww.cost_stem3d(vol, tw, tb)
    diff = (fused.float() - unfused.float()).abs()
    assert float(diff.max()) <= ATOL_F16
    assert float((diff == 0).float().mean()) >= 0.99
    ref_vol = orc.corr_f16(x["left"], x["right"], cfg.D, cfg.G)
    assert np.array_equal(_u16(vol.cpu().numpy()), _u16(ref_vol))


@pytest.fixture
def cuda_core_engine(ww):
    prev = ww.set_fused_corr_engine(ww.CORR_ENGINE_CUDA_CORES)
    yield
    ww.set_fused_corr_engine(prev)


@pytest.mark.parametrize("shape", [
    # (B, C, G, H, W, D, Cout): Cg = 8, 4, 12, 16 (unrolled channel loops) and
    # 32, 20, 3, 1 (run-time loop); odd W (scalar staging), D < 8, lone octets
    (1, 320, 40, 6, 40, 48, 32),
    (2, 64, 16, 5, 32, 32, 16),
    (1, 96, 8, 4, 48, 64, 16),
    (1, 64, 4, 3, 24, 40, 16),
    (1, 64, 2, 5, 24, 24, 16),
    (1, 40, 2, 4, 20, 20, 8),
    (2, 24, 8, 6, 33, 13, 32),
    (1, 16, 16, 3, 16, 70, 16),
    (1, 48, 3, 5, 16, 7, 4),
])
def test_cuda_core_engine_equals_unfused_composition(ww, torch, cuda_core_engine, shape):
    """With the CUDA-core correlation engine the fused volume is
    ww_corr_volume's bit for bit (channel-order fp32 fma chain, the same
    scale rule), and the stem is the same kernel in both modes, so the fused
    output equals corr_volume -> cost_stem3d exactly."""
    from whirlwind_trt_plugins_b200.configs import FrontEnd, make_inputs
    B, C, G, H, W, D, Cout = shape
    cfg = FrontEnd("edge", B=B, C=C, G=G, H=H, W=W, D=D, Cout=Cout)
    x = make_inputs(cfg, seed=C + W + D + 1)
    tl, tr, tw, tb = (_t(torch, x[k]) for k in ("left", "right", "w", "b"))
    fused = ww.corr_cost_stem3d(tl, tr, tw, tb, cfg.D, cfg.G)
    unfused = ww.cost_stem3d(ww.corr_volume(tl, tr, cfg.D, cfg.G), tw, tb)
    assert torch.equal(fused, unfused)
    assert ww.device_error() == 0


@pytest.mark.parametrize("cfg_id,B", [(2, 1), (3, 1), (4, 1), (5, 2)])
def test_cuda_core_engine_full_size(ww, torch, orc, cuda_core_engine, cfg_id, B):
    """The benchmark configurations at full H x W x D through the CUDA-core
    engine: bit-identical to the unfused composition and within the fp16
    tolerance of the oracle."""
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[cfg_id].scaled(B=B)
    x = make_inputs(cfg)
    t = {k: _t(torch, x[k]) for k in ("left", "right", "w", "b")}
    fused = ww.corr_cost_stem3d(t["left"], t["right"], t["w"], t["b"], cfg.D, cfg.G, act=cfg.act)
    unfused = ww.cost_stem3d(ww.corr_volume(t["left"], t["right"], cfg.D, cfg.G), t["w"], t["b"], act=cfg.act)
    assert torch.equal(fused, unfused)
    ref = orc.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, act=cfg.act,
                        acc_mode=orc.ACC_F32_SEQ).astype(np.float32)
    assert float(np.abs(fused.cpu().numpy().astype(np.float32) - ref).max()) <= ATOL_F16
    assert ww.device_error() == 0


@pytest.mark.parametrize("shape", [
    # (B, C, G, H, W, D, Cout): disparity ranges that run as several bands
    (1, 64, 8, 5, 40, 96, 32),    # bands of 80 + 16
    (1, 32, 4, 4, 48, 192, 16),   # 160 + 32 (two column tiles per CTA)
    (2, 64, 8, 3, 24, 200, 16),   # 160 + 40: D not a multiple of 16
    (1, 40, 5, 4, 33, 120, 32),   # 80 + 40, odd W (cp.async staging), lone octet
])
def test_fused_disparity_bands(ww, torch, orc, shape):
    """Disparity ranges that one launch cannot hold run as bands, each with
    the volume plane below and above it: within the fp16 tolerance of the
    oracle, and with the CUDA-core correlation bit-identical to
    corr_volume -> cost_stem3d (the volume form runs the same bands)."""
    from whirlwind_trt_plugins_b200.configs import FrontEnd, make_inputs
    B, C, G, H, W, D, Cout = shape
    cfg = FrontEnd("bands", B=B, C=C, G=G, H=H, W=W, D=D, Cout=Cout)
    x = make_inputs(cfg, seed=D + W)
    tl, tr, tw, tb = (_t(torch, x[k]) for k in ("left", "right", "w", "b"))
    out = ww.corr_cost_stem3d(tl, tr, tw, tb, cfg.D, cfg.G)
    ref = orc.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, acc_mode=orc.ACC_F64)
    err = np.abs(out.cpu().numpy().astype(np.float32) - ref.astype(np.float32)).max()
    assert err <= ATOL_F16, f"max abs err {err}"
    prev = ww.set_fused_corr_engine(ww.CORR_ENGINE_CUDA_CORES)
    try:
        fused = ww.corr_cost_stem3d(tl, tr, tw, tb, cfg.D, cfg.G)
        unfused = ww.cost_stem3d(ww.corr_volume(tl, tr, cfg.D, cfg.G), tw, tb)
    finally:
        ww.set_fused_corr_engine(prev)
    assert torch.equal(fused, unfused)
    assert ww.device_error() == 0


def test_stem_disparity_bands_volume_form(ww, torch, orc):
    """The generalised stem on a 96-disparity volume with Cout = 32 (two
    bands) against the oracle's conv3d."""
    rng = np.random.default_rng(96)
    B, Cin, D, H, W, Cout = 1, 16, 96, 4, 24, 32
    vol = (rng.standard_normal((B, Cin, D, H, W)) * 0.5).astype(np.float16)
    w = (rng.standard_normal((Cout, Cin, 3, 3, 3)) * 0.05).astype(np.float16)
    b = (rng.standard_normal(Cout) * 0.1).astype(np.float16)
    out = ww.cost_stem3d(_t(torch, vol), _t(torch, w), _t(torch, b)).cpu().numpy().astype(np.float32)
    ref = orc.stem(vol, w, b, acc_mode=orc.ACC_F64).astype(np.float32)
    assert float(np.abs(out - ref).max()) <= ATOL_F16
    assert ww.device_error() == 0


@pytest.mark.parametrize("shape", [
    # (B, C, G, H, W, D, Cout): channel widths on every correlation path
    (1, 64, 2, 5, 24, 24, 16),     # Cg = 32: channels in two tensor-core chunks
    (1, 40, 2, 4, 20, 20, 8),      # Cg = 20 (zero-padded chunk), W % 8 != 0 (scalar staging)
    (2, 24, 8, 6, 33, 13, 32),     # Cg = 3, odd W and D
    (1, 16, 16, 3, 16, 70, 16),    # Cg = 1, five M-blocks along D
    (1, 96, 8, 4, 24, 64, 16),     # Cg = 12 (m16n8k16 with padded channels)
    (1, 48, 3, 5, 16, 9, 4),       # lone octet with 3 groups, D < 16
])
def test_fused_shapes_match_oracle(ww, torch, orc, shape):
    from whirlwind_trt_plugins_b200.configs import FrontEnd, make_inputs
    B, C, G, H, W, D, Cout = shape
    cfg = FrontEnd("edge", B=B, C=C, G=G, H=H, W=W, D=D, Cout=Cout)
    x = make_inputs(cfg, seed=C + W + D)
    out = _fused(ww, torch, x, cfg).cpu().numpy().astype(np.float32)
    ref = orc.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, acc_mode=orc.ACC_F64)
    err = np.abs(out - ref.astype(np.float32)).max()
    assert err <= ATOL_F16, f"max abs err {err}"
    assert ww.device_error() == 0


@pytest.mark.parametrize("cfg_id,B", [(2, 1), (3, 4), (4, 1), (4, 2), (5, 2)])
def test_fused_full_size_matches_oracle(ww, torch, orc, cfg_id, B):
    """The benchmark configurations at their full H x W x D (and full batch,
    except config 4, whose 64 items are checked as B = 1 and B = 2 with the
    5 % zeroed-pixel mask): every output within the fp16 tolerance of the
    oracle (fp32 sequential accumulation), and the fused volume within one
    fp16 ulp of the unfused CorrVolume -> stem composition."""
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[cfg_id].scaled(B=B)
    x = make_inputs(cfg)
    t = {k: _t(torch, x[k]) for k in ("left", "right", "w", "b")}
    fused = ww.corr_cost_stem3d(t["left"], t["right"], t["w"], t["b"], cfg.D, cfg.G, act=cfg.act)
    out = fused.cpu().numpy().astype(np.float32)
    ref = orc.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, act=cfg.act,
                        acc_mode=orc.ACC_F32_SEQ).astype(np.float32)
    err = np.abs(out - ref)
    assert float(err.max()) <= ATOL_F16, f"max abs err {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"
    assert np.all(np.isfinite(out))
    vol = ww.corr_volume(t["left"], t["right"], cfg.D, cfg.G)
    unfused = ww.cost_stem3d(vol, t["w"], t["b"], act=cfg.act)
    diff = (fused.float() - unfused.float()).abs()
    assert float(diff.max()) <= ATOL_F16
    assert float((diff == 0).float().mean()) >= 0.99
    assert ww.device_error() == 0


def test_fused_band_stitches_full_width(ww, torch):
    """Row bands of a full-width config-3 image (W = 320, D = 64): four bands
    of uneven height, each from its rows plus the one-row halo, stitch to the
    unsharded output bit for bit."""
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[3].scaled(B=1)
    x = make_inputs(cfg)
    tl, tr, tw, tb = (_t(torch, x[k]) for k in ("left", "right", "w", "b"))
    full = ww.corr_cost_stem3d(tl, tr, tw, tb, cfg.D, cfg.G)
    parts = []
    for (r0, r1) in ((0, 45), (45, 46), (46, 113), (113, 180)):
        i0, i1 = max(0, r0 - 1), min(cfg.H, r1 + 1)
        parts.append(ww.corr_cost_stem3d_band(tl[:, :, i0:i1].contiguous(), tr[:, :, i0:i1].contiguous(), tw, tb,
                                              cfg.D, cfg.G, cfg.H, i0, r0, r1 - r0))
    stitched = torch.cat(parts, dim=3)
    assert torch.equal(stitched.view(torch.int16), full.view(torch.int16))


def test_fused_band_stitches_to_full(ww, torch):
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[3].scaled(B=1, H=23, W=40)
    x = make_inputs(cfg)
    tl, tr, tw, tb = (_t(torch, x[k]) for k in ("left", "right", "w", "b"))
    full = ww.corr_cost_stem3d(tl, tr, tw, tb, cfg.D, cfg.G)
    parts = []
    for (r0, r1) in ((0, 7), (7, 8), (8, 23)):
        i0, i1 = max(0, r0 - 1), min(cfg.H, r1 + 1)
        band_l = tl[:, :, i0:i1].contiguous()
        band_r = tr[:, :, i0:i1].contiguous()
        parts.append(ww.corr_cost_stem3d_band(band_l, band_r, tw, tb, cfg.D, cfg.G, cfg.H, i0, r0, r1 - r0))
    stitched = torch.cat(parts, dim=3)
    assert torch.equal(stitched.view(torch.int16), full.view(torch.int16))


def test_fused_relu6(ww, torch, orc):
    from whirlwind_trt_plugins_b200.configs import CONFIGS, make_inputs
    cfg = CONFIGS[5].scaled(B=1, H=6, W=24)
    x = make_inputs(cfg)
    x["b"] = (x["b"].astype(np.float32) + 5.0).astype(np.float16)  # push values past 6
    out = _fused(ww, torch, x, cfg, act=1).cpu().numpy().astype(np.float32)
    ref = orc.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, act=1).astype(np.float32)
    assert out.max() <= 6.0 and np.abs(out - ref).max() <= ATOL_F16


def test_no_device_error_recorded(ww, torch):
    assert ww.device_error() == 0
