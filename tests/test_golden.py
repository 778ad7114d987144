"""Pin the CPU oracle to the reference: every golden fixture in tests/golden/
was produced on a B200 by the reference's own CUDA kernels (rebuilt from the
unmodified reference sources; see tests/golden/make_golden.py).  The oracle
must reproduce each one bit for bit -- including which of the reference's two
CorrVolume kernels (acc / C or acc * 1/C) the reference picked.  CPU only."""
import numpy as np
import pytest

from conftest import golden_files, load_golden

FILES = golden_files()


def test_fixtures_present():
    assert len(FILES) >= 10, "golden fixtures missing: run tests/golden/make_golden.py on a GPU"


@pytest.mark.parametrize("name", FILES)
def test_oracle_reproduces_reference(orc, name):
    g = load_golden(name)
    kind = str(g["kind"])
    if kind == "corr32":
        got = orc.corr_f32(g["left"], g["right"], int(g["D"]))
        assert np.array_equal(got.view(np.uint32), g["out"].view(np.uint32))
    elif kind in ("corr16", "gcorr16"):
        got = orc.corr_f16(g["left"], g["right"], int(g["D"]), int(g["G"]))
        assert got.shape == g["out"].shape
        assert np.array_equal(got.view(np.uint16), g["out"].view(np.uint16))
    elif kind == "stem3":
        got = orc.stem_ref3(g["vol"], g["w0"], g["b0"], g["w1"], g["b1"], g["w2"], g["b2"])
        assert np.array_equal(got.view(np.uint16), g["out"].view(np.uint16))
    elif kind in ("nv12_16", "nv12_32"):
        f16 = kind == "nv12_16"
        got = orc.nv12_decode(g["nv12"], int(g["H_OUT"]), int(g["W_OUT"]), out_f16=f16)
        assert got.shape == g["out"].shape
        if f16:
            assert np.array_equal(got.view(np.uint16), g["out"].view(np.uint16))
        else:
            assert np.array_equal(got.view(np.uint32), g["out"].view(np.uint32))
    else:
        pytest.fail(f"unknown fixture kind {kind}")


def test_fixtures_cover_both_reference_kernels(orc):
    """The set includes calls the reference routes to its naive kernel and
    calls it routes to its fast kernel, with a non-power-of-two channel count
    on each side (where acc / C and acc * (1/C) can differ)."""
    modes = set()
    for name in FILES:
        g = load_golden(name)
        if str(g["kind"]) not in ("corr16", "gcorr16"):
            continue
        B, C, G = int(g["B"]), int(g["C"]), int(g["G"])
        H, W, D = int(g["H"]), int(g["W"]), int(g["D"])
        m = orc.grouped_scale_mode(True, B, C, G, H, W, D)
        modes.add((m, (C // G) & (C // G - 1) != 0))
    assert (orc.SCALE_MULINV, True) in modes and (orc.SCALE_DIV, True) in modes
