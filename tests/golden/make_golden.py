"""Generate the golden fixtures that pin the CPU oracle to the reference.

The reference (IntelligentRoboticsLab/whirlwind_trt_plugins) ships no test
vectors, so the fixtures are produced by the reference's OWN CUDA kernels:
``oracle/_ref/libww_ref.so`` is compiled by ``oracle/Makefile`` from the
unmodified reference sources (src/plugins/corr_volume/corr_volume_kernel.cu,
src/plugins/cost_stem_3d/cost_stem_3d_kernel.cu,
src/plugins/nv12_decode/nv12_decode_kernel.cu) for sm_100a.  This script runs
them on a B200 on seeded inputs and saves inputs + outputs as .npz:

    python tests/golden/make_golden.py [out_dir [name_filter]]   (needs a GPU)

Each case calls the reference launcher exactly as the reference plugin does
(launchCorrVolume<T>(left, right, out, B, C, H, W, D, stream) and
launchCostStem3D(in, out, w0, b0, w1, b1, w2, b2, B, D, H, W, stream) and
launchNv12Decode<T>(nv12, out, H_IN, W_IN, H_OUT, W_OUT, stream));
group-wise correlation is the reference called once per (batch, group), the
only way the reference can produce it.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

# (name, kind, params).  kind: corr16 / corr32 / gcorr16 / stem3.
CASES = [
    ("corr16_naive_small", "corr16", dict(B=1, C=8, H=6, W=20, D=5, seed=10)),
    ("corr16_naive_wlt_d", "corr16", dict(B=2, C=4, H=3, W=16, D=24, seed=11)),
    ("corr16_naive_ragged_w", "corr16", dict(B=1, C=6, H=5, W=37, D=12, seed=12)),
    ("corr16_fast_c16", "corr16", dict(B=1, C=16, H=32, W=128, D=48, seed=13)),
    ("corr16_fast_c12", "corr16", dict(B=1, C=12, H=32, W=128, D=48, seed=14)),
    ("corr16_fast_c200_tile8", "corr16", dict(B=1, C=200, H=10, W=128, D=96, seed=15)),
    ("corr32_c1_small", "corr32", dict(B=1, C=32, H=20, W=40, D=24, seed=16)),
    ("corr32_ragged", "corr32", dict(B=2, C=3, H=4, W=9, D=7, seed=17)),
    ("gcorr16_naive_g4", "gcorr16", dict(B=2, C=32, G=4, H=16, W=64, D=24, seed=18)),
    ("gcorr16_fast_g2_c12", "gcorr16", dict(B=1, C=24, G=2, H=32, W=128, D=48, seed=19)),
    ("gcorr16_naive_g2_c12_d64", "gcorr16", dict(B=1, C=24, G=2, H=8, W=64, D=64, seed=20)),
    ("stem3_native", "stem3", dict(B=1, D=48, H=32, W=40, seed=21)),
    ("stem3_ragged", "stem3", dict(B=1, D=13, H=9, W=11, seed=22)),
    ("stem3_tiny", "stem3", dict(B=1, D=1, H=1, W=1, seed=23)),
    ("nv12_16_down2", "nv12_16", dict(H_IN=96, W_IN=128, H_OUT=48, W_OUT=64, seed=24)),
    ("nv12_16_up_odd", "nv12_16", dict(H_IN=30, W_IN=40, H_OUT=45, W_OUT=61, seed=25)),
    ("nv12_16_default", "nv12_16", dict(H_IN=120, W_IN=160, H_OUT=224, W_OUT=288, seed=26)),
    ("nv12_32_default", "nv12_32", dict(H_IN=120, W_IN=160, H_OUT=224, W_OUT=288, seed=27)),
    ("nv12_32_ragged", "nv12_32", dict(H_IN=14, W_IN=22, H_OUT=9, W_OUT=13, seed=28)),
]


def _feat(rng, shape, dtype):
    return rng.standard_normal(size=shape, dtype=np.float32).astype(dtype)


def run_case(name: str, kind: str, prm: dict) -> dict:
    import torch
    from oracle import ref_lib
    R = ref_lib()
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(prm["seed"])
    out = {"kind": np.array(kind)}
    if kind in ("corr16", "corr32", "gcorr16"):
        B, C, H, W, D = prm["B"], prm["C"], prm["H"], prm["W"], prm["D"]
        G = prm.get("G", 1)
        dt = np.float32 if kind == "corr32" else np.float16
        L = _feat(rng, (B, C, H, W), dt)
        Rt = _feat(rng, (B, C, H, W), dt)
        tl = torch.from_numpy(L).to(dev)
        tr = torch.from_numpy(Rt).to(dev)
        shape = (B, G, D, H, W) if kind == "gcorr16" else (B, D, H, W)
        to = torch.full(shape, float("nan"), dtype=tl.dtype, device=dev)
        if kind == "corr16":
            rc = R.wwref_corr_volume_f16(tl.data_ptr(), tr.data_ptr(), to.data_ptr(), B, C, H, W, D, stream)
        elif kind == "corr32":
            rc = R.wwref_corr_volume_f32(tl.data_ptr(), tr.data_ptr(), to.data_ptr(), B, C, H, W, D, stream)
        else:
            rc = R.wwref_corr_volume_grouped_f16(tl.data_ptr(), tr.data_ptr(), to.data_ptr(), B, C, H, W, D, G,
                                                  stream)
        torch.cuda.synchronize()
        assert rc == 0, f"{name}: reference launcher returned {rc}"
        out.update(left=L, right=Rt, out=to.cpu().numpy(), B=B, C=C, G=G, H=H, W=W, D=D)
    elif kind == "stem3":
        B, D, H, W = prm["B"], prm["D"], prm["H"], prm["W"]
        x = (rng.standard_normal((B, 1, D, H, W), dtype=np.float32) * 2.0).astype(np.float16)
        ws = {
            "w0": (rng.standard_normal(108, dtype=np.float32) * 0.3).astype(np.float16),
            "b0": (rng.standard_normal(4, dtype=np.float32) * 0.2).astype(np.float16),
            "w1": (rng.standard_normal(432, dtype=np.float32) * 0.2).astype(np.float16),
            "b1": (rng.standard_normal(4, dtype=np.float32) * 0.2).astype(np.float16),
            "w2": (rng.standard_normal(108, dtype=np.float32) * 0.2).astype(np.float16),
            "b2": (rng.standard_normal(1, dtype=np.float32) * 0.2 + 0.5).astype(np.float16),
        }
        tx = torch.from_numpy(x).to(dev)
        tws = {k: torch.from_numpy(v).to(dev) for k, v in ws.items()}
        to = torch.full_like(tx, float("nan"))
        rc = R.wwref_cost_stem3d(tx.data_ptr(), to.data_ptr(), *[tws[k].data_ptr() for k in
                                 ("w0", "b0", "w1", "b1", "w2", "b2")], B, D, H, W, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"{name}: reference launcher returned {rc}"
        out.update(vol=x, out=to.cpu().numpy(), B=B, D=D, H=H, W=W, **ws)
    elif kind in ("nv12_16", "nv12_32"):
        Hi, Wi, Ho, Wo = prm["H_IN"], prm["W_IN"], prm["H_OUT"], prm["W_OUT"]
        img = rng.integers(0, 256, size=(Hi * 3 // 2, Wi), dtype=np.uint8)
        img[0, :4] = (0, 255, 0, 255)  # the extremes of both planes
        img[Hi, :4] = (0, 255, 255, 0)
        ti = torch.from_numpy(img).to(dev)
        f16 = kind == "nv12_16"
        to = torch.full((1, 3, Ho, Wo), float("nan"), dtype=torch.float16 if f16 else torch.float32, device=dev)
        fn = R.wwref_nv12_decode_f16 if f16 else R.wwref_nv12_decode_f32
        rc = fn(ti.data_ptr(), to.data_ptr(), Hi, Wi, Ho, Wo, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"{name}: reference launcher returned {rc}"
        out.update(nv12=img, out=to.cpu().numpy(), H_IN=Hi, W_IN=Wi, H_OUT=Ho, W_OUT=Wo)
    else:
        raise ValueError(kind)
    return out


def main() -> None:
    out_dir = sys.argv[1] if len(sys.argv) > 1 else HERE
    only = sys.argv[2] if len(sys.argv) > 2 else ""
    os.makedirs(out_dir, exist_ok=True)
    for name, kind, prm in CASES:
        if only not in name:
            continue
        d = run_case(name, kind, prm)
        np.savez(os.path.join(out_dir, f"{name}.npz"), **d)
        print(f"{name}: {kind} {prm} -> out {d['out'].shape} {d['out'].dtype}")


if __name__ == "__main__":
    main()
