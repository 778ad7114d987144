"""Profiling driver (not a test): runs the reference-shaped 3-stage stem at
its native shape [1, 1, 48, 32, 40] four times, either alone (`stem`) or fused
with its G = 1 correlation from C = 64 features (`fused`), for an ncu capture
of one launch:

    python tests/profiling/native_stem_driver.py stem
    ncu --set full --clock-control none -k regex:cost_stem3d_ref3 -s 3 -c 1 \\
        python tests/profiling/native_stem_driver.py stem
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402

import whirlwind_trt_plugins_b200 as ww  # noqa: E402


def main(mode: str) -> None:
    g = torch.Generator(device="cuda").manual_seed(7)
    ws = [(torch.randn((n,), generator=g, device="cuda") * s).half()
          for n, s in ((108, 0.2), (4, 0.1), (432, 0.2), (4, 0.1), (108, 0.2), (1, 0.1))]
    if mode == "stem":
        vol = torch.randn((1, 1, 48, 32, 40), generator=g, device="cuda").half()
        for _ in range(4):
            ww.cost_stem3d_ref3(vol, *ws)
    else:
        L = torch.randn((1, 64, 32, 40), generator=g, device="cuda").half()
        R = torch.randn((1, 64, 32, 40), generator=g, device="cuda").half()
        for _ in range(4):
            ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=48)
    torch.cuda.synchronize()
    print("ok", mode)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "stem")
