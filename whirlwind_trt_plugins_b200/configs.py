"""Workload configurations of the stereo cost-volume front end and their
seeded synthetic inputs.

The five configurations are the benchmark / parity cases of this project
(quarter-resolution stereo feature maps).  Inputs are synthetic and seeded:
left features from seed ``seed``, right from ``seed + 1``, conv weights from
``seed + 2``, BatchNorm scale/bias from ``seed + 3`` and the invalid-pixel
mask from ``seed + 4``.  BatchNorm is folded on the host (fp32 product,
rounded to fp16 once) before anything reaches the GPU.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class FrontEnd:
    name: str
    B: int
    C: int
    G: int
    H: int
    W: int
    D: int
    Cout: int            # 0: correlation only (no stem)
    dtype: str = "f16"   # "f16" | "f32"
    dist: str = "normal"  # "normal" N(0,1) | "uniform" U(-1,1)
    zero_frac: float = 0.0  # fraction of (b, h, w) pixels zeroed across all channels
    act: int = 0         # 0 ReLU, 1 ReLU6

    @property
    def voxels(self) -> int:
        return self.B * self.D * self.H * self.W

    def algorithmic_bytes(self) -> int:
        """Ideal HBM traffic: read left and right once, write the stem output."""
        s_in = 2 if self.dtype == "f16" else 4
        out = (self.B * self.Cout * self.D * self.H * self.W * 2) if self.Cout else \
            (self.B * self.G * self.D * self.H * self.W * s_in)
        return 2 * self.B * self.C * self.H * self.W * s_in + out

    def stem_flops(self) -> int:
        return 2 * self.B * self.Cout * self.G * 27 * self.D * self.H * self.W

    def corr_flops(self) -> int:
        return 2 * self.B * self.C * self.D * self.H * self.W

    def scaled(self, **kw) -> "FrontEnd":
        d = dict(self.__dict__)
        d.update(kw)
        return FrontEnd(**d)


CONFIGS: dict[int, FrontEnd] = {
    1: FrontEnd("c1_corr_fp32", B=1, C=32, G=1, H=60, W=80, D=24, Cout=0, dtype="f32"),
    2: FrontEnd("c2_gwc40_stem32", B=1, C=320, G=40, H=120, W=160, D=48, Cout=32),
    3: FrontEnd("c3_hd_gwc8_stem16", B=4, C=96, G=8, H=180, W=320, D=64, Cout=16),
    4: FrontEnd("c4_batched_gwc32_stem32", B=64, C=256, G=32, H=94, W=312, D=48, Cout=32, zero_frac=0.05),
    5: FrontEnd("c5_edge_gwc16_stem16", B=2, C=64, G=16, H=96, W=128, D=32, Cout=16, dist="uniform"),
}


def _features(cfg: FrontEnd, seed: int, shape) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if cfg.dist == "uniform":
        x = rng.uniform(-1.0, 1.0, size=shape).astype(np.float32)
    else:
        x = rng.standard_normal(size=shape, dtype=np.float32)
    return x


def make_inputs(cfg: FrontEnd, seed: int = 0) -> dict:
    """numpy inputs: left/right (fp16 or fp32), folded stem weights w16 [Cout, G, 3, 3, 3]
    and bias b16 [Cout] (fp16)."""
    shape = (cfg.B, cfg.C, cfg.H, cfg.W)
    L = _features(cfg, seed, shape)
    R = _features(cfg, seed + 1, shape)
    if cfg.zero_frac > 0:
        m = np.random.default_rng(seed + 4).random((cfg.B, 1, cfg.H, cfg.W)) < cfg.zero_frac
        L = np.where(m, 0.0, L).astype(np.float32)
        R = np.where(m, 0.0, R).astype(np.float32)
    out = {}
    if cfg.dtype == "f16":
        out["left"], out["right"] = L.astype(np.float16), R.astype(np.float16)
    else:
        out["left"], out["right"] = L, R
    if cfg.Cout:
        w = (np.random.default_rng(seed + 2).standard_normal((cfg.Cout, cfg.G, 3, 3, 3), dtype=np.float32)
             * np.float32(0.05)).astype(np.float32)
        rng = np.random.default_rng(seed + 3)
        scale = rng.uniform(0.5, 1.5, size=(cfg.Cout,)).astype(np.float32)
        bias = (rng.standard_normal(size=(cfg.Cout,), dtype=np.float32) * np.float32(0.1)).astype(np.float32)
        w16 = (w * scale[:, None, None, None, None]).astype(np.float16)
        out["w"], out["b"] = w16, bias.astype(np.float16)
        out["w_raw"], out["scale"], out["bias_raw"] = w, scale, bias
    return out


def make_inputs_torch(cfg: FrontEnd, device, seed: int = 0) -> dict:
    """The same distributions generated on the GPU with a seeded torch
    generator (for full-size benchmark inputs; not bit-identical to
    make_inputs)."""
    import torch
    g = torch.Generator(device=device)
    shape = (cfg.B, cfg.C, cfg.H, cfg.W)
    dt = torch.float16 if cfg.dtype == "f16" else torch.float32

    def feat(s):
        g.manual_seed(s)
        if cfg.dist == "uniform":
            return torch.rand(shape, generator=g, device=device, dtype=torch.float32).mul_(2).sub_(1)
        return torch.randn(shape, generator=g, device=device, dtype=torch.float32)

    L, R = feat(seed), feat(seed + 1)
    if cfg.zero_frac > 0:
        g.manual_seed(seed + 4)
        keep = (torch.rand((cfg.B, 1, cfg.H, cfg.W), generator=g, device=device) >= cfg.zero_frac).float()
        L.mul_(keep)
        R.mul_(keep)
    out = {"left": L.to(dt), "right": R.to(dt)}
    del L, R
    if cfg.Cout:
        host = make_inputs(cfg.scaled(B=1, H=1, W=8), seed)  # weights do not depend on B/H/W
        out["w"] = torch.from_numpy(host["w"]).to(device)
        out["b"] = torch.from_numpy(host["b"]).to(device)
    return out
