"""Build libww_trt_plugins.so in-tree for sm_100a with nvcc.

    python whirlwind_trt_plugins_b200/build.py [--force] [--trt-include DIR]

(run by path: importing the package loads the library this script builds)

Each CUDA/C++ source in csrc/ compiles to an object under _build/ (parallel),
then everything links into whirlwind_trt_plugins_b200/libww_trt_plugins.so
with a static CUDA runtime.  The TensorRT plugin shim (csrc/trt/) is added
only when TensorRT headers are given (--trt-include or $TENSORRT_INCLUDE);
without them the library exports the C ABI of include/ww_trt_plugins.h only.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libww_trt_plugins.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              "--expt-relaxed-constexpr", f"-I{ROOT}/include"] + ARCH

SOURCES = [
    "capi.cu",
    "corr_volume.cu",
    "cost_stem3d_ref3.cu",
    "stem_tc.cu",
    "tensor_map.cu",
    "nv12_decode.cu",
    "disparity_regression.cu",
    "multi.cu",
    "plugin_core.cpp",
]
TRT_SOURCES = ["trt/ww_trt_plugins.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _headers() -> list[str]:
    hs = [os.path.join(ROOT, "include", "ww_trt_plugins.h")]
    for f in os.listdir(CSRC):
        if f.endswith((".cuh", ".h", ".hpp")):
            hs.append(os.path.join(CSRC, f))
    return hs


def build(force: bool = False, trt_include: str | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    trt_include = trt_include or os.environ.get("TENSORRT_INCLUDE")
    srcs = list(SOURCES) + (TRT_SOURCES if trt_include else [])
    hdrs = _headers()
    cmds = []
    objs = []
    for s in srcs:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace("/", "_") + ".o")
        objs.append(obj)
        if not force and _newer(obj, [src] + hdrs):
            continue
        extra = [f"-I{trt_include}", "-DWW_WITH_TENSORRT"] if trt_include else []
        cmds.append([nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for cmd, res in zip(cmds, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds)):
            if verbose or res.returncode != 0:
                sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed for {cmd[-3]}")
    if force or cmds or not os.path.exists(LIB):
        link = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs
        if trt_include:
            link += ["-lnvinfer"]
        res = subprocess.run(link, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(" ".join(link) + "\n" + res.stdout + res.stderr)
            raise RuntimeError("link failed")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--trt-include", default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, trt_include=a.trt_include, verbose=a.verbose))


if __name__ == "__main__":
    main()
