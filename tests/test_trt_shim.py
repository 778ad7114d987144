"""The TensorRT plugin shim (csrc/trt/ww_trt_plugins.cpp) compiles: TensorRT is
not installed here, so it is checked with `g++ -fsyntax-only -Werror` against
stand-in declarations of the IPluginV3 interface (tests/trt_stub/), which
catch a wrong override, a missing method or a type mismatch against the
interface the shim implements.  Building it for real needs TensorRT's headers
and libnvinfer (the build script's --trt-include option)."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

CUDA_INCLUDE = "/usr/local/cuda/include"


@pytest.mark.skipif(shutil.which("g++") is None or not os.path.isdir(CUDA_INCLUDE),
                    reason="needs g++ and the CUDA headers")
def test_shim_compiles_against_the_plugin_interface():
    src = os.path.join(ROOT, "whirlwind_trt_plugins_b200", "csrc", "trt", "ww_trt_plugins.cpp")
    cmd = ["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Werror",
           "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(ROOT, "tests", "trt_stub"),
           "-I" + CUDA_INCLUDE, src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
