"""The product path has no CPU fallback: importing the package from a copy
that lacks the built CUDA library fails at import time with an error naming
the missing library, rather than computing anything on the host."""
import os
import shutil
import subprocess
import sys

from conftest import ROOT


def test_import_without_library_fails_loudly(tmp_path):
    pkg = tmp_path / "whirlwind_trt_plugins_b200"
    pkg.mkdir()
    shutil.copy(os.path.join(ROOT, "whirlwind_trt_plugins_b200", "__init__.py"), pkg / "__init__.py")
    r = subprocess.run([sys.executable, "-c", "import whirlwind_trt_plugins_b200"], cwd=tmp_path,
                       env=dict(os.environ, PYTHONPATH=str(tmp_path)), capture_output=True, text=True,
                       timeout=120)
    assert r.returncode != 0
    assert "ImportError" in r.stderr and "libww_trt_plugins.so is missing" in r.stderr
    assert "no CPU fallback" in r.stderr
