"""bench.py's reference arm (`--impl reference`) on CPU: the plain-C oracle
port of the path timed on the host, printed as one JSON line with the fields
the benchmark contract names; under torchrun only rank 0 works and prints."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_reference_arm_loads_nothing_from_the_package():
    """The reference arm must not import the product package or map its CUDA
    library, and prints the same config dict as the GPU arm (config_dict)."""
    code = (
        "import json, runpy, sys, io, contextlib\n"
        f"sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1']\n"
        "buf = io.StringIO()\n"
        "with contextlib.redirect_stdout(buf):\n"
        f"    runpy.run_path({os.path.join(ROOT, 'bench.py')!r}, run_name='__main__')\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'libww_trt_plugins' not in maps, 'library mapped'\n"
        "assert 'whirlwind_trt_plugins_b200' not in sys.modules, 'package imported'\n"
        "line = json.loads(buf.getvalue().strip().splitlines()[-1])\n"
        f"sys.path.insert(0, {ROOT!r})\n"
        "import bench\n"
        "C = bench.load_configs()\n"
        "assert line['config'] == bench.config_dict(C.CONFIGS[bench.DEFAULT_CONFIG], 1), line['config']\n"
        "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=dict(os.environ, RANK="0", WORLD_SIZE="1"),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith("ok")
