"""Benchmark of the fused stereo front end (group-wise correlation -> 3x3x3
stem) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 4] [--impl ours|reference]

One step = one fused correlation + stem pass (ww_corr_cost_stem3d) over the
whole batch of the workload.  The headline workload is config 4, the batched
wide-aspect stereo set (B=64 C=256 G=32 H=94 W=312 D=48 Cout=32, fp16, 5 %
of the pixels zeroed), the largest configuration that fits one GPU.  Under
torchrun (N > 1) its 64 pairs are split across the ranks (split_even), each
rank computing its share on its own GPU with no collective on the data
path: the global batch is fixed, so scaling is strong.

Printed (rank 0, one JSON line):
  value      whole-job cost voxels/s (B*D*H*W of the full batch per step),
             inputs resident in HBM, CUDA-event time of exactly K steps, max
             over ranks.  Every step's inputs (1.9 GB for config 4) are
             larger than the 126 MB L2; smaller configs rotate over input /
             output sets of >= 400 MB.
  e2e        the same metric through the public API from pinned HOST
             buffers: every step copies its pairs host->device, runs the op
             and copies the whole output device->host, all inside the timed
             region (chunks of the batch rotate over three streams so the
             copies overlap the kernels).
  roofline   the fused kernel against the measured B200 peaks
             (MEASURED_PEAKS.json): stem FLOPs / kernel time vs the bf16 / fp16
             tensor peak, algorithmic bytes / time vs HBM; `traffic` from an
             ncu capture of the same kernel (per launch).
  cpu_baseline  the CPU oracle (plain-C restatement of the reference's
             semantics; the reference has no CPU implementation of its own)
             on a bounded row band of the same workload, all host threads.
  secondary  the other configurations measured the same way in the same run:
             at N = 1 configs 2, 3 and 5 (config 5 also as us per call); at
             N > 1 config 3 split into row bands over the N ranks, the
             one-row halo exchange (NCCL send/recv) inside the timed region.
--impl reference times the CPU implementation on the same workload (rank 0
only; the other ranks exit 0) and loads nothing from the product package.

Other ops (one GPU): --op corr_volume (the standalone group-wise CorrVolume,
HBM roofline, end to end from pinned host buffers), --op cost_stem3d (the
generalised stem on a configuration's volume, tensor roofline), --op
nv12_decode (camera decode), --op disparity_regression (soft-argmin after
aggregation), --op stem3_native (the reference's 3-stage stem at its native
shape, alone and fused with its G = 1 correlation).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "cost voxels/s (B*D*H*W) corr+3D stem"
UNIT = "voxels/s"
DEFAULT_CONFIG = 4
# The standalone CorrVolume line: config 2 (one 120 x 160 pair, 40 groups);
# config 4's 5.8 GB volume per batch would need ~23 GB of pinned host buffers
# for the end-to-end leg.
CORR_VOLUME_CONFIG = 2

# DRAM bytes (read + write) per launch of the fused kernel on the full
# configuration, from ncu captures (profiles/stem_tc_fused_*.md).  Configs 2
# and 5 leave most or all of their output in L2 when the launch ends; config 4
# is captured at B = 8 and scaled by 64 / 8 (traffic is per pair).
NCU_TRAFFIC_BYTES = {
    "c2_gwc40_stem32": 24.87e6 + 7.26e6,
    "c3_hd_gwc8_stem16": 125.60e6 + 448.59e6,
    "c4_batched_gwc32_stem32": (265.48e6 + 680.47e6) * 8,
    "c5_edge_gwc16_stem16": 6.57e6 + 0.18e6,
}

# Streams the end-to-end loop rotates over (copy in, op, copy out per chunk).
N_E2E_STREAMS = 3


def load_configs():
    """whirlwind_trt_plugins_b200/configs.py by its path: importing it as part
    of the package would run the package __init__ and load the CUDA library,
    which the reference arm must not do."""
    spec = importlib.util.spec_from_file_location(
        "ww_bench_configs", os.path.join(ROOT, "whirlwind_trt_plugins_b200", "configs.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=None,
                    help=f"configuration (default {DEFAULT_CONFIG}; --op corr_volume / cost_stem3d: "
                         f"{CORR_VOLUME_CONFIG})")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the configuration's batch (profiling captures of a smaller case)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--op", choices=["corr_cost_stem3d", "corr_volume", "cost_stem3d", "nv12_decode",
                                     "disparity_regression", "stem3_native"],
                    default="corr_cost_stem3d")
    ap.add_argument("--corr-engine", choices=["tensor", "cuda_cores"], default="tensor",
                    help="correlation engine of the fused op (ww_set_fused_corr_engine)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="profiling driver for ncu: one input set, W + K launches, nothing else")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d["bf16_tflops"],
                "tflops_sustained": d.get("bf16_tflops_sustained"), "src": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "src": "fallback"}


def workload_name(cfg) -> str:
    return (f"{cfg.name}: B={cfg.B} C={cfg.C} G={cfg.G} H={cfg.H} W={cfg.W} D={cfg.D} Cout={cfg.Cout} fp16"
            + (f", {cfg.zero_frac:.0%} of pixels zeroed" if cfg.zero_frac else ""))


def config_dict(cfg, world: int, mode: str = "batch") -> dict:
    """The workload description both arms print (identical for the same run)."""
    if mode == "rows":
        par = f"row bands over {world} GPU(s), one-row halo by NCCL send/recv, no collective in the op"
    elif world > 1:
        par = f"batch split over {world} GPUs (split_even), no collective in the op"
    else:
        par = "one GPU"
    per_set = cfg.algorithmic_bytes()
    l2 = (f"each step's inputs and output ({per_set / 1e9:.1f} GB) exceed the 126 MB L2"
          if per_set > 400 * 2**20 else "steps rotate over input/output sets totalling >= 400 MB (> 126 MB L2)")
    return {"workload": workload_name(cfg), "global_batch": cfg.B, "parallelism": par, "l2": l2}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- CPU arm

def cpu_sample_inputs(C, cfg, rows: int):
    """Inputs for output rows [0, rows) of batch item 0 (plus the halo row)."""
    return C.make_inputs(cfg.scaled(B=1, H=min(cfg.H, rows + 1)))


def cpu_oracle_seconds(cfg, x, rows: int, nthreads: int) -> float:
    """Wall time of the CPU oracle (corr + stem, fp32 accumulation) on output
    rows [0, rows) of batch item 0."""
    import oracle
    t0 = time.perf_counter()
    oracle.corr_stem(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, act=cfg.act,
                     acc_mode=oracle.ACC_F32_SEQ, rows=(0, rows), nthreads=nthreads)
    return time.perf_counter() - t0


def pick_cpu_rows(C, cfg, budget_s: float, nthreads: int) -> int:
    """Rows of batch item 0 whose oracle time is about `budget_s` seconds."""
    probe = min(cfg.H, 4)
    dt = cpu_oracle_seconds(cfg, cpu_sample_inputs(C, cfg, probe), probe, nthreads) / probe
    return max(1, min(cfg.H, int(budget_s / max(dt, 1e-4))))


def cpu_baseline(C, cfg, budget_s: float) -> dict:
    import oracle
    n = oracle.nthreads_default()
    rows = pick_cpu_rows(C, cfg, budget_s, n)
    x = cpu_sample_inputs(C, cfg, rows)
    dt = cpu_oracle_seconds(cfg, x, rows, n)
    return {"value": rows * cfg.W * cfg.D / dt, "unit": UNIT, "cores": n, "kind": "port",
            "sample": f"output rows [0,{rows}) of batch item 0 of {cfg.name}: corr+stem in the C oracle "
                      f"(fp32 accumulation), {dt:.1f} s"}


def run_reference(args, C, cfg, rank, world):
    """Reference arm: the CPU implementation of the path (the oracle port of
    the reference's semantics), each step a bounded row band of the
    workload; the whole run is sized to about two minutes.  Nothing from the
    product package is imported."""
    if rank != 0:
        return
    import oracle
    n = oracle.nthreads_default()
    per_step = min(2.0, 120.0 / max(1, args.steps + args.warmup))
    rows = pick_cpu_rows(C, cfg, per_step, n)
    x = cpu_sample_inputs(C, cfg, rows)
    for _ in range(args.warmup):
        cpu_oracle_seconds(cfg, x, rows, n)
    times = [cpu_oracle_seconds(cfg, x, rows, n) for _ in range(args.steps)]
    vox = rows * cfg.W * cfg.D
    value = vox * len(times) / sum(times)
    sample = f"output rows [0,{rows}) of batch item 0 of {cfg.name} per step (corr+stem, fp32 accumulation)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded normal/uniform features, N(0,0.05) weights)",
        "config": config_dict(cfg, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": n, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference has no CPU implementation of this path; its semantics run as the "
                "plain-C oracle port (oracle/ww_oracle.c) on all host threads",
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU arm

class Ctx:
    def __init__(self, world, rank, local):
        import torch
        self.world, self.rank, self.local = world, rank, local
        torch.cuda.set_device(local)
        self.dev = torch.device("cuda", local)
        self.dist = None
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.dist = dist

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        if self.dist is None:
            return v
        import torch
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()


def roofline(cfg, ms_per_step: float, peaks: dict) -> dict:
    """The fused kernel (the only kernel of a step) against the measured peaks."""
    t = ms_per_step * 1e-3
    tflops = cfg.stem_flops() / t / 1e12
    gbs = cfg.algorithmic_bytes() / t / 1e9
    f_tc, f_hbm = tflops / peaks["tflops"], gbs / peaks["hbm_gbs"]
    if f_tc >= f_hbm:
        roof = {"bound": "tensor", "achieved": tflops, "peak": peaks["tflops"], "unit": "TFLOP/s", "frac": f_tc}
    else:
        roof = {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": f_hbm}
    roof.update({"traffic": NCU_TRAFFIC_BYTES.get(cfg.name), "peak_source": peaks["src"] + " (burst)",
                 "other": {"hbm_gbs": gbs, "hbm_frac": f_hbm, "tensor_tflops": tflops, "tensor_frac": f_tc,
                           "tensor_frac_of_sustained": (tflops / peaks["tflops_sustained"]
                                                        if peaks.get("tflops_sustained") else None),
                           "algorithmic_bytes": cfg.algorithmic_bytes(), "stem_flops": cfg.stem_flops()}})
    return roof


def local_batch(cfg, ctx) -> tuple[int, int]:
    from whirlwind_trt_plugins_b200.shard import split_even
    return split_even(cfg.B, ctx.world, ctx.rank)


def make_sets(C, cfg, ctx, b_local: int, n_max: int):
    """Rotating resident input/output sets of this rank's share of the batch."""
    import torch
    lcfg = cfg.scaled(B=b_local)
    per_set = lcfg.algorithmic_bytes()
    n_sets = min(n_max, max(1, -(-400 * 2**20 // max(per_set, 1))))
    sets = []
    for s in range(n_sets):
        x = C.make_inputs_torch(lcfg, ctx.dev, seed=1000 * ctx.rank + 10 * s)
        out = torch.empty((b_local, cfg.Cout, cfg.D, cfg.H, cfg.W), dtype=torch.float16, device=ctx.dev)
        sets.append((x["left"], x["right"], x["w"], x["b"], out))
    return sets


def soak(step, soak_s: float, soak_steps: int | None, sync) -> int:
    """Untimed steps before a timed region: for soak_s seconds of wall time,
    or exactly soak_steps steps when given; `sync` every 16 steps.  Returns
    the number of steps run."""
    t_end = time.time() + soak_s
    i = 0
    while (i < soak_steps) if soak_steps is not None else (time.time() < t_end):
        step(i)
        i += 1
        if i % 16 == 0:
            sync()
    return i


def time_steps(ctx, step, steps: int, soak_s: float, clocks: bool, soak_steps: int | None = None):
    """CUDA-event time (ms) of exactly `steps` steps after a soak, max over
    ranks; nvidia-smi clocks sampled during the soak and the timed region.
    The soak runs for soak_s seconds of wall time -- a different number of
    steps on each rank, so only for steps without a collective -- or, given
    soak_steps, exactly that many steps on every rank (steps that exchange
    data between ranks must all take the same collective calls)."""
    import torch
    stream = torch.cuda.current_stream()
    sampler = ClockSampler(ctx.local) if clocks else None
    if sampler is not None:
        sampler.__enter__()
    try:
        soak(step, soak_s, soak_steps, torch.cuda.synchronize)
        torch.cuda.synchronize()
        ctx.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
    finally:
        if sampler is not None:
            sampler.__exit__()
    ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    return ms, (sampler.summary() if sampler is not None else None)


def e2e_batch(ww, cfg, ctx, src, b_local: int, steps: int) -> dict | None:
    """End to end through the public API from pinned host memory: per step
    this rank's pairs go host->device, through ww.corr_cost_stem3d and the
    whole output back device->host, in chunks of the batch rotating over
    N_E2E_STREAMS streams (each with its own device buffers), so one chunk's
    copies overlap another's kernel."""
    import torch
    if b_local == 0:          # same collective sequence as the ranks with work
        ctx.barrier()
        ctx.max_over_ranks(0.0)
        return None
    L, R, w, b = src          # resident inputs: copied once into the host buffers
    chunk = max(1, min(b_local, 4))
    n_chunks = -(-b_local // chunk)
    shape_in = (b_local, cfg.C, cfg.H, cfg.W)
    shape_out = (b_local, cfg.Cout, cfg.D, cfg.H, cfg.W)
    hL = torch.empty(shape_in, dtype=torch.float16, pin_memory=True)
    hR = torch.empty(shape_in, dtype=torch.float16, pin_memory=True)
    hL.copy_(L)
    hR.copy_(R)
    del L, R
    hout = torch.empty(shape_out, dtype=torch.float16, pin_memory=True)
    lanes = []
    for _ in range(N_E2E_STREAMS):
        lanes.append({"s": torch.cuda.Stream(ctx.dev),
                      "dL": torch.empty((chunk,) + shape_in[1:], dtype=torch.float16, device=ctx.dev),
                      "dR": torch.empty((chunk,) + shape_in[1:], dtype=torch.float16, device=ctx.dev),
                      "dout": torch.empty((chunk,) + shape_out[1:], dtype=torch.float16, device=ctx.dev)})

    def run_step():
        for k in range(n_chunks):
            ln = lanes[k % N_E2E_STREAMS]
            c0, c1 = k * chunk, min(b_local, (k + 1) * chunk)
            n = c1 - c0
            with torch.cuda.stream(ln["s"]):
                ln["dL"][:n].copy_(hL[c0:c1], non_blocking=True)
                ln["dR"][:n].copy_(hR[c0:c1], non_blocking=True)
                ww.corr_cost_stem3d(ln["dL"][:n], ln["dR"][:n], w, b, cfg.D, cfg.G, act=cfg.act,
                                    out=ln["dout"][:n], stream=ln["s"])
                hout[c0:c1].copy_(ln["dout"][:n], non_blocking=True)

    stream = torch.cuda.current_stream()
    run_step()
    torch.cuda.synchronize()
    ctx.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for ln in lanes:                      # every lane starts after f0
        ln["s"].wait_stream(stream)
    for _ in range(steps):
        run_step()
    for ln in lanes:                      # f1 waits for every lane
        stream.wait_stream(ln["s"])
    f1.record(stream)
    torch.cuda.synchronize()
    ems = ctx.max_over_ranks(f0.elapsed_time(f1))
    return {"value": cfg.voxels * steps / (ems * 1e-3), "unit": UNIT,
            "h2d_bytes_per_step": 2 * hL.numel() * 2, "d2h_bytes_per_step": hout.numel() * 2,
            "steps": steps, "streams": N_E2E_STREAMS, "chunk_pairs": chunk,
            "note": "bytes are this rank's share; the value counts the whole batch over the max-over-ranks time"}


def bench_config(args, C, ww, cfg, ctx, *, steps, soak_s, clocks, e2e_steps, cpu_budget_s):
    """Batch-split (or single-GPU) measurement of one configuration."""
    import torch
    b0, b1 = local_batch(cfg, ctx)
    b_local = b1 - b0
    sets = make_sets(C, cfg, ctx, b_local, n_max=1 if args.profile else 8) if b_local else []
    stream = torch.cuda.current_stream()

    def step(i):
        if not sets:
            return
        L, R, w, b, out = sets[i % len(sets)]
        ww.corr_cost_stem3d(L, R, w, b, cfg.D, cfg.G, act=cfg.act, out=out, stream=stream)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(steps):
            step(i)
        torch.cuda.synchronize()
        return {"profile": f"{cfg.name} B={b_local}: {max(3, args.warmup)} + {steps} launches of the fused kernel"}
    ms, clk = time_steps(ctx, step, steps, soak_s, clocks)
    if ww.device_error() != 0:
        raise SystemExit("device error word set during the benchmark")
    ms_per_step = ms / steps
    res = {"value": cfg.voxels * steps / (ms * 1e-3), "ms_per_step": ms_per_step,
           "roofline": roofline(cfg.scaled(B=b_local) if ctx.world > 1 else cfg, ms_per_step, load_peaks()),
           "gpu_launches": steps if b_local else 0, "clocks": clk,
           "n_sets": len(sets)}
    if ctx.world > 1:
        res["roofline"]["note"] = f"per GPU: {b_local} of {cfg.B} pairs on rank {ctx.rank}"
    src = sets[0][:4] if sets else None
    del sets
    if not args.no_e2e:
        res["e2e"] = e2e_batch(ww, cfg, ctx, src, b_local, e2e_steps)
    else:
        res["e2e"] = None
    del src
    torch.cuda.empty_cache()
    res["cpu_baseline"] = None
    if not args.no_cpu_baseline and ctx.world == 1 and cpu_budget_s > 0:
        try:
            res["cpu_baseline"] = cpu_baseline(C, cfg, cpu_budget_s)
        except Exception as e:  # the baseline never blocks the measurement
            res["cpu_baseline"] = {"value": None, "unit": UNIT, "cores": None, "kind": "port",
                                   "sample": f"failed: {e}"}
    return res


def us_per_call(ww, C, cfg, ctx, calls: int = 200) -> dict:
    """Config 5's latency figures: device time per call from one CUDA graph of
    `calls` launches, and wall time per call of the Python API issuing them."""
    import torch
    x = C.make_inputs_torch(cfg, ctx.dev, seed=77)
    out = torch.empty((cfg.B, cfg.Cout, cfg.D, cfg.H, cfg.W), dtype=torch.float16, device=ctx.dev)

    def call(s):
        ww.corr_cost_stem3d(x["left"], x["right"], x["w"], x["b"], cfg.D, cfg.G, act=cfg.act, out=out, stream=s)

    stream = torch.cuda.current_stream()
    for _ in range(5):
        call(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap):
        for _ in range(calls):
            call(torch.cuda.current_stream())
    stream.wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    dev_us = e0.elapsed_time(e1) * 1e3 / calls
    del graph
    t0 = time.perf_counter()
    for _ in range(calls):
        call(stream)
    torch.cuda.synchronize()
    host_us = (time.perf_counter() - t0) * 1e6 / calls
    return {"us_per_call": dev_us, "us_per_call_api": host_us,
            "how": f"device: {calls} launches replayed from one CUDA graph (L2-resident inputs); "
                   f"api: {calls} ww.corr_cost_stem3d calls from Python, wall time"}


def bench_rows(args, C, ww, cfg, ctx, steps: int) -> dict:
    """Config 3 split into row bands over the ranks: per step each rank
    exchanges its one-row halo with its neighbours (NCCL send/recv of
    [B, C, 1, W] per side, left and right features) and runs the band form of
    the fused op on its rows.  Value: the whole image's voxels per
    max-over-ranks step time."""
    import torch
    from whirlwind_trt_plugins_b200 import shard
    x = C.make_inputs_torch(cfg, ctx.dev, seed=3)   # same seed on every rank: one image pair
    hl = shard.HaloBand(cfg.B, cfg.C, cfg.H, cfg.W, torch.float16, ctx.dev)
    hr = shard.HaloBand(cfg.B, cfg.C, cfg.H, cfg.W, torch.float16, ctx.dev)
    hl.own.copy_(x["left"][:, :, hl.r0:hl.r1])
    hr.own.copy_(x["right"][:, :, hr.r0:hr.r1])
    w, b = x["w"], x["b"]
    del x
    out = torch.empty((cfg.B, cfg.Cout, cfg.D, hl.r1 - hl.r0, cfg.W), dtype=torch.float16, device=ctx.dev)
    stream = torch.cuda.current_stream()

    def step(i):
        hl.exchange()
        hr.exchange()
        ww.corr_cost_stem3d_band(hl.band, hr.band, w, b, cfg.D, cfg.G, cfg.H, hl.i0, hl.r0, hl.r1 - hl.r0,
                                 act=cfg.act, out=out, stream=stream)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    # The step exchanges halo rows (NCCL send/recv): a fixed soak count, the
    # same on every rank.
    ms, _ = time_steps(ctx, step, steps, 0.0, False, soak_steps=100)
    return {"config": config_dict(cfg, ctx.world, "rows"), "value": cfg.voxels * steps / (ms * 1e-3),
            "unit": UNIT, "ms_per_step": ms / steps, "scaling": "strong",
            "gpu_launches": steps, "halo_bytes_per_rank_step": 2 * 2 * cfg.B * cfg.C * cfg.W * 2}


def bench_main(args, C, cfg, world, rank, local):
    import torch
    import whirlwind_trt_plugins_b200 as ww
    ctx = Ctx(world, rank, local)
    ww.set_fused_corr_engine(ww.CORR_ENGINE_CUDA_CORES if args.corr_engine == "cuda_cores"
                             else ww.CORR_ENGINE_TENSOR)
    head = bench_config(args, C, ww, cfg, ctx, steps=args.steps, soak_s=1.5, clocks=True,
                        e2e_steps=max(2, min(args.steps, 5)), cpu_budget_s=10.0)
    if args.profile:
        ctx.close()
        if rank == 0:
            print(head["profile"], flush=True)
        return
    secondary = []
    if not args.no_secondary:
        if world == 1:
            for cid in (2, 3, 5):
                if cid == cfg_id_of(C, cfg):
                    continue
                c2 = C.CONFIGS[cid]
                r = bench_config(args, C, ww, c2, ctx, steps=max(args.steps, 100), soak_s=0.3, clocks=False,
                                 e2e_steps=20, cpu_budget_s=6.0)
                r = {"config": config_dict(c2, world), "unit": UNIT, **r}
                if cid == 5:
                    r.update(us_per_call(ww, C, c2, ctx))
                secondary.append(r)
        else:
            secondary.append(bench_rows(args, C, ww, C.CONFIGS[3], ctx, steps=max(args.steps, 50)))
    ctx.close()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded normal/uniform features, N(0,0.05) weights)",
        "config": config_dict(cfg, world), "roofline": head["roofline"], "cpu_baseline": head["cpu_baseline"],
        "e2e": head["e2e"], "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
        "corr_engine": args.corr_engine, "secondary": secondary,
    }
    print(json.dumps(line), flush=True)


def cfg_id_of(C, cfg) -> int:
    for k, v in C.CONFIGS.items():
        if v.name == cfg.name:
            return k
    return -1


# --------------------------------------------------------------- other ops

# Nv12Decode workload: a batch of 720p NV12 camera frames decoded and
# resized to the plugin's default 224 x 288 output, fp16.
NV12_B, NV12_H, NV12_W, NV12_OH, NV12_OW = 8, 720, 1280, 224, 288


def bench_nv12(args):
    """One step = ww_nv12_decode over NV12_B frames (one GPU).  value: output
    pixels/s; roofline against HBM with bytes = the whole NV12 input + the
    fp16 output (the downscale reads fewer input bytes than that)."""
    import torch
    import whirlwind_trt_plugins_b200 as ww
    torch.cuda.set_device(0)
    B, H, W, OH, OW = NV12_B, NV12_H, NV12_W, NV12_OH, NV12_OW
    in_bytes, out_bytes = B * H * 3 // 2 * W, B * 3 * OH * OW * 2
    n_sets = max(2, -(-160 * 2**20 // (in_bytes + out_bytes)))  # > 126 MB of L2
    g = torch.Generator(device="cuda").manual_seed(1)
    sets = [(torch.randint(0, 256, (B, H * 3 // 2, W), generator=g, device="cuda", dtype=torch.uint8),
             torch.empty((B, 3, OH, OW), dtype=torch.float16, device="cuda")) for _ in range(n_sets)]
    stream = torch.cuda.current_stream()

    def step(i, st=None):
        x, o = sets[i % n_sets]
        ww.nv12_decode(x, OH, OW, out=o, stream=st if st is not None else stream)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
        print(f"profile run: nv12_decode, {max(3, args.warmup)} + {args.steps} launches", flush=True)
        return
    # A launch takes ~6 us on the device, less than the host needs to issue it
    # from Python, so the K timed launches are captured once in a CUDA graph and
    # replayed: the events then time the kernels, not the launch path.
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap):
        for i in range(args.steps):
            step(i, torch.cuda.current_stream())
    stream.wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        t_end = time.time() + 1.0
        while time.time() < t_end:
            graph.replay()
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    del graph
    px = B * OH * OW
    value = px / (ms * 1e-3)
    # end to end from pinned host frames, three streams
    hosts = [torch.empty((B, H * 3 // 2, W), dtype=torch.uint8, pin_memory=True) for _ in range(3)]
    for h in hosts:
        h.copy_(sets[0][0])
    houts = [torch.empty((B, 3, OH, OW), dtype=torch.float16, pin_memory=True) for _ in range(3)]
    dins = [torch.empty_like(sets[0][0]) for _ in range(3)]
    douts = [torch.empty_like(sets[0][1]) for _ in range(3)]
    strs = [torch.cuda.Stream() for _ in range(3)]

    def e2e_step(i):
        k = i % 3
        with torch.cuda.stream(strs[k]):
            dins[k].copy_(hosts[k], non_blocking=True)
            ww.nv12_decode(dins[k], OH, OW, out=douts[k], stream=strs[k])
            houts[k].copy_(douts[k], non_blocking=True)

    for i in range(6):
        e2e_step(i)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for st in strs:
        st.wait_stream(stream)
    n_e2e = max(3, min(args.steps, 60))
    for i in range(n_e2e):
        e2e_step(i)
    for st in strs:
        stream.wait_stream(st)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e = {"value": px * n_e2e / (f0.elapsed_time(f1) * 1e-3), "unit": "pixels/s",
           "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes, "steps": n_e2e, "streams": 3}
    peaks = load_peaks()
    gbs = (in_bytes + out_bytes) / (ms * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        n = oracle.nthreads_default()
        img = sets[0][0][:2].cpu().numpy()
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 5.0:
            oracle.nv12_decode(img, OH, OW, nthreads=n)
            reps += 1
        dt = time.perf_counter() - t0
        cpu = {"value": 2 * OH * OW * reps / dt, "unit": "pixels/s", "cores": n, "kind": "port",
               "sample": f"{reps} decodes of 2 frames in the C oracle, {dt:.1f} s"}
    line = {
        "metric": "nv12 decode output pixels/s", "value": value, "unit": "pixels/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u8->f16", "data": "synthetic (uniform random bytes)",
        "config": {"workload": f"nv12_decode: B={B} {H}x{W} NV12 -> 3x{OH}x{OW} fp16",
                   "l2": f"{n_sets} rotating input/output sets > 126 MB L2",
                   "timing": "the K launches replayed from one CUDA graph"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["src"]},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def corr_volume_e2e(ww, torch, dev_set, cfg, n, stream) -> dict:
    """CorrVolume end to end: pinned host features in, pinned host volume out,
    copies inside the timed region, three streams."""
    L0, R0, O0 = dev_set
    k3 = range(3)
    hl = [torch.empty(L0.shape, dtype=L0.dtype, pin_memory=True).copy_(L0) for _ in k3]
    hr = [torch.empty(R0.shape, dtype=R0.dtype, pin_memory=True).copy_(R0) for _ in k3]
    ho = [torch.empty(O0.shape, dtype=O0.dtype, pin_memory=True) for _ in k3]
    dl, dr, do = [torch.empty_like(L0) for _ in k3], [torch.empty_like(R0) for _ in k3], [torch.empty_like(O0) for _ in k3]
    strs = [torch.cuda.Stream() for _ in k3]

    def one(i):
        k = i % 3
        with torch.cuda.stream(strs[k]):
            dl[k].copy_(hl[k], non_blocking=True)
            dr[k].copy_(hr[k], non_blocking=True)
            ww.corr_volume(dl[k], dr[k], cfg.D, cfg.G, out=do[k], stream=strs[k])
            ho[k].copy_(do[k], non_blocking=True)

    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for st in strs:
        st.wait_stream(stream)
    for i in range(n):
        one(i)
    for st in strs:
        stream.wait_stream(st)
    f1.record(stream)
    torch.cuda.synchronize()
    vals = cfg.B * cfg.G * cfg.D * cfg.H * cfg.W
    return {"value": vals * n / (f0.elapsed_time(f1) * 1e-3), "unit": "values/s", "steps": n, "streams": 3}


def corr_volume_cpu(dev_set, cfg) -> dict:
    """The C oracle (the reference's fp32 channel-order sum and scale rule) on
    all host threads over a bounded sample of image rows, scaled to values/s."""
    import oracle
    n = oracle.nthreads_default()
    rows = max(1, min(cfg.H, 8))
    L = dev_set[0][:1, :, :rows].cpu().numpy()
    R = dev_set[1][:1, :, :rows].cpu().numpy()
    mode = oracle.grouped_scale_mode(True, cfg.B, cfg.C, cfg.G, cfg.H, cfg.W, cfg.D)
    t0 = time.perf_counter()
    reps = 0
    while time.perf_counter() - t0 < 5.0:
        oracle.corr_f16(L, R, cfg.D, cfg.G, scale_mode=mode, nthreads=n)
        reps += 1
    dt = time.perf_counter() - t0
    return {"value": cfg.G * cfg.D * rows * cfg.W * reps / dt, "unit": "values/s", "cores": n, "kind": "port",
            "sample": f"{reps} runs over rows [0,{rows}) of batch item 0 in the C oracle, {dt:.1f} s"}


def bench_corr_volume(args):
    """The reference's CorrVolume on a configuration's features (--config,
    default 2), group-wise: one step = one ww_corr_volume launch.  value:
    output values/s (B*G*D*H*W); roofline against HBM with bytes = both
    feature maps read once + the fp16 volume written."""
    import torch
    import whirlwind_trt_plugins_b200 as ww
    C_ = load_configs()
    cfg = C_.CONFIGS[args.config or CORR_VOLUME_CONFIG]
    if args.batch:
        cfg = cfg.scaled(B=args.batch)
    torch.cuda.set_device(0)
    B, C, G, H, W, D = cfg.B, cfg.C, cfg.G, cfg.H, cfg.W, cfg.D
    in_bytes, out_bytes = 2 * B * C * H * W * 2, B * G * D * H * W * 2
    n_sets = max(2, -(-400 * 2**20 // (in_bytes + out_bytes)))  # > 126 MB of L2
    sets = []
    for k in range(n_sets):
        x = C_.make_inputs_torch(cfg, torch.device("cuda", 0), seed=11 + k)
        sets.append((x["left"], x["right"], torch.empty((B, G, D, H, W), dtype=torch.float16, device="cuda")))
    stream = torch.cuda.current_stream()

    def step(i, st=None):
        L, R, o = sets[i % n_sets]
        ww.corr_volume(L, R, D, G, out=o, stream=st if st is not None else stream)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
        print(f"profile run: corr_volume {cfg.name}, {max(3, args.warmup)} + {args.steps} launches", flush=True)
        return
    graph = torch.cuda.CUDAGraph()  # launches of ~30 us: time the kernels, not the Python launch path
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap):
        for i in range(args.steps):
            step(i, torch.cuda.current_stream())
    stream.wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        t_end = time.time() + 1.0
        while time.time() < t_end:
            graph.replay()
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    del graph
    vals = B * G * D * H * W
    e2e = corr_volume_e2e(ww, torch, sets[0], cfg, max(3, min(args.steps, 20)), stream)
    e2e.update({"h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes})
    peaks = load_peaks()
    gbs = (in_bytes + out_bytes) / (ms * 1e-3) / 1e9
    cpu = None if args.no_cpu_baseline else corr_volume_cpu(sets[0], cfg)
    line = {
        "metric": "corr volume values/s (B*G*D*H*W)", "value": vals / (ms * 1e-3), "unit": "values/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic (the configuration's features)",
        "config": {"workload": f"corr_volume {workload_name(cfg)}",
                   "l2": f"{n_sets} rotating input/output sets > 126 MB L2",
                   "timing": "the K launches replayed from one CUDA graph"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": None, "peak_source": peaks["src"]},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


# Disparity regression workload: the aggregated cost of the batched config
# (config 4: B = 64, D = 48, 94 x 312), fp16 in and out, soft-argmin.
DISP_B, DISP_D, DISP_H, DISP_W = 64, 48, 94, 312
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of this workload
# (ncu capture: 180.2 MB read, the cost volume once, + 8.0 MB written)
DISP_NCU_TRAFFIC_BYTES = 188.2e6


def bench_disparity(args):
    """One step = ww_disparity_regression over a [DISP_B, DISP_D, DISP_H,
    DISP_W] fp16 cost (180 MB, larger than L2; two rotating sets).  value:
    output pixels/s; roofline against HBM with bytes = the cost read once +
    the fp16 disparity written."""
    import torch
    import whirlwind_trt_plugins_b200 as ww
    torch.cuda.set_device(0)
    B, D, H, W = DISP_B, DISP_D, DISP_H, DISP_W
    in_bytes, out_bytes = B * D * H * W * 2, B * H * W * 2
    n_sets = 2
    g = torch.Generator(device="cuda").manual_seed(3)
    sets = [((torch.randn((B, D, H, W), generator=g, device="cuda") * 2.0).half(),
             torch.empty((B, 1, H, W), dtype=torch.float16, device="cuda")) for _ in range(n_sets)]
    stream = torch.cuda.current_stream()
    mode = ww.DISP_SOFTARGMIN

    def step(i):
        x, o = sets[i % n_sets]
        ww.disparity_regression(x, mode, out=o, stream=stream)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.steps):
            step(i)
        torch.cuda.synchronize()
        print(f"profile run: disparity_regression, {max(3, args.warmup)} + {args.steps} launches", flush=True)
        return
    with ClockSampler(0) as clk:
        t_end = time.time() + 1.0
        i = 0
        while time.time() < t_end:
            step(i)
            i += 1
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    px = B * H * W
    value = px / (ms * 1e-3)
    e2e = None
    if not args.no_e2e:
        # end to end from pinned host memory: the cost up, the disparity back
        host = torch.empty((B, D, H, W), dtype=torch.float16, pin_memory=True)
        host.copy_(sets[0][0])
        hout = torch.empty((B, 1, H, W), dtype=torch.float16, pin_memory=True)
        din, dout = torch.empty_like(sets[0][0]), torch.empty_like(sets[0][1])

        def e2e_step():
            din.copy_(host, non_blocking=True)
            ww.disparity_regression(din, mode, out=dout, stream=stream)
            hout.copy_(dout, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        n_e2e = max(3, min(args.steps, 20))
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
        e2e = {"value": px * n_e2e / (f0.elapsed_time(f1) * 1e-3), "unit": "pixels/s",
               "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes, "steps": n_e2e}
    peaks = load_peaks()
    gbs = (in_bytes + out_bytes) / (ms * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline:
        import oracle
        n = oracle.nthreads_default()
        sample = sets[0][0][:2].cpu().numpy()
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 5.0:
            oracle.disparity_regression(sample, mode, out_f16=True, nthreads=n)
            reps += 1
        dt = time.perf_counter() - t0
        cpu = {"value": 2 * H * W * reps / dt, "unit": "pixels/s", "cores": n, "kind": "port",
               "sample": f"{reps} regressions of 2 of the {B} cost volumes in the C oracle, {dt:.1f} s"}
    line = {
        "metric": "disparity regression output pixels/s", "value": value, "unit": "pixels/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16->f32 math->f16",
        "data": "synthetic (cost ~ 2 N(0,1))",
        "config": {"workload": f"disparity_regression soft-argmin: cost [{B}, {D}, {H}, {W}] fp16 -> [{B}, 1, {H}, {W}]",
                   "l2": f"{n_sets} rotating sets of {in_bytes / 1e6:.0f} MB > 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "traffic": DISP_NCU_TRAFFIC_BYTES, "peak_source": peaks["src"]},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps, "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def bench_stem_volume(args):
    """The generalised CostStem3D (volume form, ww_cost_stem3d) on a
    configuration's group-wise volume (--config, default 2; --batch to scale):
    one step = one launch over a [B, G, D, H, W] fp16 volume made by
    ww_corr_volume from the configuration's features.  value: voxels/s
    (B*D*H*W); roofline against the tensor peak with the stem's FLOPs."""
    import torch
    import whirlwind_trt_plugins_b200 as ww
    C_ = load_configs()
    cfg = C_.CONFIGS[args.config or CORR_VOLUME_CONFIG]
    if args.batch:
        cfg = cfg.scaled(B=args.batch)
    torch.cuda.set_device(0)
    B, G, D, H, W, Cout = cfg.B, cfg.G, cfg.D, cfg.H, cfg.W, cfg.Cout
    vol_bytes, out_bytes = B * G * D * H * W * 2, B * Cout * D * H * W * 2
    n_sets = max(2, -(-400 * 2**20 // (vol_bytes + out_bytes)))  # > 126 MB of L2
    sets = []
    for k in range(n_sets):
        x = C_.make_inputs_torch(cfg, torch.device("cuda", 0), seed=21 + k)
        vol = ww.corr_volume(x["left"], x["right"], D, G)
        del x["left"], x["right"]
        sets.append((vol, x["w"], x["b"], torch.empty((B, Cout, D, H, W), dtype=torch.float16, device="cuda")))
    stream = torch.cuda.current_stream()

    def step(i, st):
        v, w, b, o = sets[i % n_sets]
        ww.cost_stem3d(v, w, b, act=cfg.act, out=o, stream=st)

    for i in range(max(3, args.warmup)):
        step(i, stream)
    torch.cuda.synchronize()
    if args.profile:
        for i in range(args.steps):
            step(i, stream)
        torch.cuda.synchronize()
        print(f"profile run: cost_stem3d {cfg.name}, {max(3, args.warmup)} + {args.steps} launches", flush=True)
        return
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream()
    cap.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap):
        for i in range(args.steps):
            step(i, torch.cuda.current_stream())
    stream.wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        t_end = time.time() + 1.0  # the sampler needs load for a few of its 200 ms periods
        while time.time() < t_end:
            graph.replay()
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    del graph
    voxels = B * D * H * W
    flops = 2.0 * B * Cout * G * 27 * D * H * W
    peaks = load_peaks()
    tf = flops / (ms * 1e-3) / 1e12
    line = {
        "metric": "cost voxels/s (B*D*H*W) 3D stem, volume form", "value": voxels / (ms * 1e-3),
        "unit": "voxels/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (the configuration's features through ww_corr_volume)",
        "config": {"workload": f"cost_stem3d {workload_name(cfg)}",
                   "l2": f"{n_sets} rotating volume/output sets > 126 MB L2",
                   "timing": "the K launches replayed from one CUDA graph"},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["tflops"], "unit": "TFLOP/s",
                     "frac": tf / peaks["tflops"], "traffic": None, "peak_source": peaks["src"],
                     "hbm_gbs": (vol_bytes + out_bytes) / (ms * 1e-3) / 1e9},
        "cpu_baseline": None, "e2e": None, "gpu_launches": args.steps, "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def bench_stem3_native(args):
    """The reference's 3-stage CostStem3D at its native shape [1, 1, 48, 32,
    40] (1 -> 4 -> 4 -> 1, ReLU6), alone (ww_cost_stem3d_ref3) and fused with
    its G = 1 correlation from C = 64 features (ww_corr_cost_stem3d_ref3):
    device time per call from a CUDA graph of K launches each."""
    import torch
    import whirlwind_trt_plugins_b200 as ww
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(7)
    ws = [(torch.randn((n,), generator=g, device="cuda") * s).half()
          for n, s in ((108, 0.2), (4, 0.1), (432, 0.2), (4, 0.1), (108, 0.2), (1, 0.1))]
    vol = torch.randn((1, 1, 48, 32, 40), generator=g, device="cuda").half()
    L = torch.randn((1, 64, 32, 40), generator=g, device="cuda").half()
    R = torch.randn((1, 64, 32, 40), generator=g, device="cuda").half()
    out = torch.empty_like(vol)
    calls = {"stem": lambda s: ww.cost_stem3d_ref3(vol, *ws, out=out, stream=s),
             "corr_stem": lambda s: ww.corr_cost_stem3d_ref3(L, R, *ws, max_disp=48, out=out, stream=s)}
    stream = torch.cuda.current_stream()
    if args.profile:
        for name in ("stem", "corr_stem"):
            for _ in range(max(3, args.warmup) + args.steps):
                calls[name](stream)
        torch.cuda.synchronize()
        print(f"profile run: stem3_native, {max(3, args.warmup)} + {args.steps} launches of each kernel", flush=True)
        return
    res = {}
    for name, fn in calls.items():
        for _ in range(3):
            fn(stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.graph(graph, stream=cap):
            for _ in range(args.steps):
                fn(torch.cuda.current_stream())
        stream.wait_stream(cap)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) * 1e3 / args.steps
        del graph
    vox = 48 * 32 * 40
    line = {"metric": "cost voxels/s, reference 3-stage CostStem3D at its native shape", "unit": UNIT,
            "value": vox / (res["stem"] * 1e-6), "us_per_call": res["stem"],
            "corr_stem_us_per_call": res["corr_stem"], "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "CostStem3D [1,1,48,32,40] (and CorrVolume G=1 from C=64 fused with it)",
                       "timing": "K launches replayed from one CUDA graph, L2-resident"},
            "gpu_launches": args.steps}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.op != "corr_cost_stem3d":
        if rank == 0 and args.impl == "ours":
            {"corr_volume": bench_corr_volume, "cost_stem3d": bench_stem_volume, "nv12_decode": bench_nv12, "disparity_regression": bench_disparity,
             "stem3_native": bench_stem3_native}[args.op](args)
        return
    if args.config is None:
        args.config = DEFAULT_CONFIG
    C = load_configs()
    cfg = C.CONFIGS[args.config]
    if cfg.Cout == 0:
        raise SystemExit("bench.py measures the fused front end; config %d has no stem" % args.config)
    if args.batch:
        cfg = cfg.scaled(B=args.batch)
    if args.impl == "reference":
        run_reference(args, C, cfg, rank, world)
        return
    bench_main(args, C, cfg, world, rank, local)


if __name__ == "__main__":
    main()
