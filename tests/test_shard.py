"""Host logic of the multi-GPU sharding (whirlwind_trt_plugins_b200.shard) on
CPU: gloo process groups of 2 and 3 ranks on 127.0.0.1.

The per-rank compute is the plain-C oracle (the checker) run on each rank's
band, so these tests check the partitioning, the halo exchange and the
stitching: the stitched rows must equal the unsharded oracle bit for bit.
The CUDA band kernel itself is checked against the unsharded kernel in
tests/test_gpu_stem.py and over NCCL in tests/test_gpu_shard.py."""
import os
import socket
import multiprocessing as mp

import numpy as np
import pytest

from conftest import ROOT

SHAPE = dict(B=1, C=16, G=4, H=7, W=16, D=8, Cout=8)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(11)
    s = SHAPE
    L = rng.standard_normal((s["B"], s["C"], s["H"], s["W"])).astype(np.float16)
    R = rng.standard_normal((s["B"], s["C"], s["H"], s["W"])).astype(np.float16)
    w = (rng.standard_normal((s["Cout"], s["G"], 3, 3, 3)) * 0.2).astype(np.float16)
    b = (rng.standard_normal(s["Cout"]) * 0.1).astype(np.float16)
    return L, R, w, b


def _oracle_band_fn(scale_mode):
    import torch
    import oracle

    def fn(lb, rb, w, b, D, G, H, i0, out_row0, out_rows, act):
        band = oracle.corr_stem(lb.numpy(), rb.numpy(), w.numpy(), b.numpy(), D, G, act=act,
                                scale_mode=scale_mode)
        k = out_row0 - i0
        return torch.from_numpy(np.ascontiguousarray(band[:, :, :, k:k + out_rows]))
    return fn


def _init(rank, world, port, timeout_s=20):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _rows_worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import oracle
    from whirlwind_trt_plugins_b200 import shard
    dist = _init(rank, world, port)
    try:
        s = SHAPE
        L, R, w, b = _inputs()
        sm = oracle.grouped_scale_mode(True, s["B"], s["C"], s["G"], s["H"], s["W"], s["D"])
        r0, r1 = shard.split_even(s["H"], world, rank)
        lt = torch.from_numpy(np.ascontiguousarray(L[:, :, r0:r1]))
        rt = torch.from_numpy(np.ascontiguousarray(R[:, :, r0:r1]))
        band, i0 = shard.exchange_halo(lt, s["H"])
        i0e, i1e = shard.halo_rows(s["H"], r0, r1)
        assert i0 == i0e and band.shape[2] == i1e - i0e
        np.save(os.path.join(outdir, f"band{rank}.npy"), band.numpy())
        out = shard.corr_cost_stem3d_rows(lt, rt, torch.from_numpy(w), torch.from_numpy(b), s["D"], s["G"],
                                          s["H"], act=0, band_fn=_oracle_band_fn(sm))
        full = shard.gather_rows(out, s["H"])
        np.save(os.path.join(outdir, f"full{rank}.npy"), full.numpy())
    finally:
        dist.destroy_process_group()


def _run(world, target, args, timeout=120):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return codes


def test_split_even_and_halo():
    from whirlwind_trt_plugins_b200.shard import split_even, halo_rows
    for n in (0, 1, 7, 120, 181):
        for world in (1, 2, 3, 8):
            parts = [split_even(n, world, k) for k in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
            sizes = [e - s for s, e in parts]
            assert max(sizes) - min(sizes) <= 1
    assert halo_rows(10, 0, 5) == (0, 6)
    assert halo_rows(10, 5, 10) == (4, 10)
    assert halo_rows(10, 3, 6) == (2, 7)
    with pytest.raises(ValueError):
        split_even(4, 2, 2)


@pytest.mark.parametrize("world", [2, 3])
def test_row_shards_stitch_to_unsharded_oracle(orc, tmp_path, world):
    codes = _run(world, _rows_worker, (str(tmp_path),))
    assert codes == [0] * world, codes
    s = SHAPE
    L, R, w, b = _inputs()
    sm = orc.grouped_scale_mode(True, s["B"], s["C"], s["G"], s["H"], s["W"], s["D"])
    ref = orc.corr_stem(L, R, w, b, s["D"], s["G"], act=0, scale_mode=sm)
    from whirlwind_trt_plugins_b200.shard import split_even, halo_rows
    for r in range(world):
        full = np.load(tmp_path / f"full{r}.npy")
        assert full.shape == ref.shape
        assert np.array_equal(full.view(np.uint16), ref.view(np.uint16))
        r0, r1 = split_even(s["H"], world, r)
        i0, i1 = halo_rows(s["H"], r0, r1)
        band = np.load(tmp_path / f"band{r}.npy")
        assert np.array_equal(band.view(np.uint16), L[:, :, i0:i1].view(np.uint16))


def _failing_worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    from whirlwind_trt_plugins_b200 import shard
    dist = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        # this rank fails before its halo exchange and leaves
        os._exit(3)
    err = "none"
    try:
        x = torch.zeros((1, 2, 4, 8), dtype=torch.float16)
        shard.exchange_halo(x, 8)
    except Exception as e:  # the surviving rank must see an error, not hang
        err = type(e).__name__
    with open(os.path.join(outdir, f"err{rank}.txt"), "w") as f:
        f.write(err)
    os._exit(0)


def test_failed_rank_surfaces_as_error(tmp_path):
    codes = _run(2, _failing_worker, (str(tmp_path),), timeout=90)
    assert codes[1] == 3
    assert codes[0] == 0, codes
    err = (tmp_path / "err0.txt").read_text()
    assert err != "none"


def test_rows_rejects_wrong_local_shape(tmp_path):
    codes = _run(2, _bad_shape_worker, (str(tmp_path),))
    assert codes == [0, 0], codes
    assert (tmp_path / "bad0.txt").read_text() == "ValueError"


def _bad_shape_worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    from whirlwind_trt_plugins_b200 import shard
    dist = _init(rank, world, port)
    try:
        x = torch.zeros((1, 2, 3, 8), dtype=torch.float16)  # should hold 4 of 8 rows
        try:
            shard.exchange_halo(x, 8)
            res = "none"
        except ValueError:
            res = "ValueError"
        with open(os.path.join(outdir, f"bad{rank}.txt"), "w") as f:
            f.write(res)
    finally:
        dist.destroy_process_group()


def _haloband_worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    from whirlwind_trt_plugins_b200 import shard
    dist = _init(rank, world, port)
    try:
        s = SHAPE
        L, _, _, _ = _inputs()
        hb = shard.HaloBand(s["B"], s["C"], s["H"], s["W"], torch.float16, "cpu")
        hb.own.copy_(torch.from_numpy(np.ascontiguousarray(L[:, :, hb.r0:hb.r1])))
        for _ in range(2):  # repeated exchanges reuse the same buffers
            hb.exchange()
        np.save(os.path.join(outdir, f"hb{rank}.npy"), hb.band.numpy())
        with open(os.path.join(outdir, f"hb{rank}.txt"), "w") as f:
            f.write(f"{hb.i0} {hb.i1}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_haloband_holds_rows_and_halo(tmp_path, world):
    codes = _run(world, _haloband_worker, (str(tmp_path),))
    assert codes == [0] * world, codes
    L, _, _, _ = _inputs()
    from whirlwind_trt_plugins_b200.shard import split_even, halo_rows
    for r in range(world):
        i0, i1 = (int(v) for v in (tmp_path / f"hb{r}.txt").read_text().split())
        r0, r1 = split_even(SHAPE["H"], world, r)
        assert (i0, i1) == halo_rows(SHAPE["H"], r0, r1)
        band = np.load(tmp_path / f"hb{r}.npy")
        assert np.array_equal(band.view(np.uint16), L[:, :, i0:i1].view(np.uint16))


def _soak_worker(rank, world, port, outdir):
    """Steps that each take a collective (as the row-band bench's halo
    exchange does), with per-rank step times that differ: a soak by step count
    keeps every rank on the same collective calls."""
    import sys
    import time
    sys.path.insert(0, ROOT)
    import torch
    import bench
    dist = _init(rank, world, port, timeout_s=15)
    try:
        t = torch.zeros(1)

        def step(i):
            time.sleep(0.002 * (rank + 1))  # rank-dependent step time
            t.fill_(i)
            dist.all_reduce(t)

        n = bench.soak(step, 0.0, 12, lambda: None)
        dist.barrier()
        np.save(os.path.join(outdir, f"soak{rank}.npy"), np.array([n, float(t.item())]))
    finally:
        dist.destroy_process_group()


def test_bench_soak_by_count_keeps_ranks_in_step(tmp_path):
    codes = _run(3, _soak_worker, (str(tmp_path),), timeout=60)
    assert codes == [0, 0, 0]
    got = [np.load(tmp_path / f"soak{r}.npy") for r in range(3)]
    assert all(g[0] == 12 for g in got)
    assert all(g[1] == 3 * 11 for g in got)  # the last step's all-reduce of i = 11 over 3 ranks
