"""Row sharding of the fused op over NCCL on 2 GPUs (skipped with fewer):
each rank holds its rows of the features, fetches a one-row halo from each
neighbour by send/recv, runs the band kernel, and the all-gathered result
must equal the unsharded kernel bit for bit.  NVLS is off (NCCL_NVLS_ENABLE=0)
and the op's own kernels read only local memory."""
import os
import socket
import multiprocessing as mp

import numpy as np
import pytest

from conftest import ROOT

SHAPE = dict(B=1, C=64, G=8, H=37, W=48, D=24, Cout=16)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import sys
    import datetime
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import whirlwind_trt_plugins_b200 as ww
        from whirlwind_trt_plugins_b200 import shard
        s = SHAPE
        g = torch.Generator(device="cuda").manual_seed(3)
        L = torch.randn((s["B"], s["C"], s["H"], s["W"]), generator=g, device="cuda").half()
        R = torch.randn((s["B"], s["C"], s["H"], s["W"]), generator=g, device="cuda").half()
        w = (torch.randn((s["Cout"], s["G"], 3, 3, 3), generator=g, device="cuda") * 0.1).half()
        b = (torch.randn((s["Cout"],), generator=g, device="cuda") * 0.1).half()
        r0, r1 = shard.split_even(s["H"], world, rank)
        out = shard.corr_cost_stem3d_rows(L[:, :, r0:r1].contiguous(), R[:, :, r0:r1].contiguous(), w, b,
                                          s["D"], s["G"], s["H"])
        full = shard.gather_rows(out, s["H"])
        ref = ww.corr_cost_stem3d(L, R, w, b, s["D"], s["G"])
        torch.cuda.synchronize()
        same = bool(torch.equal(full, ref))
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{int(same)} {ww.device_error()}")
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_row_sharded_fused_matches_unsharded(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    assert codes == [0, 0], codes
    for r in range(world):
        same, err = (tmp_path / f"rank{r}.txt").read_text().split()
        assert same == "1" and err == "0"
