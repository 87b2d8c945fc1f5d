"""
The host side of tile-row bands on CPU ranks (gloo, world size 2, 127.0.0.1), with the oracle standing in for the GPU kernels: each rank
renders the image, keeps the L1 gradient of its own rows only (normalised by the whole image's pixel count), back-propagates, and the
ranks sum their partial gradients and losses with one all-reduce; every rank then finishes the projection backward. The result must equal
the single-process step. A second test makes a rank die before the all-reduce: the survivor's collective must fail within the process
group's timeout instead of hanging.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def init(rank, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=timeout_s))


def band_step_on_cpu(rank, port):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "image-gs_b200"), os.path.join(root, "tests")]
    from common import assert_close_grad
    from igs_b200 import bands, workloads
    from oracle import cpu

    init(rank, port)
    try:
        wl = workloads.custom_workload(100, 120, 400, seed=81)
        inp = workloads.make_inputs(wl)
        a = [inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")]
        h, w = wl.height, wl.width
        full = cpu.train_step(*a, h, w)
        r0, r1 = bands.band_rows(wl.tile_bounds[1], WORLD, rank)
        rows = slice(16 * r0, min(h, 16 * r1))
        diff = full["image"] - a[4]
        v_out = np.zeros_like(full["image"])
        v_out[:, rows] = (np.sign(diff[:, rows]) * np.float32(1.0 / diff.size)).astype(np.float32)
        loss = float(np.abs(diff[:, rows].astype(np.float64)).sum() / diff.size)
        v_xy, v_conic, v_colors = cpu.raster_bwd(h, w, full["xys"], full["conics"], a[3], v_out, full["pixel_topk"])
        buf = torch.from_numpy(np.concatenate([v_xy.ravel(), v_conic.ravel(), v_colors.ravel(), np.array([loss], np.float32)]))
        dist.all_reduce(buf)
        n = len(a[0])
        r_xy, r_conic = buf[:2 * n].numpy().reshape(n, 2), buf[2 * n:5 * n].numpy().reshape(n, 3)
        r_colors = buf[5 * n:-1].numpy().reshape(n, 3)
        _, v_mean2d, v_scale, v_rot = cpu.project_bwd(a[1], a[2], h, w, full["radii"], full["conics"], r_xy, r_conic)
        assert abs(float(buf[-1]) - full["loss"]) <= 1e-5 * full["loss"]
        for got, key in ((r_colors, "v_colors"), (v_mean2d, "v_mean2d"), (v_scale, "v_scale"), (v_rot, "v_rot")):
            assert_close_grad(got, full[key], what=key)
    finally:
        dist.destroy_process_group()


def dying_rank(rank, port):
    init(rank, port, timeout_s=10)
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective, without a GPU involved
    buf = torch.ones(16)
    try:
        dist.all_reduce(buf)
    except Exception:  # the expected outcome: the collective fails instead of waiting forever
        os._exit(0)
    os._exit(3)


def test_band_all_reduce_matches_single_process():
    mp.spawn(band_step_on_cpu, args=(free_port(),), nprocs=WORLD, join=True)


@pytest.mark.timeout(120)
def test_lost_rank_fails_the_collective_instead_of_hanging():
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=dying_rank, args=(r, port)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
