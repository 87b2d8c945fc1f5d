"""
Tile-row bands across two GPUs over NCCL (one process per GPU, 127.0.0.1 rendezvous): each rank bins, renders and back-propagates its
band, the partial gradients and loss are summed with one NCCL all-reduce, and every rank finishes the projection backward. Every rank's
parameter gradients and loss must equal the single-GPU step's on the same inputs, both for eager launches and for the CUDA-graph replay.
Skipped with fewer than two GPUs.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WORLD = 2


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def band_rank(rank, port):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "image-gs_b200"), os.path.join(root, "tests")]
    from common import assert_close_grad, make_case, to_dev
    from igs_b200 import bands, pipeline

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60), device_id=device)
    try:
        wl, inp = make_case(200, 330, 1500, seed=91)
        d = to_dev(inp, device)
        h, w = wl.height, wl.width
        full = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"])
        full.launch()
        r0, r1 = bands.band_rows_balanced(d["means"], d["scales"], d["rotations"], h, w, WORLD, rank)
        step = bands.BandStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], h, w, r0, r1, group=dist.group.WORLD,
                              capacity=full.capacity)
        for mode in ("launch", "replay", "replay"):
            getattr(step, mode)()
            torch.cuda.synchronize()
            for key in ("v_colors", "v_mean2d", "v_scale", "v_rot"):
                assert_close_grad(getattr(step, key), getattr(full, key), what=f"{key} ({mode})")
            assert abs(float(step.loss) - float(full.loss)) <= 1e-5 * float(full.loss)
        step.release()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_bands_over_nccl_match_single_gpu():
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    mp.spawn(band_rank, args=(free_port(),), nprocs=WORLD, join=True)
