"""
Tile-row bands across two GPUs (one process per GPU, 127.0.0.1 rendezvous, NVLS off): each rank bins, renders and back-propagates its
band; the partial gradients and loss are combined either by one NCCL all-reduce followed by the projection backward on every rank, or by
the peer-memory exchange (igs_band_reduce over CUDA IPC mappings, plain peer loads and stores). Every rank's parameter gradients and loss
must equal the single-GPU step's on the same inputs, for eager launches and for the CUDA-graph replay; with the peer exchange every rank
must hold bit-identical gradients. Skipped with fewer than two GPUs.
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


def band_rank(rank, port, exchange):
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
                              capacity=full.capacity, exchange=exchange)
        assert step.exchange == exchange
        for mode in ("launch", "replay", "replay"):
            getattr(step, mode)()
            torch.cuda.synchronize()
            step.check()
            for key in ("v_colors", "v_mean2d", "v_scale", "v_rot"):
                assert_close_grad(getattr(step, key), getattr(full, key), what=f"{key} ({mode})")
            assert abs(float(step.loss) - float(full.loss)) <= 1e-5 * float(full.loss)
            mine = torch.cat([getattr(step, k).reshape(-1) for k in ("v_colors", "v_mean2d", "v_scale", "v_rot", "v_cov2d")])
            gathered = [torch.empty_like(mine) for _ in range(WORLD)]
            dist.all_gather(gathered, mine)
            assert all(torch.equal(g, gathered[0]) for g in gathered)
        if exchange == "peer":
            # launch, the graph capture's warm-up run, and the two replays: four exchanges, every wait met
            assert step.peer.steps() == 4 and step.peer.error() == 0
        step.release()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_bands_on_two_gpus_match_single_gpu(exchange):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    mp.spawn(band_rank, args=(free_port(), exchange), nprocs=WORLD, join=True)
