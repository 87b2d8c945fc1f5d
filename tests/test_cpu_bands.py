"""
The host side of tile-row bands on CPU ranks (gloo, world sizes 2 and 3, 127.0.0.1): igs_b200.bands.BandStep itself, with the oracle
standing in for its GPU kernels. Each rank's step bins and renders its rows, takes the L1 loss of its rows normalised by the whole image's
pixel count and back-propagates them into the step's exchange buffer; the product's all-reduce sums the ranks' buffers and every rank
finishes the projection backward. The result must equal the single-process step, and every rank must hold the same gradients. A second
test makes a rank die before the all-reduce: the survivor's collective must fail within the process group's timeout instead of hanging.
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


def init(rank, port, timeout_s=60, world=WORLD):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def oracle_band_step_class():
    """bands.BandStep with the oracle standing in for its GPU kernels (a test double): each kernel stage is overridden to fill the same
    buffers the CUDA kernels fill, so the band's buffer layout, the one all-reduce of its partial gradients and loss, the launch order and
    the projection backward on the reduced data are the product's own code."""
    from igs_b200 import bands
    from oracle import cpu

    def arr(t):
        return t.detach().numpy()

    class OracleBandStep(bands.BandStep):
        def _whole_lists(self):
            xys, radii = arr(self.xys), arr(self.radii)
            hits = arr(self.hits)
            total = int(hits.astype(np.int64).sum())
            return cpu.sort_intersects(self.n, total, xys, radii, cpu.cumsum(hits), self.h, self.w)

        def _project(self):
            xys, radii, conics, hits = cpu.project_fwd(arr(self.means), arr(self.scales), arr(self.rotations), self.h, self.w)
            for dst, src in ((self.xys, xys), (self.radii, radii), (self.conics, conics), (self.hits, hits)):
                dst.copy_(torch.from_numpy(src))
            # igs_band_tiles_hit: the tiles of the band's rows that each Gaussian hits
            ids, bins = self._whole_lists()
            t0, t1 = self.r0 * self.tb[0], self.r1 * self.tb[0]
            lengths = bins[:, 1] - bins[:, 0]
            band = np.concatenate([ids[bins[t, 0]:bins[t, 1]] for t in range(t0, t1) if lengths[t] > 0] or [np.zeros(0, np.int32)])
            self.band_hits.copy_(torch.from_numpy(np.bincount(band, minlength=self.n).astype(np.int32)))

        def _cumsum(self):
            cum = cpu.cumsum(arr(self.band_hits))
            self.cum.copy_(torch.from_numpy(cum))
            self.num_intersects.fill_(int(cum[-1]) if len(cum) else 0)

        def _bin(self):
            # igs_sort_intersects_band: the whole image's lists of the band's tiles, tile_bins relative to the band's list
            ids, bins = self._whole_lists()
            t0, t1 = self.r0 * self.tb[0], self.r1 * self.tb[0]
            self.ids.zero_()
            self.bins.zero_()
            at = 0
            for t in range(t0, t1):
                n = int(bins[t, 1] - bins[t, 0])
                if n > 0:
                    self.ids[at:at + n] = torch.from_numpy(ids[bins[t, 0]:bins[t, 1]])
                    self.bins[t - t0] = torch.tensor([at, at + n], dtype=torch.int32)
                    at += n

        def _raster(self):
            # igs_raster_step_l1_band: the band's rows of the render, their L1 loss and its gradient normalised by the whole image's
            # pixel count, and the backward pass of those rows
            ids, bins = self._whole_lists()
            colors = arr(self.features)
            image, topk = cpu.raster_fwd(self.h, self.w, ids, bins, arr(self.xys), arr(self.conics), colors)
            rows = slice(self.px0, self.px0 + self.band_h)
            self.image.copy_(torch.from_numpy(np.ascontiguousarray(image[:, rows])))
            d = image[:, rows] - arr(self.target)
            v_out = np.zeros_like(image)
            v_out[:, rows] = (np.sign(d) * np.float32(np.float32(self.l1_ratio) / np.float32(image.size))).astype(np.float32)
            v_xy, v_conic, v_colors = cpu.raster_bwd(self.h, self.w, arr(self.xys), arr(self.conics), colors, v_out, topk)
            self.v_xy.copy_(torch.from_numpy(v_xy))
            self.v_conic.copy_(torch.from_numpy(v_conic))
            self.v_colors.copy_(torch.from_numpy(v_colors))
            self.loss.fill_(self.l1_ratio * float(np.abs(d.astype(np.float64)).sum() / image.size))

        def _train_step(self):
            # igs_train_step_l1 over the band's rows: the same buffers as the stages one by one
            self._project()
            self._cumsum()
            self._bin()
            self._raster()

        def _project_backward(self):
            v_cov2d, v_mean2d, v_scale, v_rot = cpu.project_bwd(arr(self.scales), arr(self.rotations), self.h, self.w, arr(self.radii),
                                                                arr(self.conics), arr(self.v_xy), arr(self.v_conic))
            for dst, src in ((self.v_cov2d, v_cov2d), (self.v_mean2d, v_mean2d), (self.v_scale, v_scale), (self.v_rot, v_rot)):
                dst.copy_(torch.from_numpy(src).view_as(dst))

    return OracleBandStep


def band_step_on_cpu(rank, port, world):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "image-gs_b200"), os.path.join(root, "tests")]
    from common import assert_close_grad
    from igs_b200 import bands, workloads
    from oracle import cpu

    init(rank, port, world=world)
    try:
        wl = workloads.custom_workload(100, 120, 400, seed=81)
        inp = workloads.make_inputs(wl)
        h, w = wl.height, wl.width
        full = cpu.train_step(*[inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")], h, w)
        r0, r1 = bands.band_rows(wl.tile_bounds[1], world, rank)
        step = oracle_band_step_class()(inp["means"], inp["scales"], inp["rotations"], inp["features"], inp["target"], h, w, r0, r1,
                                        group=dist.group.WORLD)
        assert step.target.shape[1] == step.band_h  # the band keeps only its rows of the target
        step.launch()  # kernels of the band, the product's all-reduce of step.reduced, the projection backward
        assert abs(float(step.loss) - full["loss"]) <= 1e-5 * full["loss"]
        for key in ("v_xy", "v_conic", "v_colors", "v_mean2d", "v_scale", "v_rot"):
            assert_close_grad(getattr(step, key).numpy(), full[key].reshape(getattr(step, key).shape), what=key)
        # every rank ends with the same parameter gradients, bit for bit
        mine = torch.cat([step.v_mean2d.view(-1), step.v_scale.view(-1), step.v_rot.view(-1), step.v_colors.view(-1)])
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        assert all(torch.equal(g, gathered[0]) for g in gathered)
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


@pytest.mark.parametrize("world", [2, 3])
def test_band_step_exchange_matches_single_process(world):
    mp.spawn(band_step_on_cpu, args=(free_port(), world), nprocs=world, join=True)


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
