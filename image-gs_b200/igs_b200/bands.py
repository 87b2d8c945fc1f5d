"""
One image split into tile-row bands across GPUs (one process per GPU): the Gaussian parameters are replicated; every rank projects all
Gaussians, bins and renders only its rows, takes the L1 loss and its gradient on its rows (normalised by the whole image's pixel count),
and runs the backward pass for its band. The partial gradients with respect to the projected Gaussians (v_xy, v_conic, v_colors:
N (5 + C) floats, 2.6 MB at 80,000 Gaussians) and the partial loss are summed over the ranks with one NCCL all-reduce; every rank then
finishes the projection backward on identical data, so all ranks hold the same parameter gradients.

The band's tile lists, renders and per-pixel gradients equal the matching rows of the single-GPU step bit for bit (pixel coordinates are
the image's); the summed gradients differ from the single-GPU ones only in the order of float additions.
"""
import ctypes
from typing import Optional, Sequence

import torch

from . import _lib, ops
from ._lib import ptr

TILE = ops.TILE
TOP_K = ops.TOP_K


def band_rows(tiles_y: int, world: int, rank: int, row_weights: Optional[Sequence[float]] = None):
    """Tile rows [begin, end) of `rank`'s band: contiguous bands, with equal row counts or, given per-row work estimates (e.g. the
    intersections per tile row), balanced so that each band holds about 1/world of the total."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if row_weights is None:
        return (tiles_y * rank) // world, (tiles_y * (rank + 1)) // world
    w = [float(x) for x in row_weights]
    if len(w) != tiles_y:
        raise ValueError("one weight per tile row")
    total = sum(w)
    bounds, acc, row = [0], 0.0, 0
    for r in range(1, world):
        target = total * r / world
        while row < tiles_y and acc + w[row] <= target:
            acc += w[row]
            row += 1
        bounds.append(max(row, bounds[-1]))
    bounds.append(tiles_y)
    return bounds[rank], bounds[rank + 1]


def row_intersections(means, scales, rotations, img_h, img_w):
    """Tile-list entries per tile row of the whole image ([tiles_y] int64 on the host): one projection and binning pass, the work
    estimate that band_rows balances."""
    n = means.shape[0]
    tb = ops.tile_grid(img_h, img_w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, means, scales, rotations, img_h, img_w, tb)
    cum, total = ops.cumulative_intersects(hits)
    total = int(total.item())
    if total < 1:
        return [0] * tb[1]
    _, bins = ops.sort_intersects_by_tile(n, total, xys, radii, cum, tb)
    lengths = (bins[:, 1] - bins[:, 0]).to(torch.int64).view(tb[1], tb[0])
    return lengths.sum(1).cpu().tolist()


def band_rows_balanced(means, scales, rotations, img_h, img_w, world, rank, entry_weight=1.0, tile_weight=32.0):
    """band_rows weighted by each tile row's estimated cost: entry_weight per tile-list entry plus tile_weight per tile (the per-pixel
    work that does not depend on the lists)."""
    tiles_x, tiles_y, _ = ops.tile_grid(img_h, img_w)
    per_row = row_intersections(means, scales, rotations, img_h, img_w)
    return band_rows(tiles_y, world, rank, [entry_weight * r + tile_weight * tiles_x for r in per_row])


class BandStep:
    """One rank's share of a step. Device tensors: means [N,2], scales [N,2], rotations [N,1], features [N,C] (replicated), the whole
    target [C,H,W] or just its band rows; rows [row_begin, row_end) are tile rows. group: a torch.distributed process group (None: a
    single band, no communication)."""

    def __init__(self, means, scales, rotations, features, target, img_h, img_w, row_begin, row_end, group=None, capacity=None,
                 capacity_ratio: float = 2.0, l1_ratio: float = 1.0, fused: bool = True):
        self.lib = _lib.load()
        self.fused = fused  # the band's forward, loss and backward in one kernel (igs_raster_step_l1_band); else two kernels
        self.device = means.device
        self.n, self.c = features.shape
        self.h, self.w = img_h, img_w
        self.tb = ops.tile_grid(img_h, img_w)
        self.r0, self.r1 = int(row_begin), int(row_end)
        self.px0 = self.r0 * TILE
        self.band_h = max(0, min(img_h, self.r1 * TILE) - self.px0)
        self.num_tiles = self.tb[0] * (self.r1 - self.r0)
        self.group = group
        self.means, self.scales, self.rotations, self.features = means, scales, rotations, features
        if target.shape[1] == img_h:
            target = target[:, self.px0:self.px0 + self.band_h]
        self.target = target.contiguous()
        dev, f32, i32, n, nc = self.device, torch.float32, torch.int32, self.n, self.c
        self.xys = torch.empty(n, 2, device=dev, dtype=f32)
        self.radii = torch.empty(n, device=dev, dtype=i32)
        self.conics = torch.empty(n, 3, device=dev, dtype=f32)
        self.hits = torch.empty(n, device=dev, dtype=i32)
        self.band_hits = torch.empty(n, device=dev, dtype=i32)
        self.cum = torch.empty(n, device=dev, dtype=i32)
        self.num_intersects = torch.empty(1, device=dev, dtype=i32)
        self.cum_ws_bytes = self.lib.igs_cumsum_workspace(n)
        self.cum_ws = torch.empty(self.cum_ws_bytes, device=dev, dtype=torch.uint8)
        self.image = torch.empty(nc, self.band_h, img_w, device=dev, dtype=f32)
        self.v_image = None if fused else torch.empty_like(self.image)
        # the band's loss is its share of the whole image's, ratio * sum over the band |d| / (C H W), computed by the forward kernel
        self.l1_ratio = float(l1_ratio)
        self.l1_ws_bytes = self.lib.igs_raster_l1_workspace(max(1, self.num_tiles))
        self.l1_ws = torch.zeros(self.l1_ws_bytes, device=dev, dtype=torch.uint8)
        # one buffer for the all-reduce: the partial gradients, then the partial loss
        self.reduced = torch.empty(n * (5 + nc) + 1, device=dev, dtype=f32)
        self.v_xy = self.reduced[:2 * n].view(n, 2)
        self.v_conic = self.reduced[2 * n:5 * n].view(n, 3)
        self.v_colors = self.reduced[5 * n:n * (5 + nc)].view(n, nc)
        self.loss = self.reduced[n * (5 + nc)]
        self.v_cov2d = torch.empty(n, 3, device=dev, dtype=f32)
        self.v_mean2d = torch.empty(n, 2, device=dev, dtype=f32)
        self.v_scale = torch.empty(n, 2, device=dev, dtype=f32)
        self.v_rot = torch.empty(n, 1, device=dev, dtype=f32)
        if capacity is None:
            self._project()
            self._cumsum()
            capacity = max(1024, round(capacity_ratio * int(self.num_intersects.item())))
        self.capacity = int(capacity)
        self.ids = torch.empty(self.capacity, device=dev, dtype=i32)
        self.bins = torch.empty(max(1, self.num_tiles), 2, device=dev, dtype=i32)
        self.sort_ws_bytes = self.lib.igs_sort_workspace(self.capacity, self.tb[0], self.r1 - self.r0)
        self.sort_ws = torch.empty(self.sort_ws_bytes, device=dev, dtype=torch.uint8)
        self.max_list = min(self.n, self.capacity)
        self.topk = None if fused else torch.empty(max(1, self.num_tiles), TOP_K, TILE * TILE, device=dev, dtype=torch.int16)
        self.local_graph = self.final_graph = None

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _project(self):
        _lib.check(self.lib.igs_project_fwd(self.n, ptr(self.means), ptr(self.scales), ptr(self.rotations), self.h, self.w, self.tb[0],
                                            self.tb[1], ptr(self.xys), ptr(self.radii), ptr(self.conics), ptr(self.hits), self._stream()),
                   "project")
        _lib.check(self.lib.igs_band_tiles_hit(self.n, ptr(self.xys), ptr(self.radii), self.tb[0], self.tb[1], self.r0, self.r1,
                                               ptr(self.band_hits), self._stream()), "band tiles")

    def _cumsum(self):
        _lib.check(self.lib.igs_cumsum(self.n, ptr(self.band_hits), ptr(self.cum), ptr(self.num_intersects), ptr(self.cum_ws),
                                       self.cum_ws_bytes, self._stream()), "cumsum")

    def _bin(self):
        _lib.check(self.lib.igs_sort_intersects_band(self.n, self.capacity, ptr(self.xys), ptr(self.radii), ptr(self.cum), self.tb[0],
                                                     self.tb[1], self.r0, self.r1, ptr(self.ids), ptr(self.bins), ptr(self.sort_ws),
                                                     self.sort_ws_bytes, self._stream()), "bin")

    def _raster(self):
        _lib.check(self.lib.igs_raster_step_l1_band(self.tb[0], self.tb[1], self.h, self.w, self.r0, self.r1, self.c, self.n, ptr(self.ids),
                                                    ptr(self.bins), ptr(self.xys), ptr(self.conics), ptr(self.features), ptr(self.target),
                                                    self.l1_ratio, ptr(self.image), ptr(self.loss), None, ptr(self.v_xy), ptr(self.v_conic),
                                                    ptr(self.v_colors), ptr(self.l1_ws), self.l1_ws_bytes, self._stream()), "raster step")

    def _forward(self):
        if self.num_tiles == 0:
            self.loss.zero_()
            return
        _lib.check(self.lib.igs_raster_fwd_topk_tiles_l1_band(self.tb[0], self.tb[1], self.h, self.w, self.r0, self.r1, self.c, self.max_list,
                                                              ptr(self.ids), ptr(self.bins), ptr(self.xys), ptr(self.conics),
                                                              ptr(self.features), ptr(self.target), self.l1_ratio, ptr(self.image),
                                                              ptr(self.topk), ptr(self.loss), ptr(self.v_image), ptr(self.l1_ws),
                                                              self.l1_ws_bytes, self._stream()), "forward")

    def _backward(self):
        _lib.check(self.lib.igs_raster_bwd_topk_tiles_band(self.h, self.w, self.r0, self.r1, self.c, self.n, ptr(self.ids), ptr(self.bins),
                                                           ptr(self.xys), ptr(self.conics), ptr(self.features), ptr(self.v_image),
                                                           ptr(self.topk), ptr(self.v_xy), ptr(self.v_conic), ptr(self.v_colors),
                                                           self._stream()), "backward")

    def _project_backward(self):
        _lib.check(self.lib.igs_project_bwd(self.n, ptr(self.scales), ptr(self.rotations), self.h, self.w, ptr(self.radii), ptr(self.conics),
                                            ptr(self.v_xy), ptr(self.v_conic), ptr(self.v_cov2d), ptr(self.v_mean2d), ptr(self.v_scale),
                                            ptr(self.v_rot), self._stream()), "project_backward")

    KERNELS = {"_project": 2, "_cumsum": 2, "_bin": 4, "_raster": 2, "_forward": 2, "_backward": 1, "_project_backward": 1}

    @property
    def LOCAL(self):
        return ("_project", "_cumsum", "_bin") + (("_raster",) if self.fused else ("_forward", "_backward"))

    def all_reduce(self):
        if self.group is not None:
            torch.distributed.all_reduce(self.reduced, group=self.group)

    def launch(self):
        for s in self.LOCAL:
            getattr(self, s)()
        self.all_reduce()
        self._project_backward()

    def _capture(self, stages):
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for s in stages:
                getattr(self, s)()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for s in stages:
                getattr(self, s)()
        return graph

    def replay(self):
        """The band's work as one CUDA graph, the all-reduce (NCCL) on the current stream, then the projection backward as a second graph."""
        if self.local_graph is None:
            self.local_graph = self._capture(self.LOCAL)
            self.final_graph = self._capture(("_project_backward",))
        self.local_graph.replay()
        self.all_reduce()
        self.final_graph.replay()

    @property
    def kernels_per_step(self):
        return sum(self.KERNELS[s] for s in self.LOCAL + ("_project_backward",))

    def gaussian_pixel_evals(self):
        """Forward evaluations of the band: sum over its tiles of list length x in-image pixels of the tile."""
        if self.num_tiles == 0:
            return 0
        bins = self.bins[: self.num_tiles].to(torch.int64)
        lengths = (bins[:, 1] - bins[:, 0]).view(self.r1 - self.r0, self.tb[0])
        rows = torch.clamp(self.h - torch.arange(self.r0, self.r1, device=self.device) * TILE, max=TILE)
        cols = torch.clamp(self.w - torch.arange(self.tb[0], device=self.device) * TILE, max=TILE)
        return int((lengths * rows[:, None] * cols[None, :]).sum().item())

    def release(self):
        self.local_graph = self.final_graph = None
