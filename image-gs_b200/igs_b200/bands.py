"""
One image split into tile-row bands across GPUs (one process per GPU): the Gaussian parameters are replicated; every rank projects all
Gaussians, bins and renders only its rows, takes the L1 loss and its gradient on its rows (normalised by the whole image's pixel count),
and runs the backward pass for its band. The partial gradients with respect to the projected Gaussians (v_xy, v_conic, v_colors:
N (5 + C) floats, 2.6 MB at 80,000 Gaussians) and the partial loss are then combined in one of two ways:
  * exchange="peer" (PeerExchange, igs_band_reduce): over peer memory, each rank sums one share of the Gaussians' partials from every
    rank, runs the projection backward on that share and stores the parameter gradients into every rank's results; one kernel, no
    collective library, and the whole step is one CUDA graph;
  * exchange="nccl": one NCCL all-reduce of the partials, after which every rank runs the projection backward on all Gaussians.
Either way all ranks hold the same parameter gradients.

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
# include/igs_b200.h
MAX_BAND_RANKS = 8
IPC_HANDLE_BYTES = 64
SYNC_STEP, SYNC_ERROR = 16, 17


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


def _round_up(x, m):
    return (x + m - 1) // m * m


class PeerExchange:
    """The ranks' exchange buffers, shared over CUDA IPC. Each rank's buffer (one float32 tensor) holds its partials
    [N (5 + C) + 1] (v_xy, v_conic, v_colors, loss: what its band kernels write), its results (igs_band_results_floats: v_cov2d,
    v_mean2d, v_scale, v_rot, summed v_colors, loss) and its synchronisation words; every rank maps every other rank's buffer. Collective:
    every rank of `group` constructs it, and every rank calls release()."""

    def __init__(self, num_points, channels, device, group, timeout_ms=20000):
        import torch.distributed as dist

        self.lib = lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > MAX_BAND_RANKS:
            raise ValueError(f"the peer exchange takes at most {MAX_BAND_RANKS} ranks (got {self.world})")
        self.n, self.c, self.timeout_ms = int(num_points), int(channels), int(timeout_ms)
        n_part = self.n * (5 + self.c) + 1
        n_res = int(lib.igs_band_results_floats(self.n, self.c))
        sync_words = int(lib.igs_band_sync_bytes()) // 4
        self.res_off = _round_up(n_part, 64)  # 256-byte aligned regions
        self.sync_off = self.res_off + _round_up(n_res, 64)
        self.buf = torch.zeros(self.sync_off + sync_words, device=device, dtype=torch.float32)
        self.partials = self.buf[:n_part]
        self.results = self.buf[self.res_off:self.res_off + n_res]
        self.sync = self.buf[self.sync_off:self.sync_off + sync_words].view(torch.int32)
        # a failure on one rank is agreed on by all before anyone raises, so that every rank takes the same collective steps
        failure = None
        handle = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        offset = ctypes.c_uint64()
        try:
            _lib.check(lib.igs_ipc_export(ptr(self.buf), handle, ctypes.byref(offset)), "igs_ipc_export")
        except _lib.IgsError as err:
            failure = err
        mine = torch.tensor(list(bytes(handle)) + list(int(offset.value).to_bytes(8, "little")), dtype=torch.uint8, device=device)
        gathered = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(gathered, mine, group=group)
        self.opened = []  # (address, offset) of the peers' mapped buffers
        bases = []
        flag = torch.tensor([int(failure is not None)], dtype=torch.int32, device=device)
        dist.all_reduce(flag, group=group)
        try:
            for q, g in enumerate(gathered if int(flag.item()) == 0 else []):
                if q == self.rank:
                    bases.append(self.buf.data_ptr())
                    continue
                raw = bytes(g.cpu().tolist())
                peer = ctypes.c_void_p()
                off = int.from_bytes(raw[IPC_HANDLE_BYTES:], "little")
                _lib.check(lib.igs_ipc_open((ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(raw[:IPC_HANDLE_BYTES]), off,
                                            ctypes.byref(peer)), "igs_ipc_open")
                self.opened.append((peer.value, off))
                bases.append(peer.value)
        except _lib.IgsError as err:
            failure = failure or err
        flag = torch.tensor([int(failure is not None)], dtype=torch.int32, device=device)
        dist.all_reduce(flag, group=group)
        if int(flag.item()) != 0:
            for address, off in self.opened:
                lib.igs_ipc_close(ctypes.c_void_p(address), off)
            self.opened = []
            raise failure or RuntimeError("the peer exchange could not be set up on another rank")
        arr = ctypes.c_void_p * self.world
        self.partials_ptrs = arr(*bases)
        self.results_ptrs = arr(*[b + 4 * self.res_off for b in bases])
        self.sync_ptrs = arr(*[b + 4 * self.sync_off for b in bases])
        # every rank's synchronisation words are zero before any rank's first exchange
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def views(self):
        """(v_cov2d, v_mean2d, v_scale, v_rot, v_colors, loss) of this rank's results."""
        n, c, r = self.n, self.c, self.results
        return (r[:3 * n].view(n, 3), r[3 * n:5 * n].view(n, 2), r[5 * n:7 * n].view(n, 2), r[7 * n:8 * n].view(n, 1),
                r[8 * n:(8 + c) * n].view(n, c), r[(8 + c) * n])

    def reduce(self, scales, rotations, img_h, img_w, radii, conics, stream):
        _lib.check(self.lib.igs_band_reduce(self.world, self.rank, self.n, self.c, self.partials_ptrs, self.results_ptrs, self.sync_ptrs,
                                            ptr(scales), ptr(rotations), img_h, img_w, ptr(radii), ptr(conics), self.timeout_ms, stream),
                   "igs_band_reduce")

    def error(self):
        """The error word (0: every wait so far succeeded); reading it synchronizes with the device."""
        return int(self.sync[SYNC_ERROR].item())

    def steps(self):
        return int(self.sync[SYNC_STEP].item())

    def release(self):
        """Collective: after every rank's last exchange has completed, unmap the peers' buffers."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.buf.device)
        dist.barrier(group=self.group)
        for address, off in self.opened:
            _lib.check(self.lib.igs_ipc_close(ctypes.c_void_p(address), off), "igs_ipc_close")
        self.opened = []
        dist.barrier(group=self.group)


class BandStep:
    """One rank's share of a step. Device tensors: means [N,2], scales [N,2], rotations [N,1], features [N,C] (replicated), the whole
    target [C,H,W] or just its band rows; rows [row_begin, row_end) are tile rows. group: a torch.distributed process group (None: a
    single band, no communication). exchange: "peer" (igs_band_reduce over CUDA IPC mappings of the ranks' buffers) or "nccl" (an
    all-reduce, then the projection backward on every rank). After a step, v_colors, v_mean2d, v_scale, v_rot, v_cov2d and loss hold the
    whole image's gradients and loss on every rank."""

    def __init__(self, means, scales, rotations, features, target, img_h, img_w, row_begin, row_end, group=None, capacity=None,
                 capacity_ratio: float = 2.0, l1_ratio: float = 1.0, fused: bool = True, exchange: str = "nccl",
                 timeout_ms: int = 20000):
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer' (got {exchange!r})")
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
        # the band's partials in one buffer: v_xy, v_conic, v_colors, then the loss (summed in place by the NCCL all-reduce)
        self.peer = PeerExchange(n, nc, dev, group, timeout_ms) if exchange == "peer" and group is not None else None
        self.exchange = "peer" if self.peer is not None else "nccl"
        self.reduced = self.peer.partials if self.peer is not None else torch.empty(n * (5 + nc) + 1, device=dev, dtype=f32)
        self.p_xy = self.reduced[:2 * n].view(n, 2)
        self.p_conic = self.reduced[2 * n:5 * n].view(n, 3)
        self.p_colors = self.reduced[5 * n:n * (5 + nc)].view(n, nc)
        self.p_loss = self.reduced[n * (5 + nc)]
        if self.peer is not None:
            self.v_cov2d, self.v_mean2d, self.v_scale, self.v_rot, self.v_colors, self.loss = self.peer.views()
        else:
            self.v_xy, self.v_conic, self.v_colors, self.loss = self.p_xy, self.p_conic, self.p_colors, self.p_loss
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
        # the fused band step's workspace (igs_train_step_l1 over the band's rows, without the projection backward)
        self.step_ws_bytes = self.lib.igs_train_step_workspace(n, self.capacity, self.tb[0], self.r1 - self.r0)
        self.step_ws = torch.empty(self.step_ws_bytes, device=dev, dtype=torch.uint8) if fused else None
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
                                                    self.l1_ratio, ptr(self.image), ptr(self.p_loss), None, ptr(self.p_xy),
                                                    ptr(self.p_conic), ptr(self.p_colors), ptr(self.l1_ws), self.l1_ws_bytes, self._stream()),
                   "raster step")

    def _forward(self):
        if self.num_tiles == 0:
            self.p_loss.zero_()
            return
        _lib.check(self.lib.igs_raster_fwd_topk_tiles_l1_band(self.tb[0], self.tb[1], self.h, self.w, self.r0, self.r1, self.c, self.max_list,
                                                              ptr(self.ids), ptr(self.bins), ptr(self.xys), ptr(self.conics),
                                                              ptr(self.features), ptr(self.target), self.l1_ratio, ptr(self.image),
                                                              ptr(self.topk), ptr(self.p_loss), ptr(self.v_image), ptr(self.l1_ws),
                                                              self.l1_ws_bytes, self._stream()), "forward")

    def _backward(self):
        _lib.check(self.lib.igs_raster_bwd_topk_tiles_band(self.h, self.w, self.r0, self.r1, self.c, self.n, ptr(self.ids), ptr(self.bins),
                                                           ptr(self.xys), ptr(self.conics), ptr(self.features), ptr(self.v_image),
                                                           ptr(self.topk), ptr(self.p_xy), ptr(self.p_conic), ptr(self.p_colors),
                                                           self._stream()), "backward")

    def _project_backward(self):
        _lib.check(self.lib.igs_project_bwd(self.n, ptr(self.scales), ptr(self.rotations), self.h, self.w, ptr(self.radii), ptr(self.conics),
                                            ptr(self.p_xy), ptr(self.p_conic), ptr(self.v_cov2d), ptr(self.v_mean2d), ptr(self.v_scale),
                                            ptr(self.v_rot), self._stream()), "project_backward")

    def _train_step(self):
        """Projection (tiles hit counted over the band's rows), prefix sum, the band's binning and its fused raster step in one call
        (igs_train_step_l1 without the projection backward): the band's partials and partial loss."""
        _lib.check(self.lib.igs_train_step_l1(self.n, self.c, ptr(self.means), ptr(self.scales), ptr(self.rotations), ptr(self.features),
                                              ptr(self.target), self.l1_ratio, self.h, self.w, self.r0, self.r1, self.capacity,
                                              ptr(self.xys), ptr(self.radii), ptr(self.conics), ptr(self.band_hits), ptr(self.cum),
                                              ptr(self.num_intersects), ptr(self.ids), ptr(self.bins), ptr(self.image), ptr(self.p_loss),
                                              ptr(self.p_xy), ptr(self.p_conic), ptr(self.p_colors), None, None, None, None,
                                              ptr(self.step_ws), self.step_ws_bytes, self._stream()), "band train step")

    def _exchange(self):
        self.peer.reduce(self.scales, self.rotations, self.h, self.w, self.radii, self.conics, self._stream())

    KERNELS = {"_project": 2, "_cumsum": 2, "_bin": 4, "_raster": 2, "_forward": 2, "_backward": 1, "_project_backward": 1,
               "_exchange": 1, "_train_step": 8}

    @property
    def LOCAL(self):
        """The band's own work: one igs_train_step_l1 call (fused), or the separate forward and backward kernels after the stages."""
        return ("_train_step",) if self.fused else ("_project", "_cumsum", "_bin", "_forward", "_backward")

    @property
    def FINAL(self):
        """The stages after the band's own work: the peer exchange, or (after the NCCL all-reduce) the projection backward."""
        return ("_exchange",) if self.peer is not None else ("_project_backward",)

    def all_reduce(self):
        if self.group is not None and self.peer is None:
            torch.distributed.all_reduce(self.reduced, group=self.group)

    def launch(self):
        for s in self.LOCAL:
            getattr(self, s)()
        self.all_reduce()
        for s in self.FINAL:
            getattr(self, s)()

    def check(self):
        """Raise on every rank if a wait of the peer exchange gave up on any rank (a rank missing or late by more than the timeout);
        collective (the ranks agree before anyone raises, so they keep taking the same collective steps), synchronizes."""
        if self.peer is not None:
            import torch.distributed as dist

            code = torch.tensor([self.peer.error()], dtype=torch.int32, device=self.device)
            dist.all_reduce(code, op=dist.ReduceOp.MAX, group=self.peer.group)
            if int(code.item()):
                raise _lib.IgsError(f"band exchange: a wait for the other ranks timed out on some rank (code {int(code.item())}; "
                                    f"rank {self.peer.rank}: {self.peer.error()})")

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
        """With the peer exchange, the whole step as one CUDA graph. With NCCL, the band's work as one CUDA graph, the all-reduce on the
        current stream, then the projection backward as a second graph."""
        if self.local_graph is None:
            if self.peer is not None:
                self.local_graph = self._capture(self.LOCAL + self.FINAL)
            else:
                self.local_graph = self._capture(self.LOCAL)
                self.final_graph = self._capture(self.FINAL)
        self.local_graph.replay()
        self.all_reduce()
        if self.final_graph is not None:
            self.final_graph.replay()

    @property
    def kernels_per_step(self):
        return sum(self.KERNELS[s] for s in self.LOCAL + self.FINAL)

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
        """Drop the graphs; with the peer exchange, collective: every rank unmaps the others' buffers."""
        self.local_graph = self.final_graph = None
        if self.peer is not None:
            self.peer.release()
            self.peer = None
