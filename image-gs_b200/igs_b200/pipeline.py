"""
The rasterization training step with every buffer preallocated, issued as direct C-ABI launches and replayable as one CUDA graph: the
path of Image-GS's CUDA-graph step (model.py:1160-1209) for the hot path only:

    [quantize-STE] -> project -> prefix sum -> tile binning -> top-K forward -> L1 loss + gradient -> top-K backward -> projection backward
    [-> rate term forward/backward]

The top-K forward, the L1 loss with its gradient and the top-K backward run as one kernel per tile (igs_raster_step_l1), so the top-K
lists and the image gradient never go through HBM; fused=False runs them as the separate forward (with the loss) and backward kernels.

The intersection buffers hold `capacity` entries (capacity_ratio times the count of the first step, at least 1024, as model.py:110,1186),
so nothing is read back to the host inside the step; the true count is kept on the device (num_intersects) for overflow checks.
"""
import ctypes
from typing import Optional

import torch

from . import _lib, ops
from ._lib import ptr

TILE = ops.TILE
TOP_K = ops.TOP_K


class RasterStep:
    """One image's step. Inputs are device tensors: means [N,2], scales [N,2] (pixels), rotations [N,1], features [N,C], target [C,H,W]."""

    def __init__(self, means, scales, rotations, features, target, capacity: Optional[int] = None, capacity_ratio: float = 2.0,
                 l1_ratio: float = 1.0, quant: Optional[dict] = None, loss_transform=None, rate: Optional[dict] = None,
                 fused: bool = True):
        """quant: dict(pos_steps [2], scale_step, rot_step, feat_steps [C]) puts the straight-through quantizer in front (scales must be
        the canonical, non-negative ones); loss_transform [C,C]: render feat T^T (YUV loss space, needs quant); rate: dict(model (the
        fields of compress.rate.RateModel), inv_rot_step, factor) adds the rate term on the raw features and rotations. fused=False:
        separate forward and backward kernels, with the top-K lists and the image gradient (v_image) kept in HBM."""
        self.fused = fused
        self.lib = _lib.load()
        self.device = means.device
        self.n, self.c = features.shape
        c, self.h, self.w = target.shape
        assert c == self.c
        self.raw = (means, scales, rotations, features)
        self.means, self.scales, self.rotations, self.features, self.target = means, scales, rotations, features, target
        self.quant, self.rate = quant, rate
        self.transform = loss_transform.contiguous() if loss_transform is not None else None
        if self.quant is not None:
            self.q_means, self.q_scales, self.q_rot, self.q_feat = (torch.empty_like(means), torch.empty_like(scales),
                                                                    torch.empty_like(rotations), torch.empty_like(features))
            self.feat_t = torch.empty_like(features) if self.transform is not None else None
            self.means, self.scales, self.rotations = self.q_means, self.q_scales, self.q_rot
            self.features = self.feat_t if self.transform is not None else self.q_feat
            self._quantize()
        elif self.transform is not None:
            raise ValueError("loss_transform is applied by the quantizer stage; pass quant as well")
        self.tb = ops.tile_grid(self.h, self.w)
        self.num_tiles = self.tb[0] * self.tb[1]
        self.l1_ratio = float(l1_ratio)
        dev, f32, i32 = self.device, torch.float32, torch.int32
        n, nc = self.n, self.c
        self.xys = torch.empty(n, 2, device=dev, dtype=f32)
        self.radii = torch.empty(n, device=dev, dtype=i32)
        self.conics = torch.empty(n, 3, device=dev, dtype=f32)
        self.hits = torch.empty(n, device=dev, dtype=i32)
        self.cum = torch.empty(n, device=dev, dtype=i32)
        self.num_intersects = torch.empty(1, device=dev, dtype=i32)
        self.cum_ws_bytes = self.lib.igs_cumsum_workspace(n)
        self.cum_ws = torch.empty(self.cum_ws_bytes, device=dev, dtype=torch.uint8)
        self.image = torch.empty(nc, self.h, self.w, device=dev, dtype=f32)
        self.v_image = None if fused else torch.empty_like(self.image)
        self.loss = torch.empty((), device=dev, dtype=f32)
        self.l1_ws_bytes = self.lib.igs_raster_l1_workspace(self.num_tiles)
        self.l1_ws = torch.zeros(self.l1_ws_bytes, device=dev, dtype=torch.uint8)
        self.grads = torch.empty(n * (5 + nc), device=dev, dtype=f32)
        self.v_xy, self.v_conic, self.v_colors = self.grads[:2 * n].view(n, 2), self.grads[2 * n:5 * n].view(n, 3), self.grads[5 * n:].view(n, nc)
        self.v_cov2d = torch.empty(n, 3, device=dev, dtype=f32)
        self.v_mean2d = torch.empty(n, 2, device=dev, dtype=f32)
        self.v_scale = torch.empty(n, 2, device=dev, dtype=f32)
        self.v_rot = torch.empty(n, 1, device=dev, dtype=f32)
        if capacity is None:
            self._project()
            self._cumsum()
            count = int(self.num_intersects.item())
            capacity = max(1024, round(capacity_ratio * count))
        self.capacity = int(capacity)
        self.ids = torch.empty(self.capacity, device=dev, dtype=i32)
        self.bins = torch.empty(self.num_tiles, 2, device=dev, dtype=i32)
        self.sort_ws_bytes = self.lib.igs_sort_workspace(self.capacity, self.tb[0], self.tb[1])
        self.sort_ws = torch.empty(self.sort_ws_bytes, device=dev, dtype=torch.uint8)
        self.max_list = min(self.n, self.capacity)
        # top-K lists in the 16-bit tile-list form between the separate kernels (tiles with 65535+ entries are selected again by the
        # backward pass)
        self.topk = None if fused else torch.empty(self.num_tiles, TOP_K, TILE * TILE, device=dev, dtype=torch.int16)
        # the fused step's workspace (igs_train_step_l1: the stages below in one call, eight kernels, no memset)
        self.step_ws_bytes = self.lib.igs_train_step_workspace(n, self.capacity, self.tb[0], self.tb[1])
        self.step_ws = torch.empty(self.step_ws_bytes, device=dev, dtype=torch.uint8) if fused else None
        if self.rate is not None:
            m = self.rate["model"]
            self.rate_loss = torch.empty((), device=dev, dtype=f32)
            self.rate_weight = torch.empty(1, device=dev, dtype=f32)
            self.rate_own_grad = torch.empty_like(features)
            self.rate_rot_grad = torch.empty(n, device=dev, dtype=f32)
            self.rate_grad_feat = torch.empty_like(features)
            self.rate_grad_rot = torch.empty(n, device=dev, dtype=f32)
            self.rate_ws_bytes = self.lib.igs_rate_workspace(n)
            self.rate_ws = torch.zeros(self.rate_ws_bytes, device=dev, dtype=torch.uint8)
            self.rate_refs = ((ctypes.c_int32 * nc)(*m.color_refs), (ctypes.c_int32 * nc)(*m.pred_channels))
            self.grad_one = torch.ones((), device=dev, dtype=f32)
        if self.transform is not None or self.rate is not None:
            self.v_feat = torch.empty_like(features)  # gradient of the raw features
        self.graph = None

    # ---- stages (each one C-ABI call on the current stream) ----

    def _quantize(self):
        q = self.quant
        means, scales, rots, feats = self.raw
        self._check(self.lib.igs_quantize_ste(self.n, self.c, ptr(means), ptr(scales), ptr(rots), ptr(feats), ptr(q["pos_steps"]),
                                              float(q["scale_step"]), float(q["rot_step"]), ptr(q["feat_steps"]), ptr(self.transform),
                                              ptr(self.q_means), ptr(self.q_scales), ptr(self.q_rot), ptr(self.q_feat), ptr(self.feat_t),
                                              None, None, None, None, self._stream()), "quantize")

    def _rate_term(self):
        m, r = self.rate["model"], self.rate
        _, _, rots, feats = self.raw
        self._check(self.lib.igs_rate_fwd(self.n, self.c, m.neighbors.size(1), ptr(feats), ptr(rots), ptr(self.loss), ptr(m.neighbors),
                                          ptr(m.weights), ptr(m.slope), ctypes.cast(self.rate_refs[0], ctypes.c_void_p),
                                          ctypes.cast(self.rate_refs[1], ctypes.c_void_p), ptr(m.inv_steps), ptr(m.feat_coeffs),
                                          ptr(m.inv_rot), float(r["inv_rot_step"]), self.l1_ratio, float(r["factor"]), ptr(self.rate_loss),
                                          ptr(self.rate_weight), ptr(self.rate_own_grad), ptr(self.rate_rot_grad), ptr(self.rate_ws),
                                          self.rate_ws_bytes, self._stream()), "rate forward")
        self._check(self.lib.igs_rate_bwd(self.n, self.c, ptr(self.grad_one), ptr(self.rate_weight), ptr(self.rate_own_grad),
                                          ptr(self.rate_rot_grad), ptr(m.offsets), ptr(m.sources), ptr(m.source_weights), ptr(self.rate_grad_feat),
                                          ptr(self.rate_grad_rot), self._stream()), "rate backward")

    def _feature_grads(self):
        """Gradient of the raw features: through the loss-space transform (identity without one) plus the rate term's."""
        extra = self.rate_grad_feat if self.rate is not None else None
        if self.transform is not None:
            self._check(self.lib.igs_feat_transform_bwd(self.n, self.c, ptr(self.v_colors), ptr(self.transform), ptr(extra), ptr(self.v_feat),
                                                        self._stream()), "feature transform backward")
        else:
            torch.add(self.v_colors, extra, out=self.v_feat)

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _check(self, status, what):
        _lib.check(status, what)

    def _project(self):
        self._check(self.lib.igs_project_fwd(self.n, ptr(self.means), ptr(self.scales), ptr(self.rotations), self.h, self.w, self.tb[0],
                                             self.tb[1], ptr(self.xys), ptr(self.radii), ptr(self.conics), ptr(self.hits), self._stream()),
                    "project")

    def _cumsum(self):
        self._check(self.lib.igs_cumsum(self.n, ptr(self.hits), ptr(self.cum), ptr(self.num_intersects), ptr(self.cum_ws), self.cum_ws_bytes,
                                        self._stream()), "cumsum")

    def _bin(self):
        self._check(self.lib.igs_sort_intersects(self.n, self.capacity, ptr(self.xys), ptr(self.radii), ptr(self.cum), self.tb[0], self.tb[1],
                                                 ptr(self.ids), ptr(self.bins), ptr(self.sort_ws), self.sort_ws_bytes, self._stream()),
                    "bin")

    def _raster(self):
        """Render, the L1 loss and its gradient, and the top-K backward pass, in one kernel per tile."""
        self._check(self.lib.igs_raster_step_l1(self.tb[0], self.tb[1], self.h, self.w, self.c, self.n, ptr(self.ids), ptr(self.bins),
                                                ptr(self.xys), ptr(self.conics), ptr(self.features), ptr(self.target), self.l1_ratio,
                                                ptr(self.image), ptr(self.loss), ptr(self.v_image), ptr(self.v_xy), ptr(self.v_conic),
                                                ptr(self.v_colors), ptr(self.l1_ws), self.l1_ws_bytes, self._stream()), "raster step")

    def _forward(self):
        """Render, with the L1 loss and its gradient with respect to the image computed in the same kernel."""
        self._check(self.lib.igs_raster_fwd_topk_tiles_l1(self.tb[0], self.tb[1], self.h, self.w, self.c, self.max_list, ptr(self.ids),
                                                          ptr(self.bins), ptr(self.xys), ptr(self.conics), ptr(self.features),
                                                          ptr(self.target), self.l1_ratio, ptr(self.image), ptr(self.topk), ptr(self.loss),
                                                          ptr(self.v_image), ptr(self.l1_ws), self.l1_ws_bytes, self._stream()), "forward")

    def _backward(self):
        self._check(self.lib.igs_raster_bwd_topk_tiles(self.h, self.w, self.c, self.n, ptr(self.ids), ptr(self.bins), ptr(self.xys),
                                                       ptr(self.conics), ptr(self.features), ptr(self.v_image), ptr(self.topk), ptr(self.v_xy),
                                                       ptr(self.v_conic), ptr(self.v_colors), self._stream()), "backward")

    def _project_backward(self):
        self._check(self.lib.igs_project_bwd(self.n, ptr(self.scales), ptr(self.rotations), self.h, self.w, ptr(self.radii), ptr(self.conics),
                                             ptr(self.v_xy), ptr(self.v_conic), ptr(self.v_cov2d), ptr(self.v_mean2d), ptr(self.v_scale),
                                             ptr(self.v_rot), self._stream()), "project_backward")

    def _train_step(self):
        """Projection, prefix sum, binning, the fused raster step and the projection backward in one call (igs_train_step_l1)."""
        self._check(self.lib.igs_train_step_l1(self.n, self.c, ptr(self.means), ptr(self.scales), ptr(self.rotations), ptr(self.features),
                                               ptr(self.target), self.l1_ratio, self.h, self.w, 0, self.tb[1], self.capacity, ptr(self.xys),
                                               ptr(self.radii), ptr(self.conics), ptr(self.hits), ptr(self.cum), ptr(self.num_intersects),
                                               ptr(self.ids), ptr(self.bins), ptr(self.image), ptr(self.loss), ptr(self.v_xy),
                                               ptr(self.v_conic), ptr(self.v_colors), ptr(self.v_cov2d), ptr(self.v_mean2d),
                                               ptr(self.v_scale), ptr(self.v_rot), ptr(self.step_ws), self.step_ws_bytes, self._stream()),
                    "train step")

    # kernels each stage launches (memsets excluded)
    KERNELS = {"_quantize": 1, "_project": 1, "_cumsum": 2, "_bin": 4, "_raster": 2, "_forward": 2, "_backward": 1, "_project_backward": 1,
               "_rate_term": 2, "_feature_grads": 1, "_train_step": 8}

    @property
    def BREAKDOWN_STAGES(self):
        """The step's stages as separate calls (the fused step's kernels, one stage at a time, for per-stage timing)."""
        raster = ("_raster",) if self.fused else ("_forward", "_backward")
        return ("_project", "_cumsum", "_bin") + raster + ("_project_backward",)

    @property
    def BASE_STAGES(self):
        return ("_train_step",) if self.fused else self.BREAKDOWN_STAGES

    @property
    def STAGES(self):
        stages = (("_quantize",) if self.quant is not None else ()) + self.BASE_STAGES
        if self.rate is not None:
            stages += ("_rate_term",)
        if self.rate is not None or self.transform is not None:
            stages += ("_feature_grads",)
        return stages

    def launch(self):
        for s in self.STAGES:
            getattr(self, s)()

    @property
    def kernels_per_step(self):
        return sum(self.KERNELS[s] for s in self.STAGES)

    PACK_ALIGN = 64  # floats: each parameter array of the packed buffer starts on a 256-byte boundary

    @classmethod
    def packed_layout(cls, n, c):
        """Offsets (in floats) of means [N,2], scales [N,2], rotations [N,1], features [N,C] in the packed buffer, and its length."""
        offsets, at = [], 0
        for size in (2 * n, 2 * n, n, c * n):
            offsets.append(at)
            at += -(-size // cls.PACK_ALIGN) * cls.PACK_ALIGN
        return offsets, at

    def pack_inputs(self):
        """Move the four parameter arrays (means, scales, rotations, features; values kept) into one device buffer laid out as
        packed_layout(), so that a caller holding its parameters on the host copies a step's inputs in with one transfer of that buffer.
        Returns the buffer. Graphs captured afterwards read the packed arrays; graphs captured before keep the old ones."""
        offsets, length = self.packed_layout(self.n, self.c)
        flat = torch.empty(length, device=self.device, dtype=torch.float32)
        views = []
        for t, at in zip(self.raw, offsets):
            v = flat[at:at + t.numel()].view(t.shape)
            v.copy_(t)
            views.append(v)
        self.raw = tuple(views)
        if self.quant is None:
            self.means, self.scales, self.rotations, self.features = views
        self.graph = None
        return flat

    def capture(self, stages=None, before=None, after=None):
        """A CUDA graph of the step (or of the given stages); before() and after() issue extra work around them on the same stream (for
        example the copies of pinned host parameters in and of the loss out, which then run as nodes of the graph)."""
        stages = stages or self.STAGES

        def issue():
            if before is not None:
                before()
            for s in stages:
                getattr(self, s)()
            if after is not None:
                after()

        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            issue()  # warm-up outside the capture
        torch.cuda.current_stream(self.device).wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            issue()
        return graph

    def replay(self):
        if self.graph is None:
            self.graph = self.capture()
        self.graph.replay()

    def gaussian_pixel_evals(self):
        """Forward evaluations of the step: sum over tiles of list length x in-image pixels of the tile."""
        bins = self.bins.to(torch.int64)
        lengths = (bins[:, 1] - bins[:, 0]).view(self.tb[1], self.tb[0])
        rows = torch.clamp(self.h - torch.arange(self.tb[1], device=self.device) * TILE, max=TILE)
        cols = torch.clamp(self.w - torch.arange(self.tb[0], device=self.device) * TILE, max=TILE)
        return int((lengths * rows[:, None] * cols[None, :]).sum().item())
