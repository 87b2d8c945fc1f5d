"""
Differentiable operators of the training step, with the semantics of the reference's autograd Functions:
  - project_gaussians_2d_scale_rot (gsplat/gsplat/project_gaussians_2d_scale_rot.py:12-113)
  - rasterize_gaussians_sum with topk_norm=True (gsplat/gsplat/rasterize_sum.py:14-225), eager (one host read of the intersection count,
    as the reference) or with a fixed capacity (no host read; CUDA-graph capturable)
  - quantize_ste: the straight-through step quantization of model.py:993-1006
  - rate_loss (compress/rate.py:178-202)
  - l1_loss: ratio * F.l1_loss in one pass that keeps the signs for the backward pass; install_l1() routes model.py's F.l1_loss to it

The rasterization's autograd path keeps each pixel's top-K lists in the 16-bit tile-list form (positions in the tile's list; a quarter of
the bytes of the reference's [H, W, 10] int32 ids); the backward pass selects the lists of a tile again when its list reaches 65535
entries.
"""
import types
from typing import Optional

import torch
from torch.autograd import Function

from . import ops


class _ProjectGaussians2dScaleRot(Function):
    @staticmethod
    def forward(ctx, means2d, scales2d, rotation, img_height, img_width, tile_bounds):
        num_points = means2d.shape[-2]
        if num_points < 1 or means2d.shape[-1] != 2:
            raise ValueError(f"Invalid shape for means2d: {means2d.shape}")
        xys, radii, conics, num_tiles_hit = ops.project_gaussians_2d_scale_rot_forward(num_points, means2d, scales2d, rotation, img_height,
                                                                                       img_width, tile_bounds)
        ctx.img_height, ctx.img_width, ctx.num_points = img_height, img_width, num_points
        ctx.save_for_backward(means2d, scales2d, rotation, radii, conics)
        ctx.mark_non_differentiable(radii, num_tiles_hit)
        return xys, radii, conics, num_tiles_hit

    @staticmethod
    def backward(ctx, v_xys, v_radii, v_conics, v_num_tiles_hit):
        means2d, scales2d, rotation, radii, conics = ctx.saved_tensors
        if v_xys is None:
            v_xys = torch.zeros_like(means2d)
        if v_conics is None:
            v_conics = torch.zeros_like(conics)
        _, v_mean2d, v_scale, v_rot = ops.project_gaussians_2d_scale_rot_backward(ctx.num_points, means2d, scales2d, rotation,
                                                                                  ctx.img_height, ctx.img_width, radii, conics, v_xys,
                                                                                  v_conics)
        return v_mean2d, v_scale, v_rot.view_as(rotation), None, None, None


def project_gaussians_2d_scale_rot(means2d, scales2d, rotation, img_height, img_width, tile_bounds):
    return _ProjectGaussians2dScaleRot.apply(means2d.contiguous(), scales2d.contiguous(), rotation.contiguous(), img_height, img_width,
                                             tile_bounds)


def bin_gaussians(num_points, xys, radii, num_tiles_hit, tile_bounds, capacity: Optional[int]):
    """(gaussian_ids_sorted, tile_bins, num_intersects): with a capacity, no host synchronization; without, the exact count is read back
    (compute_cumulative_intersects of the reference) and used as the capacity."""
    cum, total = ops.cumulative_intersects(num_tiles_hit)
    if capacity is None:
        capacity = int(total.item())
        if capacity < 1:
            return None, None, 0
    ids, bins = ops.sort_intersects_by_tile(num_points, capacity, xys, radii, cum, tile_bounds)
    return ids, bins, capacity


class _RasterizeGaussiansSumTopK(Function):
    @staticmethod
    def forward(ctx, xys, radii, conics, num_tiles_hit, colors, img_height, img_width, capacity):
        num_points = xys.size(0)
        tile_bounds = ops.tile_grid(img_height, img_width)
        ids, bins, num_intersects = bin_gaussians(num_points, xys, radii, num_tiles_hit, tile_bounds, capacity)
        ctx.img_height, ctx.img_width, ctx.num_intersects = img_height, img_width, num_intersects
        if num_intersects < 1:
            ctx.save_for_backward(xys, conics, colors)
            ctx.form = "empty"
            return torch.zeros(img_height, img_width, colors.shape[-1], device=xys.device, dtype=torch.float32)
        bound = min(num_points, num_intersects)
        img_size = (img_width, img_height, 1)
        out_img, tile_topk = ops.nd_rasterize_forward_topk_norm_tiles(tile_bounds, img_size, bound, ids, bins, xys, conics, colors)
        ctx.form = "tiles"
        ctx.save_for_backward(xys, conics, colors, ids, bins, tile_topk)
        # channel-planar [C, H, W] returned as an [H, W, C] view (rasterize_sum.py:248-265)
        return out_img.permute(1, 2, 0)

    @staticmethod
    def backward(ctx, v_out_img):
        if ctx.form == "empty":
            xys, conics, colors = ctx.saved_tensors
            return torch.zeros_like(xys), None, torch.zeros_like(conics), None, torch.zeros_like(colors), None, None, None
        v_output = v_out_img.permute(2, 0, 1).contiguous()  # channel-planar; free when the caller's gradient is [C, H, W]
        xys, conics, colors, ids, bins, tile_topk = ctx.saved_tensors
        v_xy, v_conic, v_colors = ops.nd_rasterize_backward_topk_norm_tiles(ctx.img_height, ctx.img_width, ids, bins, xys, conics, colors,
                                                                            v_output, tile_topk)
        return v_xy, None, v_conic, None, v_colors, None, None, None


def rasterize_gaussians_sum_topk(xys, radii, conics, num_tiles_hit, colors, img_height, img_width, capacity=None):
    if colors.dtype == torch.uint8:
        colors = colors.float() / 255
    if xys.ndimension() != 2 or xys.size(1) != 2:
        raise ValueError("xys must have dimensions (N, 2)")
    if colors.ndimension() != 2:
        raise ValueError("colors must have dimensions (N, D)")
    if colors.size(1) > ops.MAX_CHANNELS:
        raise ValueError(f"at most {ops.MAX_CHANNELS} channels")
    return _RasterizeGaussiansSumTopK.apply(xys.contiguous(), radii.contiguous(), conics.contiguous(), num_tiles_hit.contiguous(),
                                            colors.contiguous(), int(img_height), int(img_width), capacity)


class _QuantizeSTE(Function):
    @staticmethod
    def forward(ctx, xy, scale, rot, feat, pos_steps, scale_step, rot_step, feat_steps):
        (out_xy, out_scale, out_rot, out_feat), _, _ = ops.quantize_ste_forward(xy, scale, rot, feat, pos_steps, scale_step, rot_step,
                                                                                feat_steps)
        return out_xy, out_scale, out_rot, out_feat

    @staticmethod
    def backward(ctx, g_xy, g_scale, g_rot, g_feat):
        # straight-through: x + (q(x) - x).detach() passes the gradient unchanged
        return g_xy, g_scale, g_rot, g_feat, None, None, None, None


def quantize_ste(xy, scale, rot, feat, pos_steps, scale_step, rot_step, feat_steps):
    """Straight-through step-quantized (xy, scale, rot, feat) of canonicalized parameters (scale in pixels, non-negative): the values of
    model._get_params in "step" mode during optimization (model.py:993-1006)."""
    return _QuantizeSTE.apply(xy.contiguous(), scale.contiguous(), rot.contiguous(), feat.contiguous(), pos_steps.contiguous(),
                              float(scale_step), float(rot_step), feat_steps.contiguous())


class _RateLoss(Function):
    @staticmethod
    def forward(ctx, feat, rot, l1_loss, model, inv_rot_step, l1_ratio, factor):
        loss, loss_weight, own_grad, rot_grad = ops.rate_loss_forward(
            feat.contiguous(), rot.contiguous(), l1_loss.contiguous(), model.neighbors, model.weights, model.slope, list(model.color_refs),
            list(model.pred_channels), model.inv_steps, model.feat_coeffs, model.inv_rot, inv_rot_step, l1_ratio, factor)
        ctx.save_for_backward(loss_weight, own_grad, rot_grad)
        ctx.model, ctx.rot_shape = model, rot.shape
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        loss_weight, own_grad, rot_grad = ctx.saved_tensors
        m = ctx.model
        grad_feat, grad_rot = ops.rate_loss_backward(grad_loss.contiguous(), loss_weight, own_grad, rot_grad, m.offsets, m.sources,
                                                     m.source_weights)
        return grad_feat, grad_rot.view(ctx.rot_shape), None, None, None, None, None


def rate_loss(feat, rot, l1_loss, model, inv_rot_step, l1_ratio, factor):
    """factor / max(l1_loss / l1_ratio, 1e-4) times the smooth Laplace bits of the features and rotations (compress/rate.py:197-202);
    `model` carries the fields of compress.rate.RateModel."""
    return _RateLoss.apply(feat, rot, l1_loss.detach(), model, inv_rot_step, l1_ratio, factor)


class _L1Loss(Function):
    @staticmethod
    def forward(ctx, image, target, ratio):
        loss, signs = ops.l1_loss_signs(image.contiguous(), target.contiguous(), ratio)
        ctx.save_for_backward(signs)
        ctx.ratio = ratio
        return loss

    @staticmethod
    def backward(ctx, grad_loss):
        (signs,) = ctx.saved_tensors
        scale = grad_loss if ctx.ratio == 1.0 else grad_loss * ctx.ratio
        return ops.l1_grad_from_signs(signs, scale), None, None


def l1_loss(image, target, ratio=1.0):
    """ratio * mean|image - target| (model.py:1224-1227) in one pass that keeps the signs; the backward pass forms
    sign * (g / numel) from them, ATen's l1_loss gradient bit for bit for ratio 1 (F.l1_loss)."""
    return _L1Loss.apply(image, target, float(ratio))


def _routed_l1_loss(input, target, size_average=None, reduce=None, reduction="mean"):
    """F.l1_loss with the library's loss for what it computes (the mean over two float32 CUDA tensors of one shape, no gradient for the
    target); anything else goes to torch's F.l1_loss."""
    import torch.nn.functional as F

    if (size_average is None and reduce is None and reduction == "mean" and isinstance(input, torch.Tensor)
            and isinstance(target, torch.Tensor) and input.is_cuda and target.device == input.device
            and input.dtype == torch.float32 and target.dtype == torch.float32 and input.shape == target.shape and input.numel() > 0
            and not target.requires_grad):
        return l1_loss(input, target)
    return F.l1_loss(input, target, size_average, reduce, reduction)


class _FunctionalWithL1(types.ModuleType):
    """torch.nn.functional as seen by a module after install_l1(): l1_loss routed (_routed_l1_loss), every other name torch's."""

    def __init__(self):
        super().__init__("torch.nn.functional")
        self.l1_loss = _routed_l1_loss

    def __getattr__(self, name):
        import torch.nn.functional as F

        return getattr(F, name)


def install_l1(*module_names):
    """Route F.l1_loss in the named modules (default: model, whose training loss calls it, model.py:1226) to the library's loss: the
    name F bound there to torch.nn.functional is replaced by a view of it with l1_loss routed. Returns {(module, "F"): original} for
    restore()."""
    import importlib

    import torch.nn.functional as F

    replaced = {}
    for name in module_names or ("model",):
        try:
            module = importlib.import_module(name)
        except ImportError:
            continue
        if getattr(module, "F", None) is F:
            replaced[(name, "F")] = F
            module.F = _FunctionalWithL1()
    return replaced


def restore(replaced):
    """Undo install_l1()."""
    import importlib

    for (name, attr), original in replaced.items():
        setattr(importlib.import_module(name), attr, original)
