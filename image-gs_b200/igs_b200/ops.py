"""
Tensor-level operators over the igs_b200 C ABI, with the names, argument order, return values and input checks of the reference's
pybind functions (gsplat/gsplat/cuda/csrc/ext.cpp:4-32, bindings.h). Outputs are allocated with PyTorch's caching allocator on the input's
device and every launch goes to the current CUDA stream, so the operators can be captured in CUDA graphs (the *_capacity paths never read
device memory back to the host).
"""
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import check, ptr, stream_of

TILE = 16
TOP_K = 10
MAX_CHANNELS = 12
EPS = 1e-4


def _check_input(t: torch.Tensor, name: str, dtype=None):
    # CHECK_INPUT of the reference (bindings.h:9-14): CUDA and contiguous
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")


def _lib_call(name, *args):
    check(getattr(_lib.load(), name)(*args), name)


def tile_grid(img_height: int, img_width: int) -> Tuple[int, int, int]:
    return ((img_width + TILE - 1) // TILE, (img_height + TILE - 1) // TILE, 1)


# ---- projection ----------------------------------------------------------------------------------------------------------------------

def project_gaussians_2d_scale_rot_forward(num_points, means2d, scales2d, rotation, img_height, img_width, tile_bounds):
    """-> xys [N,2], radii [N] int32, conics [N,3], num_tiles_hit [N] int32 (bindings.cu:791-837)."""
    for t, n in ((means2d, "means2d"), (scales2d, "scales2d"), (rotation, "rotation")):
        _check_input(t, n, torch.float32)
    dev = means2d.device
    xys = torch.empty(num_points, 2, device=dev, dtype=torch.float32)
    radii = torch.empty(num_points, device=dev, dtype=torch.int32)
    conics = torch.empty(num_points, 3, device=dev, dtype=torch.float32)
    num_tiles_hit = torch.empty(num_points, device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        _lib_call("igs_project_fwd", int(num_points), ptr(means2d), ptr(scales2d), ptr(rotation), int(img_height), int(img_width),
                  int(tile_bounds[0]), int(tile_bounds[1]), ptr(xys), ptr(radii), ptr(conics), ptr(num_tiles_hit), stream_of(dev))
    return xys, radii, conics, num_tiles_hit


def project_gaussians_2d_scale_rot_backward(num_points, means2d, scales2d, rotation, img_height, img_width, radii, conics, v_xy,
                                            v_conic):
    """-> v_cov2d [N,3], v_mean2d [N,2], v_scale [N,2], v_rot [N,1] (bindings.cu:845-891)."""
    scales2d, rotation, radii, conics = scales2d.contiguous(), rotation.contiguous(), radii.contiguous(), conics.contiguous()
    v_xy, v_conic = v_xy.contiguous(), v_conic.contiguous()
    for t, n in ((scales2d, "scales2d"), (rotation, "rotation"), (conics, "conics"), (v_xy, "v_xy"), (v_conic, "v_conic")):
        _check_input(t, n, torch.float32)
    _check_input(radii, "radii", torch.int32)
    dev = scales2d.device
    v_cov2d = torch.empty(num_points, 3, device=dev, dtype=torch.float32)
    v_mean2d = torch.empty(num_points, 2, device=dev, dtype=torch.float32)
    v_scale = torch.empty(num_points, 2, device=dev, dtype=torch.float32)
    v_rot = torch.empty(num_points, 1, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib_call("igs_project_bwd", int(num_points), ptr(scales2d), ptr(rotation), int(img_height), int(img_width), ptr(radii),
                  ptr(conics), ptr(v_xy), ptr(v_conic), ptr(v_cov2d), ptr(v_mean2d), ptr(v_scale), ptr(v_rot), stream_of(dev))
    return v_cov2d, v_mean2d, v_scale, v_rot


# ---- binning -------------------------------------------------------------------------------------------------------------------------

def cumulative_intersects(num_tiles_hit: torch.Tensor):
    """Inclusive int32 prefix sum and its last element as a 1-element device tensor (no host synchronization)."""
    _check_input(num_tiles_hit, "num_tiles_hit", torch.int32)
    n = num_tiles_hit.numel()
    dev = num_tiles_hit.device
    cum = torch.empty(n, device=dev, dtype=torch.int32)
    total = torch.empty(1, device=dev, dtype=torch.int32)
    ws_bytes = _lib.load().igs_cumsum_workspace(n)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib_call("igs_cumsum", int(n), ptr(num_tiles_hit), ptr(cum), ptr(total), ptr(ws), ws_bytes, stream_of(dev))
    return cum, total


def sort_intersects_by_tile(num_points, capacity, xys, radii, cum_tiles_hit, tile_bounds):
    """-> gaussian_ids_sorted [capacity] int32, tile_bins [T,2] int32 (bindings.cu:106-167)."""
    _check_input(xys, "xys", torch.float32)
    _check_input(radii, "radii", torch.int32)
    _check_input(cum_tiles_hit, "cum_tiles_hit", torch.int32)
    dev = xys.device
    tiles_x, tiles_y = int(tile_bounds[0]), int(tile_bounds[1])
    num_tiles = tiles_x * tiles_y
    capacity = int(capacity)
    if capacity <= 0:
        return (torch.zeros(0, device=dev, dtype=torch.int32), torch.zeros(num_tiles, 2, device=dev, dtype=torch.int32))
    ids = torch.empty(capacity, device=dev, dtype=torch.int32)
    tile_bins = torch.empty(num_tiles, 2, device=dev, dtype=torch.int32)
    ws_bytes = _lib.load().igs_sort_workspace(capacity, tiles_x, tiles_y)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib_call("igs_sort_intersects", int(num_points), capacity, ptr(xys), ptr(radii), ptr(cum_tiles_hit), tiles_x, tiles_y, ptr(ids),
                  ptr(tile_bins), ptr(ws), ws_bytes, stream_of(dev))
    return ids, tile_bins


# ---- rasterization -------------------------------------------------------------------------------------------------------------------

def _check_raster_geometry(tile_bounds, block, img_size):
    if tuple(block)[:2] != (TILE, TILE):
        raise ValueError(f"block must be ({TILE}, {TILE}, 1) (the tile size is fixed at compile time), got {tuple(block)}")
    w, h = int(img_size[0]), int(img_size[1])
    if (int(tile_bounds[0]), int(tile_bounds[1])) != tile_grid(h, w)[:2]:
        raise ValueError(f"tile_bounds {tuple(tile_bounds)} do not cover a {w}x{h} image with {TILE}x{TILE} tiles")
    return h, w


def nd_rasterize_forward_topk_norm(tile_bounds, block, img_size, gaussian_ids_sorted, tile_bins, xys, conics, colors):
    """-> out_img [C,H,W], pixel_topk [H,W,10] int32 (bindings.cu:380-437)."""
    h, w = _check_raster_geometry(tile_bounds, block, img_size)
    _check_input(gaussian_ids_sorted, "gaussian_ids_sorted", torch.int32)
    _check_input(tile_bins, "tile_bins", torch.int32)
    for t, n in ((xys, "xys"), (conics, "conics"), (colors, "colors")):
        _check_input(t, n, torch.float32)
    channels = colors.size(1)
    if channels > MAX_CHANNELS:
        raise RuntimeError("at most MAX_CHANNELS channels")
    dev = xys.device
    out_img = torch.empty(channels, h, w, device=dev, dtype=torch.float32)
    pixel_topk = torch.empty(h, w, TOP_K, device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        _lib_call("igs_raster_fwd_topk", int(tile_bounds[0]), int(tile_bounds[1]), h, w, channels, ptr(gaussian_ids_sorted),
                  ptr(tile_bins), ptr(xys), ptr(conics), ptr(colors), ptr(out_img), ptr(pixel_topk), stream_of(dev))
    return out_img, pixel_topk


def nd_rasterize_forward_topk_norm_tiles(tile_bounds, img_size, max_list_len, gaussian_ids_sorted, tile_bins, xys, conics, colors):
    """The training-step forward: out_img [C,H,W] and the top-K lists as 16-bit tile-list positions [T,10,256] uint16."""
    h, w = _check_raster_geometry(tile_bounds, (TILE, TILE, 1), img_size)
    channels = colors.size(1)
    dev = xys.device
    num_tiles = int(tile_bounds[0]) * int(tile_bounds[1])
    out_img = torch.empty(channels, h, w, device=dev, dtype=torch.float32)
    tile_topk = torch.empty(num_tiles, TOP_K, TILE * TILE, device=dev, dtype=torch.int16)  # uint16 bit patterns
    with torch.cuda.device(dev):
        _lib_call("igs_raster_fwd_topk_tiles", int(tile_bounds[0]), int(tile_bounds[1]), h, w, channels, int(max_list_len),
                  ptr(gaussian_ids_sorted), ptr(tile_bins), ptr(xys), ptr(conics), ptr(colors), ptr(out_img), ptr(tile_topk),
                  stream_of(dev))
    return out_img, tile_topk


def nd_rasterize_forward_topk_norm_tiles_l1(tile_bounds, img_size, max_list_len, gaussian_ids_sorted, tile_bins, xys, conics, colors,
                                            target, ratio=1.0):
    """The training-step forward with the L1 loss fused: (out_img [C,H,W], tile_topk, loss = ratio * mean|out_img - target|,
    v_output = its gradient with respect to out_img); target [C,H,W] float32."""
    h, w = _check_raster_geometry(tile_bounds, (TILE, TILE, 1), img_size)
    channels = colors.size(1)
    _check_input(target, "target", torch.float32)
    if tuple(target.shape) != (channels, h, w):
        raise RuntimeError(f"target must be [{channels}, {h}, {w}]")
    dev = xys.device
    num_tiles = int(tile_bounds[0]) * int(tile_bounds[1])
    lib = _lib.load()
    out_img = torch.empty(channels, h, w, device=dev, dtype=torch.float32)
    v_output = torch.empty_like(out_img)
    loss = torch.empty((), device=dev, dtype=torch.float32)
    tile_topk = torch.empty(num_tiles, TOP_K, TILE * TILE, device=dev, dtype=torch.int16)
    ws_bytes = lib.igs_raster_l1_workspace(num_tiles)
    ws = torch.zeros(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib_call("igs_raster_fwd_topk_tiles_l1", int(tile_bounds[0]), int(tile_bounds[1]), h, w, channels, int(max_list_len),
                  ptr(gaussian_ids_sorted), ptr(tile_bins), ptr(xys), ptr(conics), ptr(colors), ptr(target), float(ratio), ptr(out_img),
                  ptr(tile_topk), ptr(loss), ptr(v_output), ptr(ws), ws_bytes, stream_of(dev))
    return out_img, tile_topk, loss, v_output


def raster_step_l1(tile_bounds, img_size, gaussian_ids_sorted, tile_bins, xys, conics, colors, target, ratio=1.0, with_v_output=False):
    """The training step's rasterization with the L1 loss in one kernel (igs_raster_step_l1): out_img [C,H,W], loss = ratio *
    mean|out_img - target|, and the gradients of the loss v_xy [N,2], v_conic [N,3], v_colors [N,C] (plus v_output, the loss's gradient
    with respect to out_img, when with_v_output), as nd_rasterize_forward_topk_norm_tiles_l1 followed by
    nd_rasterize_backward_topk_norm_tiles would give them."""
    h, w = _check_raster_geometry(tile_bounds, (TILE, TILE, 1), img_size)
    _check_input(gaussian_ids_sorted, "gaussian_ids_sorted", torch.int32)
    _check_input(tile_bins, "tile_bins", torch.int32)
    for t, name in ((xys, "xys"), (conics, "conics"), (colors, "colors"), (target, "target")):
        _check_input(t, name, torch.float32)
    channels = colors.size(1)
    if channels > MAX_CHANNELS:
        raise RuntimeError(f"at most {MAX_CHANNELS} channels")
    if tuple(target.shape) != (channels, h, w):
        raise RuntimeError(f"target must be [{channels}, {h}, {w}]")
    n = xys.size(0)
    dev = xys.device
    num_tiles = int(tile_bounds[0]) * int(tile_bounds[1])
    lib = _lib.load()
    out_img = torch.empty(channels, h, w, device=dev, dtype=torch.float32)
    v_output = torch.empty_like(out_img) if with_v_output else None
    loss = torch.empty((), device=dev, dtype=torch.float32)
    grads = torch.empty(n * (5 + channels), device=dev, dtype=torch.float32)
    v_xy, v_conic, v_colors = grads[:2 * n].view(n, 2), grads[2 * n:5 * n].view(n, 3), grads[5 * n:].view(n, channels)
    ws_bytes = lib.igs_raster_l1_workspace(num_tiles)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib_call("igs_raster_step_l1", int(tile_bounds[0]), int(tile_bounds[1]), h, w, channels, n, ptr(gaussian_ids_sorted),
                  ptr(tile_bins), ptr(xys), ptr(conics), ptr(colors), ptr(target), float(ratio), ptr(out_img), ptr(loss), ptr(v_output),
                  ptr(v_xy), ptr(v_conic), ptr(v_colors), ptr(ws), ws_bytes, stream_of(dev))
    out = (out_img, loss, v_xy, v_conic, v_colors)
    return out + (v_output,) if with_v_output else out


def nd_rasterize_backward_topk_norm(img_height, img_width, BLOCK_H, BLOCK_W, xys, conics, colors, v_output, pixel_topk):
    """-> v_xy [N,2], v_conic [N,3], v_colors [N,C] (bindings.cu:444-502); v_output channel-planar [C,H,W]."""
    for t, n in ((xys, "xys"), (conics, "conics"), (colors, "colors"), (v_output, "v_output")):
        _check_input(t, n, torch.float32)
    _check_input(pixel_topk, "pixel_topk", torch.int32)
    if xys.ndim != 2 or xys.size(1) != 2:
        raise RuntimeError("xys must have dimensions (num_points, 2)")
    if colors.ndim != 2:
        raise RuntimeError("colors must have 2 dimensions")
    if BLOCK_W % 8 != 0 or BLOCK_H % 4 != 0 or (BLOCK_H, BLOCK_W) != (TILE, TILE):
        raise RuntimeError(f"the block must be {TILE}x{TILE} (warps cover 8x4 pixels)")
    channels = colors.size(1)
    if channels > MAX_CHANNELS:
        raise RuntimeError("at most MAX_CHANNELS channels")
    n = xys.size(0)
    dev = xys.device
    grads = torch.empty(n * (5 + channels), device=dev, dtype=torch.float32)
    v_xy, v_conic, v_colors = grads[:2 * n].view(n, 2), grads[2 * n:5 * n].view(n, 3), grads[5 * n:].view(n, channels)
    with torch.cuda.device(dev):
        _lib_call("igs_raster_bwd_topk", int(img_height), int(img_width), channels, n, ptr(xys), ptr(conics), ptr(colors), ptr(v_output),
                  ptr(pixel_topk), ptr(v_xy), ptr(v_conic), ptr(v_colors), stream_of(dev))
    return v_xy, v_conic, v_colors


def nd_rasterize_backward_topk_norm_tiles(img_height, img_width, gaussian_ids_sorted, tile_bins, xys, conics, colors, v_output, tile_topk):
    """Backward pass from the tile-list form of the top-K lists."""
    channels = colors.size(1)
    n = xys.size(0)
    dev = xys.device
    grads = torch.empty(n * (5 + channels), device=dev, dtype=torch.float32)
    v_xy, v_conic, v_colors = grads[:2 * n].view(n, 2), grads[2 * n:5 * n].view(n, 3), grads[5 * n:].view(n, channels)
    with torch.cuda.device(dev):
        _lib_call("igs_raster_bwd_topk_tiles", int(img_height), int(img_width), channels, n, ptr(gaussian_ids_sorted), ptr(tile_bins),
                  ptr(xys), ptr(conics), ptr(colors), ptr(v_output), ptr(tile_topk), ptr(v_xy), ptr(v_conic), ptr(v_colors),
                  stream_of(dev))
    return v_xy, v_conic, v_colors


def topk_norm_loo_loss_increase(img_height, img_width, xys, conics, colors, pixel_topk, targets, squared, eps):
    """-> loss_increase [N] (bindings.cu:895-936)."""
    for t, n in ((xys, "xys"), (conics, "conics"), (colors, "colors"), (targets, "targets")):
        _check_input(t, n, torch.float32)
    _check_input(pixel_topk, "pixel_topk", torch.int32)
    channels = colors.size(1)
    if channels > MAX_CHANNELS:
        raise RuntimeError("at most MAX_CHANNELS channels")
    if targets.numel() != channels * img_height * img_width:
        raise RuntimeError("targets must be [C, H, W]")
    if pixel_topk.numel() != img_height * img_width * TOP_K:
        raise RuntimeError("pixel_topk must be [H, W, TOP_K]")
    dev = xys.device
    out = torch.empty(xys.size(0), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib_call("igs_loo_loss_increase", int(img_height), int(img_width), channels, xys.size(0), ptr(xys), ptr(conics), ptr(colors),
                  ptr(pixel_topk), ptr(targets), int(bool(squared)), float(eps), ptr(out), stream_of(dev))
    return out


def topk_feature_weights_fixed(img_height, img_width, xys, conics, pixel_topk, eps=EPS):
    """Per-Gaussian sum over pixels of the squared normalized top-K weight as int64 fixed point with 40 fractional bits: the integer sums
    of compress.quantization.feature_weights (quantization.py:218-230) over model._iter_topk_weights (model.py:1404-1421)."""
    for t, n in ((xys, "xys"), (conics, "conics")):
        _check_input(t, n, torch.float32)
    _check_input(pixel_topk, "pixel_topk", torch.int32)
    if pixel_topk.numel() != img_height * img_width * TOP_K:
        raise RuntimeError("pixel_topk must be [H, W, TOP_K]")
    dev = xys.device
    out = torch.empty(xys.size(0), device=dev, dtype=torch.int64)
    with torch.cuda.device(dev):
        _lib_call("igs_feature_weights", int(img_height), int(img_width), xys.size(0), ptr(xys), ptr(conics), ptr(pixel_topk), float(eps),
                  ptr(out), stream_of(dev))
    return out


def topk_feature_weights(img_height, img_width, xys, conics, pixel_topk, eps=EPS):
    """compress.quantization.feature_weights(model._iter_topk_weights(...)) -> [N] float64."""
    return topk_feature_weights_fixed(img_height, img_width, xys, conics, pixel_topk, eps).to(torch.float64) / 2.0**40


# ---- losses, quantization, rate term -------------------------------------------------------------------------------------------------

def l1_loss_and_grad(image: torch.Tensor, target: torch.Tensor, ratio: float = 1.0, workspace: Optional[torch.Tensor] = None):
    """(ratio * mean|image - target| as a 0-dim tensor, its gradient with respect to image), in one pass."""
    _check_input(image, "image", torch.float32)
    _check_input(target, "target", torch.float32)
    if image.shape != target.shape:
        raise ValueError(f"image {tuple(image.shape)} and target {tuple(target.shape)} differ")
    dev = image.device
    numel = image.numel()
    loss = torch.empty((), device=dev, dtype=torch.float32)
    grad = torch.empty_like(image)
    ws_bytes = _lib.load().igs_l1_workspace(numel)
    if workspace is None:
        workspace = torch.zeros(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib_call("igs_l1_loss", numel, ptr(image), ptr(target), float(ratio), ptr(loss), ptr(grad), ptr(workspace), ws_bytes,
                  stream_of(dev))
    return loss, grad


def l1_loss_signs(image: torch.Tensor, target: torch.Tensor, ratio: float = 1.0, workspace: Optional[torch.Tensor] = None):
    """(ratio * mean|image - target| as a 0-dim tensor, sign(image - target) as int8), in one pass; see igs_l1_loss_signs."""
    _check_input(image, "image", torch.float32)
    _check_input(target, "target", torch.float32)
    if image.shape != target.shape:
        raise ValueError(f"image {tuple(image.shape)} and target {tuple(target.shape)} differ")
    dev = image.device
    loss = torch.empty((), device=dev, dtype=torch.float32)
    signs = torch.empty(image.shape, device=dev, dtype=torch.int8)
    ws_bytes = _lib.load().igs_l1_workspace(image.numel())
    if workspace is None:
        workspace = torch.zeros(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib_call("igs_l1_loss_signs", image.numel(), ptr(image), ptr(target), float(ratio), ptr(loss), ptr(signs), ptr(workspace),
                  ws_bytes, stream_of(dev))
    return loss, signs


def l1_grad_from_signs(signs: torch.Tensor, grad_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """sign * (g / numel) as float32 (g = grad_scale, a device scalar, or 1): the gradient of mean|image - target|, as ATen forms it."""
    _check_input(signs, "signs", torch.int8)
    dev = signs.device
    grad = torch.empty(signs.shape, device=dev, dtype=torch.float32)
    scale = None
    if grad_scale is not None:
        scale = grad_scale.detach().to(device=dev, dtype=torch.float32).contiguous()
        if scale.numel() != 1:
            raise ValueError("grad_scale must hold one value")
    with torch.cuda.device(dev):
        _lib_call("igs_l1_grad_from_signs", signs.numel(), ptr(signs), ptr(scale) if scale is not None else None, ptr(grad),
                  stream_of(dev))
    return grad


def quantize_ste_forward(xy, scale, rot, feat, pos_steps, scale_step, rot_step, feat_steps, feat_transform=None, with_symbols=False):
    """Straight-through step quantization values (and optionally symbols and loss-space features); see igs_quantize_ste."""
    for t, n in ((xy, "xy"), (scale, "scale"), (rot, "rot"), (feat, "feat"), (pos_steps, "pos_steps"), (feat_steps, "feat_steps")):
        _check_input(t, n, torch.float32)
    n, channels = feat.shape
    dev = xy.device
    out = [torch.empty_like(xy), torch.empty_like(scale), torch.empty_like(rot), torch.empty_like(feat)]
    out_t = torch.empty_like(feat) if feat_transform is not None else None
    sym = [torch.empty_like(xy), torch.empty_like(scale), torch.empty_like(rot), torch.empty_like(feat)] if with_symbols else [None] * 4
    if feat_transform is not None:
        _check_input(feat_transform, "feat_transform", torch.float32)
    with torch.cuda.device(dev):
        _lib_call("igs_quantize_ste", n, channels, ptr(xy), ptr(scale), ptr(rot), ptr(feat), ptr(pos_steps), float(scale_step),
                  float(rot_step), ptr(feat_steps), ptr(feat_transform), *[ptr(t) for t in out], ptr(out_t), *[ptr(t) for t in sym],
                  stream_of(dev))
    return out, out_t, (sym if with_symbols else None)


def rate_loss_forward(feat, rot, l1_loss, neighbors, weights, slope, color_refs, pred_refs, inv_steps, feat_coeffs, rot_coeffs,
                      inv_rot_step, l1_ratio, factor):
    """-> loss (0-dim), loss_weight [1], own_grad [N,C], rot_grad [N] (rate.cu:201-279)."""
    for t, n in ((feat, "feat"), (rot, "rot"), (l1_loss, "l1_loss"), (weights, "weights"), (slope, "slope"), (inv_steps, "inv_steps"),
                 (feat_coeffs, "feat_coeffs"), (rot_coeffs, "rot_coeffs")):
        _check_input(t, n, torch.float32)
    _check_input(neighbors, "neighbors", torch.int32)
    num, channels = feat.shape
    if channels > MAX_CHANNELS:
        raise RuntimeError("at most MAX_CHANNELS feature channels")
    if len(color_refs) != channels or len(pred_refs) != channels:
        raise RuntimeError("one reference per channel")
    if rot.numel() != num or rot_coeffs.numel() != num:
        raise RuntimeError("one rotation per Gaussian")
    if neighbors.size(0) != num or weights.shape != neighbors.shape:
        raise RuntimeError("neighbors and weights must be [P, K]")
    dev = feat.device
    loss = torch.empty((), device=dev, dtype=torch.float32)
    loss_weight = torch.empty(1, device=dev, dtype=torch.float32)
    own_grad = torch.empty_like(feat)
    rot_grad = torch.empty(num, device=dev, dtype=torch.float32)
    ws_bytes = _lib.load().igs_rate_workspace(num)
    ws = torch.zeros(ws_bytes, device=dev, dtype=torch.uint8)
    import ctypes
    crefs = (ctypes.c_int32 * channels)(*[int(c) for c in color_refs])
    prefs = (ctypes.c_int32 * channels)(*[int(c) for c in pred_refs])
    with torch.cuda.device(dev):
        _lib_call("igs_rate_fwd", num, channels, neighbors.size(1), ptr(feat), ptr(rot), ptr(l1_loss), ptr(neighbors), ptr(weights),
                  ptr(slope), ctypes.cast(crefs, ctypes.c_void_p), ctypes.cast(prefs, ctypes.c_void_p), ptr(inv_steps), ptr(feat_coeffs),
                  ptr(rot_coeffs), float(inv_rot_step), float(l1_ratio), float(factor), ptr(loss), ptr(loss_weight), ptr(own_grad),
                  ptr(rot_grad), ptr(ws), ws_bytes, stream_of(dev))
    return loss, loss_weight, own_grad, rot_grad


def rate_loss_backward(grad_loss, loss_weight, own_grad, rot_grad, offsets, sources, source_weights):
    """-> grad_feat [N,C], grad_rot [N] (rate.cu:281-321)."""
    for t, n in ((grad_loss, "grad_loss"), (loss_weight, "loss_weight"), (own_grad, "own_grad"), (rot_grad, "rot_grad"),
                 (source_weights, "source_weights")):
        _check_input(t, n, torch.float32)
    _check_input(offsets, "offsets", torch.int32)
    _check_input(sources, "sources", torch.int32)
    num, channels = own_grad.shape
    if offsets.numel() != num + 1:
        raise RuntimeError("offsets must be [P + 1]")
    dev = own_grad.device
    grad_feat = torch.empty_like(own_grad)
    grad_rot = torch.empty_like(rot_grad)
    with torch.cuda.device(dev):
        _lib_call("igs_rate_bwd", num, channels, ptr(grad_loss), ptr(loss_weight), ptr(own_grad), ptr(rot_grad), ptr(offsets),
                  ptr(sources), ptr(source_weights), ptr(grad_feat), ptr(grad_rot), stream_of(dev))
    return grad_feat, grad_rot
