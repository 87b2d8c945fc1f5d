"""
ORACLE (test infrastructure): numpy front end of the C restatement oracle.c (built into oracle/liboracle.so by oracle/Makefile). Each
function follows the reference function cited in oracle.c; arrays are float32 / int32 numpy arrays, outputs freshly allocated.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
_lib = None


def build():
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(os.path.join(HERE, "oracle.c")):
        subprocess.run(["make", "-C", HERE, "CC=gcc", "-s"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB)
        _lib.orc_sort_intersects.restype = ctypes.c_int
    return _lib


def set_threads(n):
    lib().orc_set_threads(int(n))


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _i32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def tile_grid(h, w):
    return (int(w) + 15) // 16, (int(h) + 15) // 16


def project_fwd(means, scales, rot, h, w):
    """foward2d.cu:9-59 -> xys [N,2], radii [N], conics [N,3], num_tiles_hit [N]"""
    means, scales, rot = _f32(means), _f32(scales), _f32(rot).reshape(-1)
    n = len(means)
    tx, ty = tile_grid(h, w)
    xys, conics = np.zeros((n, 2), np.float32), np.zeros((n, 3), np.float32)
    radii, hits = np.zeros(n, np.int32), np.zeros(n, np.int32)
    lib().orc_project_fwd(n, _p(means), _p(scales), _p(rot), int(h), int(w), tx, ty, _p(xys), _p(radii), _p(conics), _p(hits))
    return xys, radii, conics, hits


def project_bwd(scales, rot, h, w, radii, conics, v_xy, v_conic):
    """backward2d.cu:53-100 -> v_cov2d [N,3], v_mean2d [N,2], v_scale [N,2], v_rot [N,1]"""
    scales, rot, radii, conics = _f32(scales), _f32(rot).reshape(-1), _i32(radii), _f32(conics)
    v_xy, v_conic = _f32(v_xy), _f32(v_conic)
    n = len(scales)
    v_cov2d, v_mean2d = np.zeros((n, 3), np.float32), np.zeros((n, 2), np.float32)
    v_scale, v_rot = np.zeros((n, 2), np.float32), np.zeros((n, 1), np.float32)
    lib().orc_project_bwd(n, _p(scales), _p(rot), int(h), int(w), _p(radii), _p(conics), _p(v_xy), _p(v_conic), _p(v_cov2d), _p(v_mean2d),
                          _p(v_scale), _p(v_rot))
    return v_cov2d, v_mean2d, v_scale, v_rot


def cumsum(hits):
    hits = _i32(hits)
    out = np.zeros_like(hits)
    lib().orc_cumsum(len(hits), _p(hits), _p(out))
    return out


def sort_intersects(num_points, capacity, xys, radii, cum, h, w):
    """bindings.cu:106-167 -> gaussian_ids_sorted [capacity], tile_bins [T,2]"""
    xys, radii, cum = _f32(xys), _i32(radii), _i32(cum)
    tx, ty = tile_grid(h, w)
    ids = np.zeros(max(int(capacity), 0), np.int32)
    bins = np.zeros((tx * ty, 2), np.int32)
    lib().orc_sort_intersects(int(num_points), int(capacity), _p(xys), _p(radii), _p(cum), tx, ty, _p(ids), _p(bins))
    return ids, bins


def raster_fwd(h, w, ids_sorted, tile_bins, xys, conics, colors):
    """forward.cu:223-375 -> out_img [C,H,W], pixel_topk [H,W,10]"""
    ids_sorted, tile_bins, xys, conics, colors = _i32(ids_sorted), _i32(tile_bins), _f32(xys), _f32(conics), _f32(colors)
    c = colors.shape[1]
    tx, ty = tile_grid(h, w)
    h, w = int(h), int(w)
    out = np.zeros((c, h, w), np.float32)
    topk = np.zeros((h, w, 10), np.int32)
    lib().orc_raster_fwd(tx, ty, int(h), int(w), c, _p(ids_sorted), _p(tile_bins), _p(xys), _p(conics), _p(colors), _p(out), _p(topk))
    return out, topk


def raster_bwd(h, w, xys, conics, colors, v_output, pixel_topk):
    """backward.cu:187-308 (sums in double) -> v_xy [N,2], v_conic [N,3], v_colors [N,C]"""
    xys, conics, colors, v_output, pixel_topk = _f32(xys), _f32(conics), _f32(colors), _f32(v_output), _i32(pixel_topk)
    n, c = colors.shape
    v_xy, v_conic, v_colors = np.zeros((n, 2), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, c), np.float32)
    lib().orc_raster_bwd(int(h), int(w), c, n, _p(xys), _p(conics), _p(colors), _p(v_output), _p(pixel_topk), _p(v_xy), _p(v_conic), _p(v_colors))
    return v_xy, v_conic, v_colors


def raster_bwd_abs(h, w, xys, conics, colors, v_output, pixel_topk):
    """The sums of |term| behind each gradient value of raster_bwd (the float-rounding scale of a summed gradient) -> v_xy, v_conic,
    v_colors magnitudes"""
    xys, conics, colors, v_output, pixel_topk = _f32(xys), _f32(conics), _f32(colors), _f32(v_output), _i32(pixel_topk)
    n, c = colors.shape
    v_xy, v_conic, v_colors = np.zeros((n, 2), np.float32), np.zeros((n, 3), np.float32), np.zeros((n, c), np.float32)
    lib().orc_raster_bwd_abs(int(h), int(w), c, n, _p(xys), _p(conics), _p(colors), _p(v_output), _p(pixel_topk), _p(v_xy), _p(v_conic),
                             _p(v_colors))
    return v_xy, v_conic, v_colors


def loo_loss_increase(h, w, xys, conics, colors, pixel_topk, targets, squared, eps):
    """forward.cu:667-738 -> loss_increase [N]"""
    xys, conics, colors, pixel_topk, targets = _f32(xys), _f32(conics), _f32(colors), _i32(pixel_topk), _f32(targets)
    n, c = colors.shape
    out = np.zeros(n, np.float32)
    lib().orc_loo_loss_increase(int(h), int(w), c, n, _p(xys), _p(conics), _p(colors), _p(pixel_topk), _p(targets), int(bool(squared)),
                                ctypes.c_float(eps), _p(out))
    return out


def l1_loss_and_grad(image, target, ratio=1.0):
    """model.py:1224-1227: ratio * mean|image - target| (double sum) and sign(image - target) * ratio / numel"""
    image, target = _f32(image), _f32(target)
    d = image - target
    loss = ratio * float(np.abs(d.astype(np.float64)).sum() / d.size)
    grad = (np.sign(d) * np.float32(np.float32(ratio) / np.float32(d.size))).astype(np.float32)
    return loss, grad


def train_step(means, scales, rot, colors, target, h, w, capacity=None):
    """One forward + L1 backward of the rasterization path on the CPU: projection, binning, top-K forward, L1 loss, top-K backward,
    projection backward. Returns a dict of every intermediate and gradient."""
    n = len(means)
    xys, radii, conics, hits = project_fwd(means, scales, rot, h, w)
    cum = cumsum(hits)
    total = int(cum[-1]) if n else 0
    cap = total if capacity is None else capacity
    ids, bins = sort_intersects(n, cap, xys, radii, cum, h, w)
    image, topk = raster_fwd(h, w, ids, bins, xys, conics, colors)
    loss, v_image = l1_loss_and_grad(image, target)
    v_xy, v_conic, v_colors = raster_bwd(h, w, xys, conics, colors, v_image, topk)
    v_cov2d, v_mean2d, v_scale, v_rot = project_bwd(scales, rot, h, w, radii, conics, v_xy, v_conic)
    return dict(xys=xys, radii=radii, conics=conics, num_tiles_hit=hits, cum=cum, num_intersects=total, gaussian_ids_sorted=ids,
                tile_bins=bins, image=image, pixel_topk=topk, loss=loss, v_image=v_image, v_xy=v_xy, v_conic=v_conic, v_colors=v_colors,
                v_mean2d=v_mean2d, v_scale=v_scale, v_rot=v_rot)
