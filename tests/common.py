"""
Test helpers: the rasterization step run stage by stage through our operators, through the reference's own extension (oracle/_ref) and
through the CPU oracle, and comparisons with the tolerances of the parity contract (integers bit-exact; renders within 1e-5 relative;
gradients within 1e-4 relative, measured against max(|b|, 1e-3 * max|b|) per tensor because atomics reorder float sums).
"""
import hashlib
import math

import numpy as np
import torch

from igs_b200 import ops, workloads

RENDER_RTOL = 1e-5
GRAD_RTOL = 1e-4
GRAD_FLOOR = 1e-3  # relative to the tensor's largest magnitude


def np_(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


def digest(a):
    a = np.ascontiguousarray(np_(a))
    return hashlib.sha256(a.tobytes()).hexdigest()[:24]


RENDER_FLOOR = 0.05  # relative to the image's largest magnitude: signed features cancel, so single pixels can sit arbitrarily near 0


def assert_close_render(actual, expected, rtol=RENDER_RTOL, floor=RENDER_FLOOR, what="render"):
    """|a - b| <= rtol * max(|b|, floor * max|b|) elementwise."""
    a, b = np_(actual).astype(np.float64), np_(expected).astype(np.float64)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if b.size == 0:
        return 0.0
    err = np.abs(a - b) / np.maximum(np.abs(b), floor * np.abs(b).max() + 1e-30)
    worst = float(err.max()) if err.size else 0.0
    assert worst <= rtol, f"{what}: max relative error {worst:.3g} > {rtol:g} at {np.unravel_index(err.argmax(), err.shape)}"
    return worst


# A float32 sum of many terms, added in two different orders (unordered atomics in the reference, per-tile sums here), differs by up to
# a small multiple of the unit roundoff 2^-24 times the sum of the terms' magnitudes, however much the terms cancel. Where a gradient
# value is a near-cancelling sum (L1 gradients are sums of +-w: a Gaussian whose pixels lie above and below the target in equal measure),
# that rounding can exceed 1e-4 of the value itself, so full-size comparisons also accept a difference within SUM_NOISE times the
# magnitude sum (oracle.cpu.raster_bwd_abs). A wrong term shifts a value by far more than that.
SUM_NOISE = 64 * 2.0 ** -24


def assert_close_grad(actual, expected, rtol=GRAD_RTOL, floor=GRAD_FLOOR, what="grad", abs_sum=None):
    """|a - b| <= rtol * max(|b|, floor * max|b|) elementwise, or, given the sums of the terms' magnitudes behind each value,
    |a - b| <= SUM_NOISE * abs_sum."""
    a, b = np_(actual).astype(np.float64), np_(expected).astype(np.float64)
    assert a.shape == b.shape, f"{what}: shape {a.shape} != {b.shape}"
    if b.size == 0:
        return 0.0
    scale = np.maximum(np.abs(b), floor * np.abs(b).max() + 1e-30)
    err = np.abs(a - b) / scale
    if abs_sum is not None:
        noise = SUM_NOISE * np_(abs_sum).astype(np.float64).reshape(b.shape)
        err = np.where(np.abs(a - b) <= noise, 0.0, err)
    worst = float(err.max())
    assert worst <= rtol, f"{what}: max scaled error {worst:.3g} > {rtol:g} at {np.unravel_index(err.argmax(), err.shape)}"
    return worst


def raster_grad_abs_sums(h, w, xys, conics, colors, v_output, pixel_topk):
    """The sums of |term| behind v_xy, v_conic and v_colors (the CPU oracle on the given lists and image gradient)."""
    from oracle import cpu as orc

    sums = orc.raster_bwd_abs(h, w, np_(xys), np_(conics), np_(colors), np_(v_output), np_(pixel_topk))
    return dict(zip(("v_xy", "v_conic", "v_colors"), sums))


def make_case(h, w, n, c=3, log_scale_mean=math.log(2.0), log_scale_std=0.5, max_anisotropy=None, seed=7):
    wl = workloads.custom_workload(h, w, n, c, log_scale_mean, log_scale_std, max_anisotropy, seed=seed)
    return wl, workloads.make_inputs(wl)


def to_dev(inputs, device):
    return {k: v.to(device) for k, v in inputs.items()}


def ours_stages(inp, h, w, capacity=None, v_output=None):
    """Our operators, stage by stage, on device tensors: dict of every intermediate (device tensors)."""
    n = inp["means"].shape[0]
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, inp["means"], inp["scales"], inp["rotations"], h, w, tb)
    cum, total = ops.cumulative_intersects(hits)
    num_isect = int(total.item())
    cap = num_isect if capacity is None else capacity
    ids, bins = ops.sort_intersects_by_tile(n, cap, xys, radii, cum, tb)
    out = dict(xys=xys, radii=radii, conics=conics, num_tiles_hit=hits, cum=cum, num_intersects=num_isect, capacity=cap,
               gaussian_ids_sorted=ids, tile_bins=bins)
    if cap <= 0:
        return out
    image, topk = ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, inp["features"])
    out.update(image=image, pixel_topk=topk)
    if v_output is None:
        _, v_output = ops.l1_loss_and_grad(image, inp["target"])
    out["v_output"] = v_output
    v_xy, v_conic, v_colors = ops.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, inp["features"], v_output, topk)
    v_cov2d, v_mean2d, v_scale, v_rot = ops.project_gaussians_2d_scale_rot_backward(n, inp["means"], inp["scales"], inp["rotations"], h, w,
                                                                                    radii, conics, v_xy, v_conic)
    out.update(v_xy=v_xy, v_conic=v_conic, v_colors=v_colors, v_cov2d=v_cov2d, v_mean2d=v_mean2d, v_scale=v_scale, v_rot=v_rot)
    return out


def reference_stages(ref, inp, h, w, capacity=None, v_output=None, xys=None, radii=None, conics=None, hits=None):
    """The reference extension's pybind functions in the order of rasterize_sum.py's top-K path; projection outputs may be given so
    that later stages see exactly our inputs."""
    n = inp["means"].shape[0]
    tb = ops.tile_grid(h, w)
    if xys is None:
        xys, radii, conics, hits = ref.project_gaussians_2d_scale_rot_forward(n, inp["means"], inp["scales"], inp["rotations"], h, w, tb)
    cum = torch.cumsum(hits, dim=0, dtype=torch.int32)
    num_isect = int(cum[-1].item())
    cap = num_isect if capacity is None else capacity
    ids, bins = ref.sort_intersects_by_tile(n, cap, xys, radii, cum, tb)
    out = dict(xys=xys, radii=radii, conics=conics, num_tiles_hit=hits, cum=cum, num_intersects=num_isect, capacity=cap,
               gaussian_ids_sorted=ids, tile_bins=bins)
    if cap <= 0:
        return out
    image, topk = ref.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys.contiguous(), conics.contiguous(),
                                                     inp["features"])
    out.update(image=image, pixel_topk=topk)
    if v_output is not None:
        v_xy, v_conic, v_colors = ref.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, inp["features"], v_output, topk)
        v_cov2d, v_mean2d, v_scale, v_rot = ref.project_gaussians_2d_scale_rot_backward(n, inp["means"], inp["scales"], inp["rotations"],
                                                                                        h, w, radii, conics, v_xy, v_conic)
        out.update(v_output=v_output, v_xy=v_xy, v_conic=v_conic, v_colors=v_colors, v_cov2d=v_cov2d, v_mean2d=v_mean2d, v_scale=v_scale,
                   v_rot=v_rot)
    return out


def alpha_ties(xys, conics, ids_sorted, tile_bins, tiles_x, pixels, rel=1e-5):
    """For each (i, j) pixel, whether two of its tile's alpha values lie within `rel` of each other or one lies near the flush-to-zero
    threshold: the near-ties where float32 exp implementations may order Gaussians differently."""
    xys, conics, ids_sorted, tile_bins = np_(xys), np_(conics), np_(ids_sorted), np_(tile_bins)
    flags = []
    for i, j in pixels:
        t = (i // 16) * tiles_x + j // 16
        s, e = tile_bins[t]
        g = ids_sorted[s:e]
        dx, dy = xys[g, 0].astype(np.float64) - j, xys[g, 1].astype(np.float64) - i
        c = conics[g].astype(np.float64)
        sig = 0.5 * (c[:, 0] * dx * dx + c[:, 2] * dy * dy) + c[:, 1] * dx * dy
        a = np.sort(np.exp(-sig[sig >= 0]))
        near = bool(np.any(np.abs(sig - 87.3365) < 0.01))
        if len(a) > 1:
            gaps = np.diff(a) / np.maximum(a[1:], 1e-300)
            near = near or bool(np.any(gaps < rel))
        flags.append(near)
    return np.array(flags, dtype=bool)
