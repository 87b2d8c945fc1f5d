"""
The fused training-step kernel (igs_raster_step_l1): the top-K forward pass, the L1 loss and the top-K backward pass of each tile in one
kernel. Against the separate kernels on the same inputs (forward with the fused loss, then the backward from the 16-bit tile lists):
  * the image and the image gradient are identical bit for bit;
  * the loss agrees up to the float summation order of the per-tile partial sums;
  * the gradients agree up to the order of the float atomics across tiles (each tile's sums are the same).
Short lists (one staged chunk), lists of several chunks of 256 entries, 1, 3 and 9 channels, and ragged edge tiles; the pipeline's fused
step against its two-kernel step (the tile lists beyond 16-bit positions are covered in test_gpu_parity.py).
"""
import math

import pytest
import torch

from common import assert_close_grad, make_case, to_dev
from igs_b200 import ops, pipeline

pytestmark = pytest.mark.gpu

CASES = [
    dict(h=88, w=120, n=300, seed=11),  # short lists, ragged edge tiles
    dict(h=64, w=80, n=200, c=9, seed=13),
    dict(h=50, w=70, n=150, c=1, seed=12),
    dict(h=48, w=64, n=3000, log_scale_mean=math.log(12.0), log_scale_std=0.2, seed=14),  # lists of 1,000+ entries: several chunks
]


def separate_and_fused(d, h, w, ratio):
    n = d["means"].shape[0]
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum, total = ops.cumulative_intersects(hits)
    cap = int(total.item())
    ids, bins = ops.sort_intersects_by_tile(n, cap, xys, radii, cum, tb)
    feats, target = d["features"], d["target"]
    img, tile_topk, loss, v_out = ops.nd_rasterize_forward_topk_norm_tiles_l1(tb, (w, h, 1), cap, ids, bins, xys, conics, feats, target,
                                                                             ratio=ratio)
    grads = ops.nd_rasterize_backward_topk_norm_tiles(h, w, ids, bins, xys, conics, feats, v_out, tile_topk)
    fused = ops.raster_step_l1(tb, (w, h, 1), ids, bins, xys, conics, feats, target, ratio=ratio, with_v_output=True)
    lens = bins[:, 1] - bins[:, 0]
    return (img, loss, v_out) + tuple(grads), fused, int(lens.max())


@pytest.mark.parametrize("case", CASES)
def test_fused_step_matches_separate_kernels(case, device):
    kw = dict(case)
    h, w = kw.pop("h"), kw.pop("w")
    _, inp = make_case(h, w, **kw)
    d = to_dev(inp, device)
    (img, loss, v_out, v_xy, v_conic, v_colors), (f_img, f_loss, f_xy, f_conic, f_colors, f_vout), longest = separate_and_fused(d, h, w, 0.8)
    if case["n"] == 3000:
        assert longest > 512, longest  # the chunked path is exercised
    assert torch.equal(f_img, img)
    assert torch.equal(f_vout, v_out)
    assert abs(float(f_loss) - float(loss)) <= 2e-6 * abs(float(loss))
    for a, b, name in ((f_xy, v_xy, "v_xy"), (f_conic, v_conic, "v_conic"), (f_colors, v_colors, "v_colors")):
        assert_close_grad(a, b, rtol=1e-5, what=name)


def test_fused_step_is_repeatable_and_rejects_bad_arguments(device):
    h, w = 40, 56
    _, inp = make_case(h, w, 120, seed=15)
    d = to_dev(inp, device)
    _, first, _ = separate_and_fused(d, h, w, 1.0)
    _, second, _ = separate_and_fused(d, h, w, 1.0)
    assert torch.equal(first[0], second[0]) and float(first[1]) == float(second[1])  # image and loss: deterministic
    tb = ops.tile_grid(h, w)
    with pytest.raises(RuntimeError, match="target"):
        ops.raster_step_l1(tb, (w, h, 1), torch.zeros(1, dtype=torch.int32, device=device), torch.zeros(tb[0] * tb[1], 2, dtype=torch.int32,
                           device=device), torch.zeros(1, 2, device=device), torch.zeros(1, 3, device=device), torch.zeros(1, 3, device=device),
                           torch.zeros(3, h + 1, w, device=device))


@pytest.mark.parametrize("name", ["plain", "cfg2_480p_yuv"])
def test_pipeline_fused_step_matches_two_kernel_step(name, device):
    from igs_b200 import workloads

    if name == "plain":
        wl, inp = make_case(120, 200, 800, seed=61)
        opts = {}
    else:
        import bench

        wl = workloads.get_workload(name)
        inp = workloads.make_inputs(wl)
        opts = bench.step_options(wl, device)
    d = to_dev(inp, device)
    target = d["loss_target"] if "loss_target" in d else d["target"]
    steps = [pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], target, fused=f, **opts) for f in (True, False)]
    for s in steps:
        s.replay()
    torch.cuda.synchronize()
    fused, split = steps
    assert torch.equal(fused.image, split.image)
    assert abs(float(fused.loss) - float(split.loss)) <= 2e-6 * float(split.loss)
    names = ["v_mean2d", "v_scale", "v_rot", "v_colors"] + (["v_feat"] if opts else [])
    for k in names:  # summation order only (float atomics; the rate term's and the loss transform's sums amplify it slightly)
        assert_close_grad(getattr(fused, k), getattr(split, k), what=k)


@pytest.mark.parametrize("case", ["no_gaussians", "one_pixel", "truncated_lists"])
def test_fused_step_edge_cases(case, device):
    """No Gaussians (the image is zero, the loss is ratio * mean|target|), a 1x1 image, and lists cut short by a capacity below the
    intersection count: the fused kernel agrees with the separate kernels."""
    h, w, n = {"no_gaussians": (40, 56, 0), "one_pixel": (1, 1, 5), "truncated_lists": (64, 80, 400)}[case]
    _, inp = make_case(h, w, max(n, 1), seed=17)
    d = to_dev(inp, device)
    if n == 0:
        d = {k: (v[:0] if k in ("means", "scales", "rotations", "features") else v) for k, v in d.items()}
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum, total = ops.cumulative_intersects(hits)
    cap = int(total.item()) if n else 0
    if case == "truncated_lists":
        cap //= 2
    feats, target = d["features"], d["target"]
    ids, bins = ops.sort_intersects_by_tile(n, max(cap, 1) if n else 0, xys, radii, cum, tb)
    f_img, f_loss, f_xy, f_conic, f_colors = ops.raster_step_l1(tb, (w, h, 1), ids, bins, xys, conics, feats, target, ratio=0.5)
    if n == 0:
        assert not bool(f_img.any())
        assert abs(float(f_loss) - 0.5 * float(target.abs().mean())) <= 2e-6 * float(target.abs().mean())
        return
    img, tile_topk, loss, v_out = ops.nd_rasterize_forward_topk_norm_tiles_l1(tb, (w, h, 1), max(cap, 1), ids, bins, xys, conics, feats,
                                                                             target, ratio=0.5)
    v_xy, v_conic, v_colors = ops.nd_rasterize_backward_topk_norm_tiles(h, w, ids, bins, xys, conics, feats, v_out, tile_topk)
    assert torch.equal(f_img, img)
    assert abs(float(f_loss) - float(loss)) <= 2e-6 * max(abs(float(loss)), 1e-30)
    for a, b, name in ((f_xy, v_xy, "v_xy"), (f_conic, v_conic, "v_conic"), (f_colors, v_colors, "v_colors")):
        assert_close_grad(a, b, rtol=1e-5, what=name)
