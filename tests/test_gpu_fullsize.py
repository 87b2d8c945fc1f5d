"""
Parity at the benchmark's own sizes, on the kernels the benchmark times, against the reference's extension built from source
(oracle/_ref) running on the same GPU, and against the committed digests of the reference's outputs (tests/golden/ref_cfg3_1080p.npz):
  * 1920x1080 with 20,000 Gaussians (the headline step): every stage of the operator path, at full and at half capacity, and the fused
    training-step kernel (forward, L1 loss and backward in one kernel);
  * 3840x2160 with 80,000 Gaussians in 2, 4 and 8 tile-row bands: each band's fused step run alone on one GPU, as one rank of the
    multi-GPU step, against the reference's whole-image kernels;
  * one 2048x2048 image of the 9-channel texture stack with 50,000 Gaussians (the reference's 16-value backward path);
  * the 854x480 YUV step with the straight-through quantizer, the loss-space transform and the rate term, against the reference's kernels
    composed with the oracle's restatement of its quantization code (ATen on the GPU, bit-exact symbols).
Integers (radii, tile counts, prefix sums, tile lists, top-K lists, quantization symbols) must be bit-exact and renders within 1e-5. The
rasterizer's gradients (v_xy, v_conic, v_colors) must be within 1e-4, or within the float32 rounding of their sums where the terms cancel
(tests/common.py: SUM_NOISE times the sum of the terms' magnitudes, from the CPU oracle). The projection backward is compared stage-wise:
the reference's kernel gets our v_xy and v_conic. The reference's backward pass gets the image gradient of our render, so that an L1 sign
that flips between two renders straddling the target within rounding cannot make the two sides differ.
"""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from common import (assert_close_grad, assert_close_render, digest, np_, ours_stages, raster_grad_abs_sums, reference_stages,
                    to_dev)
from igs_b200 import bands, ops, pipeline, workloads
from oracle import quant as oquant

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

INT_KEYS = ("xys", "radii", "conics", "num_tiles_hit", "cum", "gaussian_ids_sorted", "tile_bins")
RASTER_GRADS = ("v_xy", "v_conic", "v_colors")
PROJECTION_GRADS = ("v_cov2d", "v_mean2d", "v_scale", "v_rot")


def l1_grad(image, target, ratio=1.0):
    """The image gradient of ratio * F.l1_loss(image, target): sign(image - target) * ratio / numel."""
    return (torch.sign(image - target) * (ratio / image.numel())).contiguous()


def assert_raster_grads(got, want, h, w, xys, conics, colors, v_output, pixel_topk, what=""):
    """got / want: v_xy, v_conic, v_colors of the same lists and image gradient"""
    sums = raster_grad_abs_sums(h, w, xys, conics, colors, v_output, pixel_topk)
    for key, a, b in zip(RASTER_GRADS, got, want):
        assert_close_grad(a, b, what=key + what, abs_sum=sums[key])


def assert_projection_backward(ours, d, h, w, ref_module):
    """The projection backward stage-wise: the reference's kernel on our v_xy, v_conic"""
    n = d["means"].shape[0]
    want = ref_module.project_gaussians_2d_scale_rot_backward(n, d["means"], d["scales"], d["rotations"], h, w, ours["radii"],
                                                              ours["conics"], ours["v_xy"], ours["v_conic"])
    for key, b in zip(PROJECTION_GRADS, want):
        assert_close_grad(ours[key], b, what=key)


def assert_stages_match(ours, ref, d, h, w, ref_module):
    for key in INT_KEYS:
        assert torch.equal(ours[key], ref[key]), key
    assert torch.equal(ours["pixel_topk"], ref["pixel_topk"]), "pixel_topk"
    assert_close_render(ours["image"], ref["image"], what="image")
    assert_raster_grads([ours[k] for k in RASTER_GRADS], [ref[k] for k in RASTER_GRADS], h, w, ours["xys"], ours["conics"], d["features"],
                        ours["v_output"], ours["pixel_topk"])
    assert_projection_backward(ours, d, h, w, ref_module)


def workload_on(device, name, image_index=0):
    wl = workloads.get_workload(name)
    inp = workloads.make_inputs(wl, image_index=image_index)
    return wl, inp, to_dev(inp, device)


@pytest.fixture(scope="module")
def cfg3(device):
    return workload_on(device, "cfg3_1080p")


@pytest.fixture(scope="module")
def cfg3_ours(cfg3):
    wl, _, d = cfg3
    return ours_stages(d, wl.height, wl.width)


def test_cfg3_every_stage_vs_reference(cfg3, cfg3_ours, ref_module):
    """1080p/20k: projection, prefix sum, binning and top-K lists bit-exact, render and every gradient within tolerance."""
    wl, _, d = cfg3
    ref = reference_stages(ref_module, d, wl.height, wl.width, v_output=cfg3_ours["v_output"])
    assert_stages_match(cfg3_ours, ref, d, wl.height, wl.width, ref_module)


def test_cfg3_half_capacity_vs_reference(cfg3, cfg3_ours, ref_module):
    """The fixed capacity of a graph-captured step, here half the intersections: the same slots dropped, the same lists."""
    wl, _, d = cfg3
    cap = cfg3_ours["num_intersects"] // 2
    ours = ours_stages(d, wl.height, wl.width, capacity=cap)
    ref = reference_stages(ref_module, d, wl.height, wl.width, capacity=cap, v_output=ours["v_output"])
    assert_stages_match(ours, ref, d, wl.height, wl.width, ref_module)


def test_cfg3_matches_committed_reference_digests(cfg3, cfg3_ours):
    """The committed fixture holds SHA-256 digests of the reference extension's outputs on this workload (made on a B200 by
    tests/golden/make_golden_ref.py): our integer outputs and projected floats hash the same, the image's first rows agree within
    tolerance. Needs no reference build at run time."""
    wl, inp, d = cfg3
    z = np.load(os.path.join(GOLDEN, "ref_cfg3_1080p.npz"))
    assert str(z["input_digest"]) == workloads.input_digest(inp)
    for key in ("radii", "num_tiles_hit", "cum", "gaussian_ids_sorted", "tile_bins", "pixel_topk", "xys", "conics"):
        assert digest(cfg3_ours[key]) == str(z[f"digest_{key}"]), key
    assert int(z["meta"][4]) == cfg3_ours["num_intersects"]
    assert_close_render(np_(cfg3_ours["image"])[:, :16, :512], z["image_crop"], what="image rows 0-15")
    half = ours_stages(d, wl.height, wl.width, capacity=cfg3_ours["num_intersects"] // 2)
    for key in ("gaussian_ids_sorted", "tile_bins", "pixel_topk"):
        assert digest(half[key]) == str(z[f"half_digest_{key}"]), "half capacity " + key


def fused_vs_reference(ours, d, h, w, ref_module):
    """The training step's fused kernel on our tile lists: its image equals the operator path's bit for bit, its image gradient is the L1
    gradient of that image, and its parameter gradients match the reference's backward kernel given that image gradient."""
    tb = ops.tile_grid(h, w)
    img, loss, v_xy, v_conic, v_colors, v_out = ops.raster_step_l1(tb, (w, h, 1), ours["gaussian_ids_sorted"], ours["tile_bins"],
                                                                   ours["xys"], ours["conics"], d["features"], d["target"],
                                                                   with_v_output=True)
    assert torch.equal(img, ours["image"])
    assert torch.equal(v_out, l1_grad(img, d["target"]))
    ref_img, ref_topk = ref_module.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ours["gaussian_ids_sorted"],
                                                                  ours["tile_bins"], ours["xys"], ours["conics"], d["features"])
    assert torch.equal(ref_topk, ours["pixel_topk"])
    ref_loss = F.l1_loss(ref_img, d["target"])
    assert abs(float(loss) - float(ref_loss)) <= 1e-5 * float(ref_loss)
    r_xy, r_conic, r_colors = ref_module.nd_rasterize_backward_topk_norm(h, w, 16, 16, ours["xys"], ours["conics"], d["features"], v_out,
                                                                         ref_topk)
    assert_raster_grads((v_xy, v_conic, v_colors), (r_xy, r_conic, r_colors), h, w, ours["xys"], ours["conics"], d["features"], v_out,
                        ref_topk, " (fused step)")


def test_cfg3_fused_step_vs_reference(cfg3, cfg3_ours, ref_module):
    wl, _, d = cfg3
    fused_vs_reference(cfg3_ours, d, wl.height, wl.width, ref_module)


def test_cfg3_pipeline_step_vs_reference(cfg3, cfg3_ours, ref_module):
    """The graph-replayed pipeline step the benchmark times (fused kernel): render, loss and parameter gradients against the reference's
    kernels run in model.py's order with the pipeline's own image gradient."""
    wl, _, d = cfg3
    h, w = wl.height, wl.width
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"])
    step.replay()
    step.replay()
    torch.cuda.synchronize()
    assert int(step.num_intersects.item()) == cfg3_ours["num_intersects"]
    v_out = l1_grad(step.image, d["target"])
    ref = reference_stages(ref_module, d, h, w, v_output=v_out)
    assert_close_render(step.image, ref["image"], what="image")
    assert abs(float(step.loss) - float(F.l1_loss(ref["image"], d["target"]))) <= 1e-5 * float(step.loss)
    assert_raster_grads([getattr(step, k) for k in RASTER_GRADS], [ref[k] for k in RASTER_GRADS], h, w, step.xys, step.conics,
                        d["features"], v_out, ref["pixel_topk"], " (pipeline)")
    assert_projection_backward({k: getattr(step, k) for k in ("radii", "conics", "v_xy", "v_conic") + PROJECTION_GRADS}, d, h, w,
                               ref_module)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_cfg4_bands_vs_reference(world, device, ref_module):
    """2160p/80k split into tile-row bands, each band's step run alone as one rank runs it (band-local binning and the fused kernel):
    the bands' tile lists are the reference's whole-image lists of those tiles, their rows its render, and the band gradients summed
    over the bands (what the all-reduce computes) its gradients."""
    wl, _, d = workload_on(device, "cfg4_2160p")
    h, w = wl.height, wl.width
    tiles_x, tiles_y, _ = wl.tile_bounds
    n = wl.num_gaussians
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ref_module.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum = torch.cumsum(hits, dim=0, dtype=torch.int32)
    total = int(cum[-1].item())
    ref_ids, ref_bins = ref_module.sort_intersects_by_tile(n, total, xys, radii, cum, tb)
    ref_img, ref_topk = ref_module.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ref_ids, ref_bins, xys, conics,
                                                                  d["features"])
    lengths = (ref_bins[:, 1] - ref_bins[:, 0]).to(torch.int64)
    starts = torch.cat([torch.zeros(1, dtype=torch.int64, device=device), torch.cumsum(lengths, 0)])
    weights = None
    if world == 8:  # the benchmark's balanced bands (tile-list entries per row plus a per-tile constant)
        weights = [r + 32.0 * tiles_x for r in bands.row_intersections(d["means"], d["scales"], d["rotations"], h, w)]
    image = torch.empty_like(ref_img)
    sums = {k: torch.zeros(n, m, device=device) for k, m in (("v_xy", 2), ("v_conic", 3), ("v_colors", wl.channels))}
    loss = 0.0
    for rank in range(world):
        r0, r1 = bands.band_rows(tiles_y, world, rank, weights)
        step = bands.BandStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], h, w, r0, r1)
        step.launch()
        torch.cuda.synchronize()
        t0, t1 = r0 * tiles_x, r1 * tiles_x
        band_lengths = (step.bins[: t1 - t0, 1] - step.bins[: t1 - t0, 0]).to(torch.int64)
        assert torch.equal(band_lengths, lengths[t0:t1]), f"band {rank}: list lengths"
        count = int(starts[t1] - starts[t0])
        assert torch.equal(step.ids[:count], ref_ids[int(starts[t0]):int(starts[t1])]), f"band {rank}: tile lists"
        assert torch.equal(step.xys, xys) and torch.equal(step.radii, radii) and torch.equal(step.conics, conics)
        image[:, 16 * r0:16 * r0 + step.band_h] = step.image
        for k in sums:
            sums[k] += getattr(step, k)
        loss += float(step.loss)
        step.release()
    assert_close_render(image, ref_img, what="assembled band renders")
    v_out = l1_grad(image, d["target"])
    r_xy, r_conic, r_colors = ref_module.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, d["features"], v_out, ref_topk)
    assert_raster_grads([sums[k] for k in RASTER_GRADS], (r_xy, r_conic, r_colors), h, w, xys, conics, d["features"], v_out, ref_topk,
                        f" summed over {world} bands")
    ref_loss = float(F.l1_loss(ref_img, d["target"]))
    assert abs(loss - ref_loss) <= 1e-5 * ref_loss


def test_cfg5_texture_image_vs_reference(device, ref_module):
    """One 2048x2048 image of the 9-channel texture stack, 50,000 Gaussians: the operator path (the reference's 9-channel backward)
    and the fused step kernel."""
    wl, _, d = workload_on(device, "cfg5_tex9", image_index=3)
    ours = ours_stages(d, wl.height, wl.width)
    ref = reference_stages(ref_module, d, wl.height, wl.width, v_output=ours["v_output"])
    assert_stages_match(ours, ref, d, wl.height, wl.width, ref_module)
    fused_vs_reference(ours, d, wl.height, wl.width, ref_module)


def test_cfg2_full_step_vs_reference(device, ref_module):
    """The 854x480 YUV step as model.py runs it with rate-distortion training: straight-through quantization of the parameters, features
    mapped to the loss space, render, L1 loss, rate term on the raw features and rotations. Ours is the graph-replayed pipeline step; the
    reference side composes the reference's own kernels (projection, binning, top-K forward and backward, projection backward, rate
    forward and backward) with the oracle's restatement of its quantization code on the GPU and ATen for the transform and the loss."""
    wl, inp, d = workload_on(device, "cfg2_480p_yuv")
    h, w, n = wl.height, wl.width, wl.num_gaussians
    z = np.load(os.path.join(GOLDEN, "py_cfg2_480p_yuv.npz"))
    model = workloads.RateModelTensors(z, device)
    q = workloads.quant_settings(wl, device)
    T = workloads.loss_transform_yuv().to(device)
    rate = dict(model=model, inv_rot_step=float(z["inv_rot_step"]), factor=float(z["factor"]))
    target = d["loss_target"]
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], target, quant=q, loss_transform=T, rate=rate)
    step.replay()
    step.replay()
    torch.cuda.synchronize()

    # the reference's quantization arithmetic (ATen on the GPU): symbols and straight-through values bit-exact
    (qm, qs, qr, qf), _ = oquant.quantize_ste(d["means"], d["scales"], d["rotations"], d["features"], q["pos_steps"], q["scale_step"],
                                              q["rot_step"], q["feat_steps"])
    for got, want, what in ((step.q_means, qm, "means"), (step.q_scales, qs, "scales"), (step.q_rot, qr, "rotations"),
                            (step.q_feat, qf, "features")):
        assert torch.equal(got, want), "quantized " + what
    feat_t = (qf @ T.T).contiguous()  # model.py:963-964
    assert_close_grad(step.feat_t, feat_t, rtol=1e-6, what="loss-space features")
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ref_module.project_gaussians_2d_scale_rot_forward(n, qm, qs, qr, h, w, tb)
    for got, want, what in ((step.xys, xys, "xys"), (step.radii, radii, "radii"), (step.conics, conics, "conics"), (step.hits, hits, "hits")):
        assert torch.equal(got, want), what
    cum = torch.cumsum(hits, dim=0, dtype=torch.int32)
    total = int(cum[-1].item())
    ids, bins = ref_module.sort_intersects_by_tile(n, total, xys, radii, cum, tb)
    assert torch.equal(step.ids[:total], ids) and torch.equal(step.bins, bins)
    img, topk = ref_module.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feat_t)
    assert_close_render(step.image, img, what="loss-space render")
    l1 = F.l1_loss(img, target)
    assert abs(float(step.loss) - float(l1)) <= 1e-5 * float(l1)
    v_out = l1_grad(step.image, target)
    v_xy, v_conic, v_colors = ref_module.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feat_t, v_out, topk)
    assert_raster_grads((step.v_xy, step.v_conic, step.v_colors), (v_xy, v_conic, v_colors), h, w, xys, conics, feat_t, v_out, topk)
    # the stages after the rasterizer, stage-wise from our raster gradients: the projection backward, the transform's backward (the
    # straight-through estimator passes gradients unchanged) and the rate term's gradients added
    _, v_mean2d, v_scale, v_rot = ref_module.project_gaussians_2d_scale_rot_backward(n, qm, qs, qr, h, w, radii, conics, step.v_xy,
                                                                                     step.v_conic)
    v_feat_render = step.v_colors @ T
    m = model
    r_loss, r_weight, r_own, r_rot = ref_module.rate_loss_forward(d["features"], d["rotations"], step.loss.detach().clone(), m.neighbors,
                                                                  m.weights, m.slope, list(m.color_refs), list(m.pred_channels),
                                                                  m.inv_steps, m.feat_coeffs, m.inv_rot, rate["inv_rot_step"], 1.0,
                                                                  rate["factor"])
    g_feat, g_rot = ref_module.rate_loss_backward(torch.ones((), device=device), r_weight, r_own, r_rot, m.offsets, m.sources,
                                                  m.source_weights)
    assert abs(float(step.rate_loss) - float(r_loss)) <= 1e-5 * abs(float(r_loss))
    assert_close_grad(step.v_mean2d, v_mean2d, what="means")
    assert_close_grad(step.v_scale, v_scale, what="scales")
    assert_close_grad(step.v_rot.view(-1) + step.rate_grad_rot, v_rot.view(-1) + g_rot.view(-1), what="rotations")
    assert_close_grad(step.v_feat, v_feat_render + g_feat, what="features")
