"""
Parity of the igs_b200 kernels, stage by stage, against
  (a) the CPU oracle (oracle/oracle.c): each stage is fed our previous stage's outputs so that float differences do not cascade;
      integers must match except at float near-ties that the test identifies (libm vs fast-math intrinsics), floats within tolerance;
  (b) the reference's own extension built from source (oracle/_ref), run on the same GPU: integers bit-exact, floats within tolerance.
"""
import math

import numpy as np
import pytest
import torch

from common import (assert_close_grad, assert_close_render, alpha_ties, make_case, np_, ours_stages, raster_grad_abs_sums,
                    reference_stages, to_dev)
from igs_b200 import ops
from oracle import cpu as orc

pytestmark = pytest.mark.gpu

CASES = {
    "ragged_120x88": dict(h=88, w=120, n=300, seed=11),
    "cfg1_256": dict(h=256, w=256, n=1000, seed=1001),
    "c1_70x50": dict(h=50, w=70, n=150, c=1, seed=12),
    "c9_80x64": dict(h=64, w=80, n=200, c=9, seed=13),
    "c12_40x48": dict(h=48, w=40, n=120, c=12, seed=14),
    "aniso_200x100": dict(h=100, w=200, n=600, max_anisotropy=8.0, log_scale_std=0.8, seed=15),
    "big_64x64": dict(h=64, w=64, n=400, log_scale_mean=math.log(20.0), log_scale_std=0.3, seed=16),
    "tiny_1x1": dict(h=1, w=1, n=5, log_scale_mean=math.log(1.0), seed=17),
}


def abs_sums(ours, dinp, wl):
    """The magnitude sums behind our v_xy, v_conic, v_colors (the CPU oracle over our lists and image gradient): two float sums of the
    same terms in different orders (atomics in the reference, warp and tile sums here) are held to them where the terms cancel."""
    return raster_grad_abs_sums(wl.height, wl.width, ours["xys"], ours["conics"], dinp["features"], ours["v_output"], ours["pixel_topk"])


def build_case(name, device):
    kw = dict(CASES[name])
    h, w = kw.pop("h"), kw.pop("w")
    wl, inp = make_case(h, w, **kw)
    return wl, inp, to_dev(inp, device)


@pytest.mark.parametrize("name", list(CASES))
def test_projection_vs_oracle(name, device):
    wl, inp, dinp = build_case(name, device)
    ours = ours_stages(dinp, wl.height, wl.width)
    xys, radii, conics, hits = orc.project_fwd(inp["means"], inp["scales"], inp["rotations"], wl.height, wl.width)
    valid = np_(ours["radii"]) > 0
    # centers are one IEEE multiply on both sides
    np.testing.assert_array_equal(np_(ours["xys"])[valid], xys[valid])
    # radii / tile counts: equal unless 3 sqrt(lambda) sits within float rounding of an integer (approximate vs IEEE sqrt)
    diff = np.nonzero((np_(ours["radii"]) != radii) | (np_(ours["num_tiles_hit"]) != hits))[0]
    assert len(diff) <= max(1, len(radii) // 1000), f"{len(diff)} Gaussians differ in radius/tiles"
    for g in diff:
        assert abs(int(np_(ours["radii"])[g]) - int(radii[g])) <= 1
    keep = np.ones(len(radii), bool)
    keep[diff] = False
    assert_close_grad(np_(ours["conics"])[keep], conics[keep], rtol=1e-4, what="conics")


@pytest.mark.parametrize("name", list(CASES))
def test_binning_vs_oracle(name, device):
    wl, inp, dinp = build_case(name, device)
    ours = ours_stages(dinp, wl.height, wl.width)
    ids, bins = orc.sort_intersects(len(inp["means"]), ours["capacity"], np_(ours["xys"]), np_(ours["radii"]), np_(ours["cum"]),
                                    wl.height, wl.width)
    np.testing.assert_array_equal(np_(ours["cum"]), orc.cumsum(np_(ours["num_tiles_hit"])))
    np.testing.assert_array_equal(np_(ours["gaussian_ids_sorted"]), ids)
    np.testing.assert_array_equal(np_(ours["tile_bins"]), bins)


@pytest.mark.parametrize("name", list(CASES))
def test_forward_vs_oracle(name, device):
    wl, inp, dinp = build_case(name, device)
    ours = ours_stages(dinp, wl.height, wl.width)
    if ours["capacity"] <= 0:
        pytest.skip("no intersections")
    img, topk = orc.raster_fwd(wl.height, wl.width, np_(ours["gaussian_ids_sorted"]), np_(ours["tile_bins"]), np_(ours["xys"]),
                               np_(ours["conics"]), inp["features"].numpy())
    mism = np.argwhere(np.any(np_(ours["pixel_topk"]) != topk, axis=-1))
    if len(mism):
        ties = alpha_ties(ours["xys"], ours["conics"], ours["gaussian_ids_sorted"], ours["tile_bins"], ops.tile_grid(wl.height, wl.width)[0],
                          [tuple(p) for p in mism])
        assert ties.all(), f"{int((~ties).sum())} pixels differ from the oracle without a near-tie of alpha"
        assert len(mism) <= max(2, topk.shape[0] * topk.shape[1] // 2000), f"{len(mism)} pixels differ at near-ties"
    same = np.all(np_(ours["pixel_topk"]) == topk, axis=-1)
    assert_close_render(np_(ours["image"])[:, same], img[:, same], what="image")


@pytest.mark.parametrize("name", list(CASES))
def test_backward_vs_oracle(name, device):
    wl, inp, dinp = build_case(name, device)
    ours = ours_stages(dinp, wl.height, wl.width)
    if ours["capacity"] <= 0:
        pytest.skip("no intersections")
    v_xy, v_conic, v_colors = orc.raster_bwd(wl.height, wl.width, np_(ours["xys"]), np_(ours["conics"]), inp["features"].numpy(),
                                             np_(ours["v_output"]), np_(ours["pixel_topk"]))
    sums = abs_sums(ours, dinp, wl)
    assert_close_grad(ours["v_xy"], v_xy, what="v_xy", abs_sum=sums["v_xy"])
    assert_close_grad(ours["v_conic"], v_conic, what="v_conic", abs_sum=sums["v_conic"])
    assert_close_grad(ours["v_colors"], v_colors, what="v_colors", abs_sum=sums["v_colors"])
    v_cov2d, v_mean2d, v_scale, v_rot = orc.project_bwd(inp["scales"].numpy(), inp["rotations"].numpy(), wl.height, wl.width,
                                                        np_(ours["radii"]), np_(ours["conics"]), np_(ours["v_xy"]), np_(ours["v_conic"]))
    assert_close_grad(ours["v_cov2d"], v_cov2d, what="v_cov2d")
    assert_close_grad(ours["v_mean2d"], v_mean2d, what="v_mean2d")
    assert_close_grad(ours["v_scale"], v_scale, what="v_scale")
    assert_close_grad(ours["v_rot"], v_rot, what="v_rot")


@pytest.mark.parametrize("name", list(CASES))
def test_all_stages_vs_reference(name, device, ref_module):
    wl, inp, dinp = build_case(name, device)
    ours = ours_stages(dinp, wl.height, wl.width)
    ref = reference_stages(ref_module, dinp, wl.height, wl.width, v_output=ours.get("v_output"))
    for key in ("xys", "radii", "conics", "num_tiles_hit", "cum", "gaussian_ids_sorted", "tile_bins"):
        np.testing.assert_array_equal(np_(ours[key]), np_(ref[key]), err_msg=key)
    if ours["capacity"] <= 0:
        return
    np.testing.assert_array_equal(np_(ours["pixel_topk"]), np_(ref["pixel_topk"]), err_msg="pixel_topk")
    assert_close_render(ours["image"], ref["image"], what="image")
    sums = abs_sums(ours, dinp, wl)
    for key in ("v_xy", "v_conic", "v_colors", "v_cov2d", "v_mean2d", "v_scale", "v_rot"):
        assert_close_grad(ours[key], ref[key], what=key, abs_sum=sums.get(key))
    # the training step's fused kernel (forward, L1 loss, backward in one) against the reference's kernels with the same loss gradient
    tb = ops.tile_grid(wl.height, wl.width)
    f_img, _, f_xy, f_conic, f_colors = ops.raster_step_l1(tb, (wl.width, wl.height, 1), ours["gaussian_ids_sorted"], ours["tile_bins"],
                                                           ours["xys"], ours["conics"], dinp["features"], dinp["target"])
    assert torch.equal(f_img, ours["image"])
    for key, got in (("v_xy", f_xy), ("v_conic", f_conic), ("v_colors", f_colors)):
        assert_close_grad(got, ref[key], what=key + " (fused step)", abs_sum=sums[key])


@pytest.mark.parametrize("name", ["ragged_120x88", "cfg1_256", "c9_80x64", "c12_40x48", "big_64x64"])
def test_tile_list_path_matches_pixel_path(name, device):
    """The autograd path's 16-bit tile lists hold exactly pixel_topk, and its backward agrees with the [H, W, 10] one."""
    wl, inp, dinp = build_case(name, device)
    h, w = wl.height, wl.width
    ours = ours_stages(dinp, h, w)
    tb = ops.tile_grid(h, w)
    img, tile_topk = ops.nd_rasterize_forward_topk_norm_tiles(tb, (w, h, 1), min(len(inp["means"]), ours["capacity"]),
                                                              ours["gaussian_ids_sorted"], ours["tile_bins"], ours["xys"],
                                                              ours["conics"], dinp["features"])
    assert torch.equal(img, ours["image"])
    # decode: tile t, slot k, lane -> pixel; position -> Gaussian ID
    pos = np_(tile_topk).astype(np.int64) & 0xFFFF
    ids, bins = np_(ours["gaussian_ids_sorted"]), np_(ours["tile_bins"])
    topk = np_(ours["pixel_topk"])
    for t in range(tb[0] * tb[1]):
        ty, tx = divmod(t, tb[0])
        for lane_id in range(256):
            warp, lane = divmod(lane_id, 32)
            ly, lx = (warp >> 1) * 4 + (lane >> 3), (warp & 1) * 8 + (lane & 7)
            i, j = ty * 16 + ly, tx * 16 + lx
            if i >= h or j >= w:
                continue
            p = pos[t, :, lane_id]
            dec = np.where(p == 0xFFFF, -1, ids[np.minimum(bins[t, 0] + p, len(ids) - 1)])
            np.testing.assert_array_equal(dec, topk[i, j])
    v = ops.nd_rasterize_backward_topk_norm_tiles(h, w, ours["gaussian_ids_sorted"], ours["tile_bins"], ours["xys"], ours["conics"],
                                                  dinp["features"], ours["v_output"], tile_topk)
    # two float sums of the same terms in different orders (per-entry sums over a tile here, a warp's union walk there, atomics
    # across CTAs in both): near-cancelling values are held to the sum of their terms' magnitudes
    sums = raster_grad_abs_sums(h, w, ours["xys"], ours["conics"], dinp["features"], ours["v_output"], ours["pixel_topk"])
    for a, b, nm in zip(v, (ours["v_xy"], ours["v_conic"], ours["v_colors"]), ("v_xy", "v_conic", "v_colors")):
        assert_close_grad(a, b, what=nm, abs_sum=sums[nm])


def test_tile_lists_beyond_16_bit_positions(device, ref_module):
    """Tile lists of 70,000 entries (more than 16-bit positions address): the forward pass leaves those tiles' 16-bit lists empty and the
    backward pass selects them again. Top-K lists equal the reference kernels' bit for bit (with 70,000 candidates nearly every pixel has
    near-ties in alpha, so the IEEE-exp oracle is not the pin for the selection); gradients agree with the [H, W, 10] path and with the
    reference kernels' backward over the same lists (the quotient rule cancels heavily here: ten weights near 1 per pixel)."""
    wl, inp = make_case(40, 24, 70000, log_scale_mean=math.log(40.0), log_scale_std=0.1, seed=23)
    dinp = to_dev(inp, device)
    h, w = wl.height, wl.width
    ours = ours_stages(dinp, h, w)
    bins = np_(ours["tile_bins"])
    assert (bins[:, 1] - bins[:, 0]).min() >= 65535
    ref = reference_stages(ref_module, dinp, h, w, v_output=ours["v_output"], xys=ours["xys"], radii=ours["radii"], conics=ours["conics"],
                           hits=ours["num_tiles_hit"])
    np.testing.assert_array_equal(np_(ours["gaussian_ids_sorted"]), np_(ref["gaussian_ids_sorted"]))
    np.testing.assert_array_equal(np_(ours["pixel_topk"]), np_(ref["pixel_topk"]))
    assert_close_render(ours["image"], ref["image"], what="image")
    tb = ops.tile_grid(h, w)
    img, tile_topk = ops.nd_rasterize_forward_topk_norm_tiles(tb, (w, h, 1), ours["capacity"], ours["gaussian_ids_sorted"],
                                                              ours["tile_bins"], ours["xys"], ours["conics"], dinp["features"])
    assert torch.equal(img, ours["image"])
    assert bool((tile_topk == -1).all())  # 0xFFFF everywhere: re-selected in the backward pass
    v = ops.nd_rasterize_backward_topk_norm_tiles(h, w, ours["gaussian_ids_sorted"], ours["tile_bins"], ours["xys"], ours["conics"],
                                                  dinp["features"], ours["v_output"], tile_topk)
    sums = abs_sums(ours, dinp, wl)
    for nm in ("v_xy", "v_conic", "v_colors"):
        a = v[("v_xy", "v_conic", "v_colors").index(nm)]
        assert_close_grad(a, ours[nm], what=nm, abs_sum=sums[nm])
        assert_close_grad(a, ref[nm], what=nm + " vs reference", abs_sum=sums[nm])
    # the fused step kernel keeps 32-bit list positions in shared memory: the same render and gradients without a second selection
    f_img, _, f_xy, f_conic, f_colors = ops.raster_step_l1(tb, (w, h, 1), ours["gaussian_ids_sorted"], ours["tile_bins"], ours["xys"],
                                                           ours["conics"], dinp["features"], dinp["target"])
    assert torch.equal(f_img, ours["image"])
    for nm, a in (("v_xy", f_xy), ("v_conic", f_conic), ("v_colors", f_colors)):
        assert_close_grad(a, ref[nm], what=nm + " (fused step) vs reference", abs_sum=sums[nm])


def test_capacity_drops_like_reference(device):
    """Fixed capacity below the intersection count: the excess (in Gaussian-major order) is dropped exactly as the reference does."""
    wl, inp, dinp = build_case("cfg1_256", device)
    full = ours_stages(dinp, wl.height, wl.width)
    for cap in (full["num_intersects"] // 2, 1, full["num_intersects"] + 77):
        ours = ours_stages(dinp, wl.height, wl.width, capacity=cap)
        ids, bins = orc.sort_intersects(len(inp["means"]), cap, np_(ours["xys"]), np_(ours["radii"]), np_(ours["cum"]), wl.height, wl.width)
        np.testing.assert_array_equal(np_(ours["gaussian_ids_sorted"]), ids)
        np.testing.assert_array_equal(np_(ours["tile_bins"]), bins)


def test_capacity_drops_vs_reference(device, ref_module):
    wl, inp, dinp = build_case("cfg1_256", device)
    full = ours_stages(dinp, wl.height, wl.width)
    for cap in (full["num_intersects"] // 3, full["num_intersects"] + 5):
        ours = ours_stages(dinp, wl.height, wl.width, capacity=cap)
        ref = reference_stages(ref_module, dinp, wl.height, wl.width, capacity=cap)
        for key in ("gaussian_ids_sorted", "tile_bins", "pixel_topk"):
            np.testing.assert_array_equal(np_(ours[key]), np_(ref[key]), err_msg=key)


def test_no_intersections(device):
    """Gaussians entirely off-screen: no tiles hit, empty binning, zero image and gradients through the autograd path."""
    wl, inp = make_case(64, 48, 50, seed=21)
    inp["means"] = inp["means"] + 5.0
    dinp = to_dev(inp, device)
    tb = ops.tile_grid(64, 48)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(50, dinp["means"], dinp["scales"], dinp["rotations"], 64, 48, tb)
    assert int(hits.sum()) == 0
    from igs_b200 import autograd as ag

    means = dinp["means"].clone().requires_grad_(True)
    feats = dinp["features"].clone().requires_grad_(True)
    xys, radii, conics, hits = ag.project_gaussians_2d_scale_rot(means, dinp["scales"], dinp["rotations"], 64, 48, tb)
    img = ag.rasterize_gaussians_sum_topk(xys, radii, conics, hits, feats, 64, 48)
    assert img.shape == (64, 48, 3) and float(img.abs().sum()) == 0.0
    img.sum().backward()
    assert float(feats.grad.abs().sum()) == 0.0
    ids, bins = ops.sort_intersects_by_tile(50, 0, xys.detach(), radii, ops.cumulative_intersects(hits)[0], tb)
    assert ids.numel() == 0 and int(bins.abs().sum()) == 0


def test_degenerate_scales(device):
    """Zero scales give a zero determinant: radius 0, no tiles, zero conic, like the reference's early return (foward2d.cu:42-46). With
    one zero scale the determinant is a rounding residue, whose sign and size follow the float operations; that case must match the
    reference bit for bit instead."""
    wl, inp = make_case(32, 32, 20, seed=22)
    inp["scales"][3] = 0.0
    inp["scales"][7, 1] = 0.0
    dinp = to_dev(inp, device)
    tb = ops.tile_grid(32, 32)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(20, dinp["means"], dinp["scales"], dinp["rotations"], 32, 32, tb)
    oxys, oradii, oconics, ohits = orc.project_fwd(inp["means"], inp["scales"], inp["rotations"], 32, 32)
    assert int(radii[3]) == 0 == oradii[3] and int(hits[3]) == 0
    assert float(conics[3].abs().sum()) == 0.0 and float(xys[3].abs().sum()) == 0.0


def test_degenerate_scales_vs_reference(device, ref_module):
    wl, inp = make_case(32, 32, 20, seed=22)
    inp["scales"][3] = 0.0
    inp["scales"][7, 1] = 0.0
    inp["scales"][9, 0] = 1e-20
    dinp = to_dev(inp, device)
    tb = ops.tile_grid(32, 32)
    ours = ops.project_gaussians_2d_scale_rot_forward(20, dinp["means"], dinp["scales"], dinp["rotations"], 32, 32, tb)
    ref = ref_module.project_gaussians_2d_scale_rot_forward(20, dinp["means"], dinp["scales"], dinp["rotations"], 32, 32, tb)
    for a, b in zip(ours, ref):
        np.testing.assert_array_equal(np_(a), np_(b))


def test_invalid_arguments_raise(device):
    wl, inp, dinp = build_case("ragged_120x88", device)
    tb = ops.tile_grid(88, 120)
    with pytest.raises(RuntimeError, match="contiguous"):
        ops.project_gaussians_2d_scale_rot_forward(300, dinp["means"].t().contiguous().t(), dinp["scales"], dinp["rotations"], 88, 120, tb)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.project_gaussians_2d_scale_rot_forward(300, inp["means"], dinp["scales"], dinp["rotations"], 88, 120, tb)
    feats13 = torch.zeros(300, 13, device=device)
    with pytest.raises(RuntimeError, match="MAX_CHANNELS"):
        ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (120, 88, 1), torch.zeros(1, dtype=torch.int32, device=device),
                                           torch.zeros(tb[0] * tb[1], 2, dtype=torch.int32, device=device), dinp["means"],
                                           torch.zeros(300, 3, device=device), feats13)
    with pytest.raises(ValueError):
        ops.nd_rasterize_forward_topk_norm((1, 1, 1), (16, 16, 1), (120, 88, 1), None, None, None, None, None)
