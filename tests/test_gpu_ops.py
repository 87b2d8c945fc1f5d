"""
GPU parity of the training-step operators around the rasterizer: the fused straight-through quantizer (symbols bit-exact against the
reference's quantization code, run here by ATen on the GPU and by the reference itself on the CPU for the fixtures), the rate term
(against the reference's rate_bits and its own CUDA kernels), the fused L1 loss, the leave-one-out kernel, the autograd / drop-in gsplat
path end to end, and the graph-captured pipeline.
"""
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from common import assert_close_grad, assert_close_render, make_case, np_, ours_stages, to_dev
from igs_b200 import autograd as ag
from igs_b200 import ops, pipeline, workloads
from oracle import cpu as orc
from oracle import quant as oquant

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
PY_CASES = ["cfg2_480p_yuv", "rgb_subgreen_320x200"]


def py_fixture(name):
    return dict(np.load(os.path.join(GOLDEN, f"py_{name}.npz")))


def py_inputs(name):
    wl = workloads.get_workload(name) if name in workloads.CONFIGS else workloads.custom_workload(200, 320, 800, 3, math.log(2.5), 0.5, 6.0,
                                                                                                    seed=31)
    return wl, workloads.make_inputs(wl)


@pytest.mark.parametrize("numel_shape", [(3, 37, 53), (3, 64, 64), (9, 16, 1)])
def test_l1_loss_matches_torch(numel_shape, device):
    g = torch.Generator().manual_seed(3)
    img = torch.rand(numel_shape, generator=g).to(device)
    tgt = torch.rand(numel_shape, generator=g).to(device)
    tgt.view(-1)[::7] = img.view(-1)[::7]  # exact ties: zero gradient
    loss, grad = ops.l1_loss_and_grad(img, tgt, ratio=0.75)
    x = img.clone().requires_grad_(True)
    ref = 0.75 * F.l1_loss(x, tgt)
    ref.backward()
    assert abs(float(loss) - float(ref)) <= 1e-6 * abs(float(ref))
    torch.testing.assert_close(grad, x.grad, rtol=0, atol=0)
    loss2, _ = ops.l1_loss_and_grad(img, tgt, ratio=0.75)  # the workspace ticket resets: repeatable, deterministic
    assert float(loss2) == float(loss)


@pytest.mark.parametrize("shape,ratio", [((3, 37, 53), 1.0), ((3, 64, 64), 0.75), ((9, 16, 1), 1.0)])
def test_l1_loss_with_signs_matches_torch_autograd(shape, ratio, device):
    """igs_b200.autograd.l1_loss (signs kept, gradient formed in the backward pass) against model.py's ratio * F.l1_loss: the gradient
    bit for bit, the loss within summation order; and model.py's F.l1_loss routed to it by install_l1()."""
    import sys
    import types

    g = torch.Generator().manual_seed(5)
    img = torch.rand(shape, generator=g).to(device)
    tgt = torch.rand(shape, generator=g).to(device)
    tgt.view(-1)[::5] = img.view(-1)[::5]  # exact ties: zero gradient
    x, y = img.clone().requires_grad_(True), img.clone().requires_grad_(True)
    ref = ratio * F.l1_loss(x, tgt)
    ref.backward()
    mine = ratio * ag.l1_loss(y, tgt)
    mine.backward()
    assert abs(float(mine) - float(ref)) <= 1e-6 * abs(float(ref))
    torch.testing.assert_close(y.grad, x.grad, rtol=0, atol=0)

    fake = types.ModuleType("igs_fake_model")
    fake.F = F
    sys.modules["igs_fake_model"] = fake
    try:
        replaced = ag.install_l1("igs_fake_model")
        assert fake.F is not F and fake.F.relu is F.relu
        z = img.clone().requires_grad_(True)
        routed = ratio * fake.F.l1_loss(z, tgt)
        routed.backward()
        assert float(routed) == float(mine)
        torch.testing.assert_close(z.grad, x.grad, rtol=0, atol=0)
        ag.restore(replaced)
        assert fake.F is F
    finally:
        del sys.modules["igs_fake_model"]


@pytest.mark.parametrize("case", [dict(h=88, w=120, n=300, seed=11), dict(h=64, w=80, n=200, c=9, seed=13), dict(h=50, w=70, n=150, c=1, seed=12)])
def test_forward_with_fused_l1_matches_separate_loss(case, device):
    """The forward kernel's fused L1 loss: render and lists identical to the plain forward, gradient identical to the L1 kernel's (and to
    torch's), loss within float summation order of torch's, repeatable."""
    kw = dict(case)
    h, w = kw.pop("h"), kw.pop("w")
    wl, inp = make_case(h, w, **kw)
    d = to_dev(inp, device)
    ours = ours_stages(d, h, w)
    tb = ops.tile_grid(h, w)
    bound = min(len(inp["means"]), ours["capacity"])
    args = (tb, (w, h, 1), bound, ours["gaussian_ids_sorted"], ours["tile_bins"], ours["xys"], ours["conics"], d["features"])
    img, topk = ops.nd_rasterize_forward_topk_norm_tiles(*args)
    img2, topk2, loss, v_out = ops.nd_rasterize_forward_topk_norm_tiles_l1(*args, d["target"], ratio=0.8)
    assert torch.equal(img, img2) and torch.equal(topk, topk2)
    loss_ref, grad_ref = ops.l1_loss_and_grad(img, d["target"], ratio=0.8)
    torch.testing.assert_close(v_out, grad_ref, rtol=0, atol=0)
    x = img.clone().requires_grad_(True)
    ref = 0.8 * F.l1_loss(x, d["target"])
    ref.backward()
    torch.testing.assert_close(v_out, x.grad, rtol=0, atol=0)
    assert abs(float(loss) - float(ref)) <= 2e-6 * abs(float(ref))
    _, _, loss2, _ = ops.nd_rasterize_forward_topk_norm_tiles_l1(*args, d["target"], ratio=0.8)
    assert float(loss2) == float(loss)


@pytest.mark.parametrize("name", ["weights_ragged_120x88", "weights_big_64x64", "weights_cfg1_256"])
def test_feature_weights_vs_reference(name, device):
    """igs_feature_weights against the reference's feature_weights over _iter_topk_weights: bit-identical int64 fixed-point sums to its
    code run by ATen on the GPU (oracle/weights.py, the reference's operations), and the reference's own CPU results (fixture) within the
    float32 exp differences of the two machines."""
    from oracle import weights as ow

    z = py_fixture(name)
    h, w, n = (int(v) for v in z["meta"])
    xys, conics, topk = (torch.from_numpy(z[k]).to(device) for k in ("xys", "conics", "pixel_topk"))
    fixed = ops.topk_feature_weights_fixed(h, w, xys, conics, topk)
    ref = ow.feature_weights_fixed(ow.iter_topk_weights(xys, conics, topk, h, w), n, 1e-4, device)
    assert torch.equal(fixed, ref)
    got = fixed.double() / 2.0 ** 40
    np.testing.assert_allclose(got.cpu().numpy(), z["weights"], rtol=1e-6, atol=1e-9)
    torch.testing.assert_close(ops.topk_feature_weights(h, w, xys, conics, topk), got, rtol=0, atol=0)


def test_feature_weights_full_size_vs_aten(device):
    """At 1080p/20k: the int64 fixed-point sums equal the reference's ATen operations run on the GPU (oracle/weights.py)."""
    from oracle import weights as ow

    wl = workloads.get_workload("cfg3_1080p")
    d = to_dev(workloads.make_inputs(wl), device)
    ours = ours_stages(d, wl.height, wl.width)
    fixed = ops.topk_feature_weights_fixed(wl.height, wl.width, ours["xys"], ours["conics"], ours["pixel_topk"])
    ref = ow.feature_weights_fixed(ow.iter_topk_weights(ours["xys"], ours["conics"], ours["pixel_topk"], wl.height, wl.width),
                                   wl.num_gaussians, 1e-4, device)
    assert torch.equal(fixed, ref)


@pytest.mark.parametrize("name", PY_CASES)
def test_quantize_ste_symbols_bit_exact(name, device):
    z = py_fixture(name)
    wl, inp = py_inputs(name)
    d = to_dev(inp, device)
    pos_steps = torch.from_numpy(z["steps_xy"]).to(device)
    feat_steps = torch.from_numpy(z["feat_steps"]).to(device)
    scale = d["scales"].abs()
    (oxy, osc, orot, ofeat), _, sym = ops.quantize_ste_forward(d["means"], scale, d["rotations"], d["features"], pos_steps,
                                                               float(z["scale_step"]), float(z["rot_step"]), feat_steps, with_symbols=True)
    # ATen on the GPU running the reference's quantization arithmetic: bit-exact
    values, ref_sym = oquant.quantize_ste(d["means"], scale, d["rotations"], d["features"], pos_steps, float(z["scale_step"]),
                                          float(z["rot_step"]), feat_steps)
    for a, b in zip(sym, ref_sym):
        assert torch.equal(a, b)
    for a, b in zip((oxy, osc, orot, ofeat), values):
        assert torch.equal(a, b)
    # the reference's own code on the CPU (the fixture): equal except where log2 of a scale lands within rounding of a half step
    for a, key in zip(sym, ("q_xy", "q_scale", "q_rot", "q_feat")):
        diff = np_(a) != z[key]
        assert diff.sum() <= 2, f"{key}: {int(diff.sum())} symbols differ from the CPU reference"


def test_quantize_ste_autograd_passes_gradients(device):
    wl, inp = make_case(32, 32, 50, seed=41)
    d = to_dev(inp, device)
    xs = [t.clone().requires_grad_(True) for t in (d["means"], d["scales"], d["rotations"], d["features"])]
    out = ag.quantize_ste(*xs, torch.tensor([0.004, 0.004], device=device), 0.03125, 0.0123, torch.full((3,), 1 / 64, device=device))
    sum(o.sum() * (i + 1) for i, o in enumerate(out)).backward()
    for i, x in enumerate(xs):
        assert torch.equal(x.grad, torch.full_like(x, float(i + 1)))


class _Model:
    """The fields of compress.rate.RateModel that the rate operators read."""

    def __init__(self, z, device):
        t = lambda k, dt=torch.float32: torch.from_numpy(z[k]).to(device=device, dtype=dt).contiguous()  # noqa: E731
        self.neighbors = t("neighbors", torch.int32)
        self.weights, self.slope, self.inv_steps, self.feat_coeffs, self.inv_rot = (t("weights"), t("slope"), t("inv_steps"),
                                                                                    t("feat_coeffs"), t("inv_rot"))
        self.offsets, self.sources, self.source_weights = t("offsets", torch.int32), t("sources", torch.int32), t("source_weights")
        self.color_refs = tuple(int(v) for v in z["color_refs"])
        self.pred_channels = tuple(int(v) for v in z["pred_channels"])


@pytest.mark.parametrize("name", PY_CASES)
def test_rate_loss_matches_reference_python(name, device):
    z = py_fixture(name)
    model = _Model(z, device)
    feat = torch.from_numpy(z["out_feat"]).to(device).requires_grad_(True)
    rot = torch.from_numpy(z["out_rot"]).to(device).requires_grad_(True)
    l1 = torch.tensor(float(z["l1"]), device=device)
    loss = ag.rate_loss(feat, rot, l1, model, float(z["inv_rot_step"]), float(z["l1_ratio"]), float(z["factor"]))
    loss.backward()
    assert abs(float(loss) - float(z["loss"])) <= 1e-5 * abs(float(z["loss"]))
    assert_close_grad(feat.grad, z["grad_feat"], what="grad_feat")
    assert_close_grad(rot.grad, z["grad_rot"], what="grad_rot")


@pytest.mark.parametrize("name", PY_CASES)
def test_rate_loss_matches_reference_kernels(name, device, ref_module):
    z = py_fixture(name)
    m = _Model(z, device)
    feat = torch.from_numpy(z["out_feat"]).to(device)
    rot = torch.from_numpy(z["out_rot"]).to(device)
    l1 = torch.tensor(float(z["l1"]), device=device)
    args = (feat, rot, l1, m.neighbors, m.weights, m.slope, list(m.color_refs), list(m.pred_channels), m.inv_steps, m.feat_coeffs,
            m.inv_rot, float(z["inv_rot_step"]), float(z["l1_ratio"]), float(z["factor"]))
    ours = ops.rate_loss_forward(*args)
    ref = ref_module.rate_loss_forward(*args)
    assert abs(float(ours[0]) - float(ref[0])) <= 1e-5 * abs(float(ref[0]))
    assert float(ours[1]) == float(ref[1])
    for a, b, what in zip(ours[2:], ref[2:], ("own_grad", "rot_grad")):
        assert_close_grad(a, b, what=what)
    g = torch.tensor(1.5, device=device)
    bo = ops.rate_loss_backward(g, ours[1], ours[2], ours[3], m.offsets, m.sources, m.source_weights)
    br = ref_module.rate_loss_backward(g, ref[1], ref[2], ref[3], m.offsets, m.sources, m.source_weights)
    for a, b, what in zip(bo, br, ("grad_feat", "grad_rot")):
        assert_close_grad(a, b, what=what)


@pytest.mark.parametrize("case", [dict(h=88, w=120, n=300, seed=11), dict(h=64, w=80, n=200, c=9, seed=13)])
def test_loo_matches_oracle(case, device):
    case = dict(case)
    h, w = case.pop("h"), case.pop("w")
    wl, inp = make_case(h, w, **case)
    d = to_dev(inp, device)
    ours = ours_stages(d, h, w)
    for squared in (False, True):
        got = ops.topk_norm_loo_loss_increase(h, w, ours["xys"], ours["conics"], d["features"], ours["pixel_topk"], d["target"], squared, 1e-4)
        want = orc.loo_loss_increase(h, w, np_(ours["xys"]), np_(ours["conics"]), inp["features"].numpy(), np_(ours["pixel_topk"]),
                                     inp["target"].numpy(), squared, 1e-4)
        assert_close_grad(got, want, rtol=1e-3, floor=1e-2, what=f"loo squared={squared}")


def test_loo_matches_reference(device, ref_module):
    wl, inp = make_case(88, 120, 300, seed=11)
    d = to_dev(inp, device)
    ours = ours_stages(d, 88, 120)
    for squared in (False, True):
        got = ops.topk_norm_loo_loss_increase(88, 120, ours["xys"], ours["conics"], d["features"], ours["pixel_topk"], d["target"], squared,
                                              1e-4)
        want = ref_module.topk_norm_loo_loss_increase(88, 120, ours["xys"], ours["conics"], d["features"], ours["pixel_topk"], d["target"],
                                                      squared, 1e-4)
        assert_close_grad(got, want, rtol=1e-3, floor=1e-2, what=f"loo squared={squared}")


@pytest.mark.parametrize("capacity", [None, "x2"])
def test_gsplat_shim_end_to_end(capacity, device):
    """model.forward's calls through the drop-in gsplat package, then F.l1_loss and backward: gradients of means, scales, rotations and
    features against the oracle's full step."""
    import gsplat

    wl, inp = make_case(96, 136, 500, seed=51)
    h, w = wl.height, wl.width
    d = to_dev(inp, device)
    params = [d[k].clone().requires_grad_(True) for k in ("means", "scales", "rotations", "features")]
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = gsplat.project_gaussians_2d_scale_rot(*params[:3], h, w, tb)
    cap = None if capacity is None else 2 * int(hits.sum())
    img = gsplat.rasterize_gaussians_sum(xys, radii, conics, hits, params[3], h, w, 16, 16, topk_norm=True, capacity=cap)
    assert img.shape == (h, w, 3)
    img_chw = img.view(-1, h, w, 3).permute(0, 3, 1, 2).contiguous().squeeze(0)  # model.py:975
    loss = F.l1_loss(img_chw, d["target"])
    loss.backward()
    r = orc.train_step(*[inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")], h, w)
    assert_close_render(img_chw, r["image"], rtol=3e-5, what="image")
    assert abs(float(loss) - r["loss"]) <= 1e-5 * r["loss"]
    # end to end the L1 sign can flip where the renders straddle the target within rounding; few pixels, small effect
    for p, key in zip(params, ("v_mean2d", "v_scale", "v_rot", "v_colors")):
        assert_close_grad(p.grad, r[key].reshape(p.shape), rtol=2e-3, what=key)


def test_pipeline_graph_matches_autograd(device):
    """The preallocated, graph-captured step computes what the autograd operators compute."""
    wl, inp = make_case(120, 200, 800, seed=61)
    d = to_dev(inp, device)
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"])
    step.replay()
    step.replay()
    torch.cuda.synchronize()
    params = [d[k].clone().requires_grad_(True) for k in ("means", "scales", "rotations", "features")]
    h, w = wl.height, wl.width
    xys, radii, conics, hits = ag.project_gaussians_2d_scale_rot(*params[:3], h, w, ops.tile_grid(h, w))
    img = ag.rasterize_gaussians_sum_topk(xys, radii, conics, hits, params[3], h, w, capacity=step.capacity)
    loss = ag.l1_loss(img.permute(2, 0, 1), d["target"])
    loss.backward()
    assert torch.equal(step.image, img.permute(2, 0, 1).detach())
    # the step's loss is summed per tile inside the forward kernel, the autograd one by the separate L1 kernel: summation order only
    assert abs(float(step.loss) - float(loss)) <= 2e-6 * float(loss)
    for p, mine in zip(params, (step.v_mean2d, step.v_scale, step.v_rot, step.v_colors)):
        assert_close_grad(mine, p.grad.reshape(mine.shape), what="pipeline grad")
    assert int(step.num_intersects.item()) <= step.capacity


def test_pipeline_rate_step_matches_autograd(device):
    """The 480p YUV step (quantizer, loss-space transform, L1, rate term), graph-captured, against the same step composed from the
    autograd operators and ATen."""
    z = py_fixture("cfg2_480p_yuv")
    wl = workloads.get_workload("cfg2_480p_yuv")
    inp = workloads.make_inputs(wl)
    d = to_dev(inp, device)
    model = workloads.RateModelTensors(z, device)
    q = workloads.quant_settings(wl, device)
    T = workloads.loss_transform_yuv().to(device)
    rate = dict(model=model, inv_rot_step=float(z["inv_rot_step"]), factor=float(z["factor"]))
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["loss_target"], quant=q, loss_transform=T,
                               rate=rate)
    step.replay()
    torch.cuda.synchronize()
    raw = [d[k].clone().requires_grad_(True) for k in ("means", "scales", "rotations", "features")]
    m, s_, r, f = ag.quantize_ste(*raw, q["pos_steps"], q["scale_step"], q["rot_step"], q["feat_steps"])
    ft = f @ T.T
    h, w = wl.height, wl.width
    xys, radii, conics, hits = ag.project_gaussians_2d_scale_rot(m, s_, r, h, w, ops.tile_grid(h, w))
    img = ag.rasterize_gaussians_sum_topk(xys, radii, conics, hits, ft, h, w, capacity=step.capacity)
    l1 = ag.l1_loss(img.permute(2, 0, 1), d["loss_target"])
    total = l1 + ag.rate_loss(raw[3], raw[2], l1, model, rate["inv_rot_step"], 1.0, rate["factor"])
    total.backward()
    assert abs(float(step.loss) - float(l1)) <= 2e-6 * float(l1)
    assert abs(float(step.rate_loss) - float(total - l1)) <= 1e-5 * abs(float(total - l1))
    assert_close_grad(step.v_mean2d, raw[0].grad, what="means")
    assert_close_grad(step.v_scale, raw[1].grad, what="scales")
    assert_close_grad(step.v_rot.view(-1) + step.rate_grad_rot, raw[2].grad.view(-1), what="rotations")
    assert_close_grad(step.v_feat, raw[3].grad, what="features")
