"""
Image-GS's CUDA-graph training step (the protocol of model.py's _capture_step, model.py:1160-1209) through the drop-in gsplat package:
the model optimises positions in [0, 1), inverse scales, rotations and features with Adam; one eager step runs on a side stream, then the
next step is captured into a CUDA graph with its own memory pool (torch.cuda.graph_pool_handle): forward as model.forward calls it
(project_gaussians_2d_scale_rot, then rasterize_gaussians_sum with topk_norm=True and a fixed intersection capacity of twice the current
count, model.py:966-975), F.l1_loss (ATen's, or the library's as install_l1() routes it), backward and the optimizer step. The graph is replayed; at every replay the gradients it computed
must equal those of an eager forward and backward at the same parameters (float atomics reorder sums: the gradient tolerance), and the
optimizer step inside the graph must move the parameters. The first eager step's gradients are checked against the oracle's step.
"""
import pytest
import torch
import torch.nn.functional as F

from common import assert_close_grad, make_case, to_dev

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def loss_of(params, h, w, target, capacity, routed=False):
    import gsplat
    from igs_b200 import autograd as ag
    from igs_b200 import ops

    xy, inv_scale, rot, feat = params
    xys, radii, conics, hits = gsplat.project_gaussians_2d_scale_rot(xy, 1.0 / inv_scale, rot, h, w, ops.tile_grid(h, w))
    img = gsplat.rasterize_gaussians_sum(xys, radii, conics, hits, feat, h, w, 16, 16, topk_norm=True, capacity=capacity)
    img = img.view(-1, h, w, feat.shape[1]).permute(0, 3, 1, 2).contiguous().squeeze(0)
    l1_loss = ag._routed_l1_loss if routed else F.l1_loss  # routed: model.py's F.l1_loss after igs_b200.autograd.install_l1()
    return l1_loss(img, target), hits


def eager_grads(values, h, w, target, routed=False):
    params = [v.clone().requires_grad_(True) for v in values]
    loss, _ = loss_of(params, h, w, target, None, routed)
    loss.backward()
    return [p.grad for p in params], float(loss)


@pytest.mark.parametrize("routed", [False, True])
def test_graph_captured_training_step_through_dropin(routed):
    from oracle import cpu as orc

    wl, inp = make_case(112, 144, 600, seed=29)
    h, w = wl.height, wl.width
    d = to_dev(inp, DEV)
    target = d["target"]
    params = [torch.nn.Parameter(t) for t in (d["means"].clone(), 1.0 / d["scales"], d["rotations"].clone(), d["features"].clone())]
    opt = torch.optim.Adam(params, lr=1e-3, capturable=True)  # as model.py builds its optimizer for CUDA-graph steps

    # the eager step on a side stream (model.py: before any capture; it also creates the optimizer state)
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        opt.zero_grad()
        loss, hits = loss_of(params, h, w, target, None, routed)
        loss.backward()
        first = [p.grad.clone() for p in params]
        opt.step()
        with torch.no_grad():
            capacity = max(1024, round(2.0 * int(hits.sum())))
    torch.cuda.current_stream(DEV).wait_stream(side)
    torch.cuda.synchronize()

    # the first step's gradients against the oracle's step (L1 signs can flip where two renders straddle the target within rounding)
    r = orc.train_step(*[inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")], h, w)
    assert_close_grad(first[0], r["v_mean2d"].reshape(first[0].shape), rtol=2e-3, what="v_mean2d")
    assert_close_grad(first[3], r["v_colors"].reshape(first[3].shape), rtol=2e-3, what="v_colors")
    # d loss / d inv_scale = d loss / d scale * (-1 / inv_scale^2)
    v_inv = (r["v_scale"].reshape(first[1].shape) * -(d["scales"].cpu().numpy() ** 2))
    assert_close_grad(first[1], v_inv, rtol=2e-3, what="v_inv_scale")

    # the capture (model.py: gradients set to None, so that backward allocates them from the graph's pool)
    opt.zero_grad(set_to_none=True)
    pool = torch.cuda.graph_pool_handle()
    graph = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.stream(side):
        graph.capture_begin(pool=pool)
        g_loss, _ = loss_of(params, h, w, target, capacity, routed)
        g_loss.backward()
        opt.step()
        graph.capture_end()
    torch.cuda.synchronize()

    for _ in range(3):
        before = [p.detach().clone() for p in params]
        graph.replay()
        torch.cuda.synchronize()
        want, want_loss = eager_grads(before, h, w, target, routed)
        assert abs(float(g_loss) - want_loss) <= 2e-6 * want_loss
        for p, g, name in zip(params, want, ("xy", "inv_scale", "rot", "feat")):
            assert_close_grad(p.grad, g, what=f"graph-replayed {name} gradient")
        assert any(not torch.equal(p.detach(), b) for p, b in zip(params, before)), "the optimizer step did not run"
