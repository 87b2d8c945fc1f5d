"""
The reference's own CUDA kernels (its gsplat extension, built from source into oracle/_ref) beside ours on the same B200 and the same
1080p/20k inputs: the top-K forward and backward kernels one to one, the leave-one-out pruning kernel, the feature weights (ATen
operations in the reference), and the whole step as model.py drives it (projection, prefix sum, binning with the exact count read back,
forward, ATen's L1 loss and its gradient, backward, projection backward). Times are CUDA-event
medians of eager launches after warm-up, L2 flushed before each; ours must not be slower. Run with -s to see the table.
"""
import pytest
import torch

from igs_b200 import ops, pipeline, workloads
from oracle import weights as ow

pytestmark = pytest.mark.gpu

FLUSH = 256 << 20


def median_ms(fn, reps=20, warmup=3):
    flush = torch.empty(FLUSH, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    times = []
    for _ in range(reps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return sorted(times)[len(times) // 2]


def test_faster_than_reference_kernels(device, ref_module):
    wl = workloads.get_workload("cfg3_1080p")
    inp = workloads.make_inputs(wl)
    d = {k: v.to(device) for k, v in inp.items()}
    h, w, n = wl.height, wl.width, wl.num_gaussians
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum = torch.cumsum(hits, dim=0, dtype=torch.int32)
    total = int(cum[-1].item())
    ids, bins = ops.sort_intersects_by_tile(n, total, xys, radii, cum, tb)
    feats = d["features"]
    _, topk = ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feats)
    v_out = torch.sign(torch.randn(3, h, w, generator=torch.Generator().manual_seed(2))).to(device) / (3 * h * w)

    rows = {}
    rows["top-K forward, [H,W,10] lists"] = (
        median_ms(lambda: ref_module.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feats)),
        median_ms(lambda: ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feats)))
    rows["top-K backward, [H,W,10] lists"] = (
        median_ms(lambda: ref_module.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feats, v_out, topk)),
        median_ms(lambda: ops.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feats, v_out, topk)))

    rows["leave-one-out loss increase (pruning)"] = (
        median_ms(lambda: ref_module.topk_norm_loo_loss_increase(h, w, xys, conics, feats, topk, d["target"], False, 1e-4)),
        median_ms(lambda: ops.topk_norm_loo_loss_increase(h, w, xys, conics, feats, topk, d["target"], False, 1e-4)))
    # the reference computes the feature weights with ATen operations (model.py:1404-1421, quantization.py:218-230), restated in
    # oracle/weights.py and run here on the GPU
    rows["feature weights (ATen in the reference)"] = (
        median_ms(lambda: ow.feature_weights(xys, conics, topk, h, w), reps=5),
        median_ms(lambda: ops.topk_feature_weights(h, w, xys, conics, topk)))

    def reference_step():
        x, r, c, t = ref_module.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
        cs = torch.cumsum(t, dim=0, dtype=torch.int32)
        cap = int(cs[-1].item())
        i, bn = ref_module.sort_intersects_by_tile(n, cap, x, r, cs, tb)
        img, tk = ref_module.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), i, bn, x.contiguous(), c.contiguous(), feats)
        diff = img - d["target"]
        loss = diff.abs().mean()
        grad = torch.sign(diff) / diff.numel()
        v_xy, v_conic, _ = ref_module.nd_rasterize_backward_topk_norm(h, w, 16, 16, x, c, feats, grad, tk)
        ref_module.project_gaussians_2d_scale_rot_backward(n, d["means"], d["scales"], d["rotations"], h, w, r, c, v_xy, v_conic)
        return loss

    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"])
    rows["whole step, eager"] = (median_ms(reference_step), median_ms(step.launch))
    graph = step.capture()
    rows["whole step (ours as one CUDA graph)"] = (rows["whole step, eager"][0], median_ms(graph.replay))

    print()
    print(f"{'1080p/20k on B200':40s} {'reference ms':>13s} {'ours ms':>9s} {'speed-up':>9s}")
    for name, (ref_ms, ours_ms) in rows.items():
        print(f"{name:40s} {ref_ms:13.3f} {ours_ms:9.3f} {ref_ms / ours_ms:8.2f}x")
    # none may be slower
    for name, (ref_ms, ours_ms) in rows.items():
        assert ours_ms <= ref_ms, f"{name}: ours {ours_ms:.3f} ms, reference {ref_ms:.3f} ms"


@pytest.mark.parametrize("name", ["cfg4_2160p", "cfg5_tex9"])
def test_faster_than_reference_kernels_at_other_sizes(name, device, ref_module):
    """The top-K operators one to one at 3840x2160 with 80,000 Gaussians and at one 2048x2048 image of 9 channels with 50,000 Gaussians
    (the reference's 16-value backward path), same inputs for both; ours must not be slower."""
    wl = workloads.get_workload(name)
    inp = workloads.make_inputs(wl)
    d = {k: v.to(device) for k, v in inp.items()}
    h, w, n = wl.height, wl.width, wl.num_gaussians
    tb = ops.tile_grid(h, w)
    xys, radii, conics, hits = ops.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum = torch.cumsum(hits, dim=0, dtype=torch.int32)
    total = int(cum[-1].item())
    ids, bins = ops.sort_intersects_by_tile(n, total, xys, radii, cum, tb)
    feats = d["features"]
    _, topk = ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feats)
    v_out = torch.sign(torch.randn(wl.channels, h, w, generator=torch.Generator().manual_seed(2))).to(device) / (wl.channels * h * w)
    rows = {
        "top-K forward, [H,W,10] lists": (
            median_ms(lambda: ref_module.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feats)),
            median_ms(lambda: ops.nd_rasterize_forward_topk_norm(tb, (16, 16, 1), (w, h, 1), ids, bins, xys, conics, feats))),
        "top-K backward, [H,W,10] lists": (
            median_ms(lambda: ref_module.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feats, v_out, topk)),
            median_ms(lambda: ops.nd_rasterize_backward_topk_norm(h, w, 16, 16, xys, conics, feats, v_out, topk))),
    }
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"])
    graph = step.capture()
    ours_step = median_ms(graph.replay)
    print()
    print(f"{name:40s} {'reference ms':>13s} {'ours ms':>9s} {'speed-up':>9s}   (our whole step {ours_step:.3f} ms)")
    for row, (ref_ms, ours_ms) in rows.items():
        print(f"{row:40s} {ref_ms:13.3f} {ours_ms:9.3f} {ref_ms / ours_ms:8.2f}x")
    for row, (ref_ms, ours_ms) in rows.items():
        assert ours_ms <= ref_ms, f"{name} {row}: ours {ours_ms:.3f} ms, reference {ref_ms:.3f} ms"
