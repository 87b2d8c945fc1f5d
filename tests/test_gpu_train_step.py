"""
The fused training step (igs_train_step_l1: projection with the tiles hit, the stages' memsets and the first prefix-sum pass in one
kernel, the loss finished by the projection backward's last block) against the same step as separate C-ABI calls
(igs_project_fwd, igs_cumsum, igs_sort_intersects, igs_raster_step_l1, igs_project_bwd) on the same inputs: projection, prefix sums, tile
lists and render bit for bit, gradients up to the order of float atomics, the loss up to the order of its sum. Also over a band of tile
rows (without the projection backward) against igs_band_tiles_hit / igs_sort_intersects_band / igs_raster_step_l1_band.
"""
import pytest
import torch

from common import assert_close_grad, make_case, to_dev

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
EXACT = ("xys", "radii", "conics", "hits", "cum", "num_intersects", "ids", "bins", "image")
GRADS = ("v_xy", "v_conic", "v_colors", "v_cov2d", "v_mean2d", "v_scale", "v_rot")


def snapshot(step, keys):
    return {k: getattr(step, k).detach().clone() for k in keys}


@pytest.mark.parametrize("h,w,n,c,seed", [(256, 256, 1000, 3, 1), (88, 120, 400, 3, 2), (64, 80, 300, 9, 3), (33, 47, 150, 1, 4),
                                          (16, 16, 0, 3, 5), (1, 1, 5, 3, 6)])
def test_fused_step_equals_the_stage_calls(h, w, n, c, seed):
    from igs_b200 import pipeline

    wl, inp = make_case(h, w, n, c=c, seed=seed)
    d = to_dev(inp, DEV)
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], capacity=max(1024, 3 * 64 * n))
    assert step.BASE_STAGES == ("_train_step",)
    for _ in range(2):  # a second call: everything it zeroes or accumulates starts afresh
        step.launch()
    torch.cuda.synchronize()
    fused = snapshot(step, EXACT + GRADS + ("loss",))
    for s in step.BREAKDOWN_STAGES:
        getattr(step, s)()
    torch.cuda.synchronize()
    staged = snapshot(step, EXACT + GRADS + ("loss",))
    total = int(staged["num_intersects"])
    for k in EXACT:
        a, b = fused[k], staged[k]
        if k == "ids":
            a, b = a[:total], b[:total]
        assert torch.equal(a, b), k
    for k in GRADS:
        assert_close_grad(fused[k], staged[k], what=k)
    assert abs(float(fused["loss"]) - float(staged["loss"])) <= 2e-6 * max(abs(float(staged["loss"])), 1e-12)


@pytest.mark.parametrize("rows", [(0, 3), (3, 9), (9, 16)])
def test_fused_band_step_equals_the_band_calls(rows):
    from igs_b200 import bands

    wl, inp = make_case(250, 200, 900, seed=11)
    d = to_dev(inp, DEV)
    r0, r1 = rows
    step = bands.BandStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], wl.height, wl.width, r0, r1,
                          capacity=20000)
    assert step.LOCAL == ("_train_step",)
    step._train_step()
    torch.cuda.synchronize()
    keys = ("xys", "radii", "conics", "band_hits", "cum", "num_intersects", "ids", "bins", "image")
    fused = snapshot(step, keys + ("p_xy", "p_conic", "p_colors", "p_loss"))
    for s in ("_project", "_cumsum", "_bin", "_raster"):
        getattr(step, s)()
    torch.cuda.synchronize()
    staged = snapshot(step, keys + ("p_xy", "p_conic", "p_colors", "p_loss"))
    total = int(staged["num_intersects"])
    for k in keys:
        a, b = fused[k], staged[k]
        if k == "ids":
            a, b = a[:total], b[:total]
        assert torch.equal(a, b), k
    for k in ("p_xy", "p_conic", "p_colors"):
        assert_close_grad(fused[k], staged[k], what=k)
    assert abs(float(fused["p_loss"]) - float(staged["p_loss"])) <= 2e-6 * max(abs(float(staged["p_loss"])), 1e-12)


def test_packed_inputs_give_the_same_step():
    """RasterStep.pack_inputs(): the parameters moved into one buffer in packed_layout() (one host-to-device copy per step for a
    caller keeping them on the host) give the same step bit for bit, and a write to the buffer is what the next step reads."""
    from igs_b200 import pipeline

    wl, inp = make_case(96, 128, 500, c=3, seed=8)
    d = to_dev(inp, DEV)
    step = pipeline.RasterStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], capacity=64 * 500)
    step.replay()
    torch.cuda.synchronize()
    before = snapshot(step, EXACT + ("loss",))
    flat = step.pack_inputs()
    offsets, length = pipeline.RasterStep.packed_layout(step.n, step.c)
    assert flat.numel() == length and all(o % pipeline.RasterStep.PACK_ALIGN == 0 for o in offsets)
    for t, at in zip((d["means"], d["scales"], d["rotations"], d["features"]), offsets):
        assert torch.equal(flat[at:at + t.numel()].view(t.shape), t)
    step.replay()  # captured again over the packed arrays
    torch.cuda.synchronize()
    after = snapshot(step, EXACT + ("loss",))
    for k in EXACT:
        assert torch.equal(before[k], after[k]), k
    assert float(before["loss"]) == float(after["loss"])
    flat[offsets[3]:offsets[3] + 3 * step.n].zero_()  # black features: a black image
    step.replay()
    torch.cuda.synchronize()
    assert float(step.image.abs().max()) == 0.0
