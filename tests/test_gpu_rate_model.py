"""
The rate model's preparation on the GPU (igs_b200.rate_model.rate_model, igs_rate_model) against the reference's own
compress.rate.rate_model, run on the CPU by tests/golden/make_golden_py.py for the 480p YUV workload (prediction references Y <- neighbours,
U <- Y, V <- U; channel weights 1, 1/4, 1/4) and a small RGB one with subtract-green colour references (G <- neighbours, R-G and B-G
<- G), both with 3 refinement bits of the positions:
  * neighbours, weights, the in-neighbour lists (offsets, sources) and their weights: identical;
  * slopes within 2e-6 (float32 rounding of nearly cancelling covariances), per-channel coefficients and rotation coefficients within
    2e-6 relative (the reference's ATen operations in the same order; the means of rounded residuals and rotation indices are exact
    integer sums here).
The rate term computed from this model equals the one from the reference's model.
"""
import os

import numpy as np
import pytest
import torch

from igs_b200 import ops
from igs_b200 import rate_model as rm
from igs_b200 import workloads

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
# the channel weights the fixtures were made with (make_golden_py.py)
CHANNEL_WEIGHTS = {"cfg2_480p_yuv": [1.0, 0.25, 0.25], "rgb_subgreen_320x200": [1.0, 1.0, 1.0]}


def reference_inputs(name):
    z = np.load(os.path.join(GOLDEN, f"py_{name}.npz"))
    # rate_model's arguments as make_golden_py.py passes them: dequantized features and log2 scales (symbols times steps), rotation indices
    feat = z["q_feat"] * z["feat_steps"]
    log2_scale = z["q_scale"] * np.float32(z["scale_step"])
    pred_refs = [-1 if int(p) == c else int(p) for c, p in enumerate(z["pred_channels"])]
    return z, dict(q_xy=z["q_xy"].astype(np.int64), feat=feat.astype(np.float32), log2_scale=log2_scale.astype(np.float32),
                   q_rot=z["q_rot"][:, 0], color_refs=[int(r) for r in z["color_refs"]], pred_refs=pred_refs,
                   steps=z["feat_steps"], channel_weights=np.array(CHANNEL_WEIGHTS[name], np.float32))


@pytest.mark.parametrize("name", ["cfg2_480p_yuv", "rgb_subgreen_320x200"])
def test_rate_model_matches_reference(name, device):
    z, args = reference_inputs(name)
    model = rm.rate_model(args["q_xy"], torch.from_numpy(args["feat"]).to(device), torch.from_numpy(args["log2_scale"]).to(device),
                          torch.from_numpy(args["q_rot"]).to(device), args["color_refs"], args["pred_refs"],
                          torch.from_numpy(args["steps"]).to(device), torch.from_numpy(args["channel_weights"]).to(device),
                          refine_bits=3)
    got = {k: getattr(model, k).cpu().numpy() for k in ("neighbors", "weights", "offsets", "sources", "source_weights", "slope",
                                                          "inv_steps", "feat_coeffs", "inv_rot")}
    for k in ("neighbors", "weights", "offsets", "sources", "source_weights", "inv_steps"):
        np.testing.assert_array_equal(got[k], z[k], err_msg=k)
    # slopes lie in [-4, 4]; a covariance that nearly cancels can show one float32 rounding of its sums (1 of 12,000 values here), so
    # they are held to an absolute bound at float32 resolution
    np.testing.assert_allclose(got["slope"], z["slope"], rtol=0, atol=2e-6, err_msg="slope")
    for k in ("feat_coeffs", "inv_rot"):
        np.testing.assert_allclose(got[k], z[k], rtol=2e-6, atol=0, err_msg=k)
    assert model.pred_channels == tuple(int(p) for p in z["pred_channels"])
    assert model.color_refs == tuple(int(r) for r in z["color_refs"])
    # the rate term from this model equals the one from the reference's model
    mine = workloads.RateModelTensors(dict(z, **{k: getattr(model, k).cpu().numpy() for k in got}), device)
    theirs = workloads.RateModelTensors(z, device)
    feat = torch.from_numpy(z["out_feat"]).to(device)
    rot = torch.from_numpy(z["out_rot"]).to(device)
    l1 = torch.tensor(float(z["l1"]), device=device)
    losses = []
    for m in (mine, theirs):
        loss, *_ = ops.rate_loss_forward(feat, rot, l1, m.neighbors, m.weights, m.slope, m.color_refs, m.pred_channels, m.inv_steps,
                                         m.feat_coeffs, m.inv_rot, float(z["inv_rot_step"]), float(z["l1_ratio"]), float(z["factor"]))
        losses.append(float(loss))
    assert abs(losses[0] - losses[1]) <= 1e-6 * abs(losses[1])


def test_rate_model_rejects_bad_arguments(device):
    _, args = reference_inputs("cfg2_480p_yuv")
    feat = torch.from_numpy(args["feat"]).to(device)
    with pytest.raises(ValueError):
        rm.rate_model(args["q_xy"], feat, feat[:, :2], feat[:, 0], [-1, -1], [-1, 0], args["steps"], args["channel_weights"])
    with pytest.raises(RuntimeError, match="reference"):
        rm.rate_model(args["q_xy"], feat, feat[:, :2].contiguous(), feat[:, 0].contiguous(), [-1, -1, -1], [0, 0, 1], args["steps"],
                      args["channel_weights"])  # a channel predicting from itself


def test_installed_rate_model_with_model_py_arguments(device, monkeypatch):
    """The routed function install() puts into compress.rate, called with model.py's own argument list (model.py:790-792: numpy int64
    positions, dequantized features, log2 scales, rotation indices, the reference lists, steps, channel weights, dtype, device, refinement
    bits), then its buffer update (model.py:793-797: copy_ of every tensor field into the previous model's buffers): field for field the
    direct GPU call's result. A 13-channel call goes to the replaced function."""
    import sys
    import types

    z, args = reference_inputs("cfg2_480p_yuv")
    fake = types.ModuleType("compress_rate_stand_in")
    fallback_calls = []
    fake.rate_model = lambda *a: fallback_calls.append(a) or "reference"
    fake.bitstream_neighbors = lambda *a: "reference"
    monkeypatch.setitem(sys.modules, "compress_rate_stand_in", fake)
    replaced = rm.install("compress_rate_stand_in")
    try:
        t = lambda k: torch.from_numpy(args[k]).to(device)  # noqa: E731
        call = (args["q_xy"], t("feat"), t("log2_scale"), t("q_rot"), args["color_refs"], args["pred_refs"], t("steps"),
                t("channel_weights"), torch.float32, device, 3)
        def same(a, b):
            if isinstance(a, torch.Tensor):
                return isinstance(b, torch.Tensor) and torch.equal(a, b)
            if isinstance(a, (tuple, list)):
                return isinstance(b, (tuple, list)) and len(a) == len(b) and all(same(x, y) for x, y in zip(a, b))
            return a == b

        first = fake.rate_model(*call)
        direct = rm.rate_model(*call)
        assert type(first) is type(direct) and all(same(a, b) for a, b in zip(first, direct))
        second = fake.rate_model(*call)
        for buffer, value in zip(first, second):  # model.py's in-place update of a captured step's buffers
            if isinstance(buffer, torch.Tensor):
                buffer.copy_(value)
        assert all(same(a, b) for a, b in zip(first, direct))
        assert not fallback_calls
        wide = torch.zeros(len(args["q_xy"]), 13, device=device)
        assert fake.rate_model(args["q_xy"], wide, t("log2_scale"), t("q_rot"), [-1] * 13, [-1] * 13, torch.ones(13, device=device),
                               torch.ones(13, device=device), torch.float32, device, 3) == "reference"
        assert len(fallback_calls) == 1
    finally:
        rm.restore(replaced)


def test_in_neighbour_lists_with_a_skewed_in_degree(device):
    """igs_rate_model's in-neighbour lists through the C ABI for a neighbour graph whose first Gaussian is a neighbour of every other one
    (in-degree 20,000 where a typical one is under 16), against the oracle's stable sort (compress/rate.py:116-128): identical, and in a
    time that does not grow with the square of the longest list."""
    import ctypes

    from igs_b200 import _lib
    from igs_b200._lib import ptr
    from oracle import rate_model as orm

    num, channels = 20000, 3
    rng = np.random.default_rng(5)
    nbrs = np.full((num, 8), -1, np.int64)
    nbrs[1:, 0] = 0  # every Gaussian predicts from the first
    for k in range(1, 8):  # and from up to seven others before it
        earlier = np.arange(num) - k * 3
        nbrs[:, k] = np.where(earlier > 0, earlier, -1)
    want_offsets, want_sources, want_weights = orm.predicting_sources(nbrs)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    feat = t(rng.normal(0.5, 0.2, (num, channels)).astype(np.float32))
    log2_scale = t(rng.normal(1.0, 0.5, (num, 2)).astype(np.float32))
    q_rot = t(rng.integers(-100, 100, num).astype(np.float32))
    steps, cw = t(np.full(channels, 1 / 64, np.float32)), t(np.ones(channels, np.float32))
    lib = _lib.load()
    f32, i32 = torch.float32, torch.int32
    out = dict(neighbors=torch.empty(num, 8, dtype=i32, device=device), weights=torch.empty(num, 8, dtype=f32, device=device),
               slope=torch.empty(num, channels, dtype=f32, device=device), inv_steps=torch.empty(channels, dtype=f32, device=device),
               inv_feat=torch.empty(channels, dtype=f32, device=device), feat_coeffs=torch.empty(channels, dtype=f32, device=device),
               inv_rot=torch.empty(num, 1, dtype=f32, device=device), offsets=torch.empty(num + 1, dtype=i32, device=device),
               sources=torch.empty(num * 8, dtype=i32, device=device), source_weights=torch.empty(num * 8, dtype=f32, device=device))
    ws_bytes = lib.igs_rate_model_workspace(num)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    refs = (ctypes.c_int32 * channels)(-1, -1, -1), (ctypes.c_int32 * channels)(-1, 0, 1)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nb_dev = t(nbrs)

    def call():
        return lib.igs_rate_model(num, channels, ptr(nb_dev), ptr(feat), ptr(log2_scale), ptr(q_rot), ctypes.cast(refs[0], ctypes.c_void_p),
                                  ctypes.cast(refs[1], ctypes.c_void_p), ptr(steps), ptr(cw), ptr(out["neighbors"]), ptr(out["weights"]),
                                  ptr(out["slope"]), ptr(out["inv_steps"]), ptr(out["inv_feat"]), ptr(out["feat_coeffs"]),
                                  ptr(out["inv_rot"]), ptr(out["offsets"]), ptr(out["sources"]), ptr(out["source_weights"]), ptr(ws),
                                  ws_bytes, stream)

    assert call() == 0, lib.igs_last_error().decode()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    assert call() == 0
    b.record()
    torch.cuda.synchronize()
    edges = int(want_offsets[-1])
    np.testing.assert_array_equal(out["offsets"].cpu().numpy(), want_offsets)
    np.testing.assert_array_equal(out["sources"][:edges].cpu().numpy(), want_sources)
    np.testing.assert_array_equal(out["source_weights"][:edges].cpu().numpy(), want_weights)
    assert want_offsets[1] - want_offsets[0] == num - 1  # the skewed list is there
    assert a.elapsed_time(b) < 250.0, f"{a.elapsed_time(b):.1f} ms"
