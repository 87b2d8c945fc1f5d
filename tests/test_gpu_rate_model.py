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
