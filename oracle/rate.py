"""
ORACLE (test infrastructure): PyTorch restatement of the rate term's definition (compress/rate.py: coded_values 80-84, feature_residuals
87-97, canonical_rotation 100-104, smooth_laplace_bits 107-113, rate_bits 167-175, the loss weight of rate_loss 197-202), differentiated
with autograd for the gradient. Computes in the dtype of its inputs (float32 reproduces the reference's arithmetic).
"""
import math

import torch


def coded_values(feat, color_refs):
    own = torch.arange(feat.shape[1])
    refs = torch.tensor(color_refs)
    has = refs >= 0
    if not bool(has.any()):
        return feat
    idx = torch.where(has, refs, own)
    return feat - feat[:, idx] * has.to(feat.dtype)


def rate_loss(feat, rot, l1_loss, neighbors, weights, slope, color_refs, pred_refs, inv_steps, feat_coeffs, rot_coeffs, inv_rot_step,
              l1_ratio, factor):
    """Scalar loss: factor / max(l1 / l1_ratio, 1e-4) * (feature bits + rotation bits)."""
    values = coded_values(feat, color_refs)
    nv = values[neighbors.long()]  # [P, K, C]
    mean = (weights[..., None] * nv).sum(dim=1)
    pred = torch.tensor(pred_refs).long()
    r = (values - mean - slope * (values[:, pred] - mean[:, pred])) * inv_steps
    feat_bits = ((torch.sqrt(r * r + 0.25) - 0.5) * feat_coeffs).sum()
    rot = rot.reshape(-1)
    # the quarter turns are rounded from the float32 parameters, as the reference computes them (rate.py:104 on float32 tensors)
    turns = torch.round(rot.detach().to(torch.float32) * (2.0 / math.pi)).to(rot.dtype)
    t = (rot - turns * (0.5 * math.pi)) * inv_rot_step
    rot_bits = ((torch.sqrt(t * t + 0.25) - 0.5) * rot_coeffs.reshape(-1)).sum()
    weight = factor / max(float(l1_loss) / l1_ratio, 1e-4)
    return weight * (feat_bits + rot_bits), weight
