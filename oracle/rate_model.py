"""
ORACLE (test infrastructure): numpy restatement of the rate model's preparation, compress.rate.rate_model (compress/rate.py:131-164, with
predicting_sources 116-128 and channel_operands 69-78), one float32 rounding per operation in the reference's order, with the neighbours
of oracle/neighbors.py (brute force, small cases only). The fixtures tests/golden/py_*.npz, made by the reference's own rate_model, pin it.
"""
import math

import numpy as np

from . import neighbors as nb

MIN_SCALE = np.float32(0.3)
MAX_SLOPE = np.float32(4.0)
MIN_CCLM = 3
BOUNDARIES = np.array([0.25, 0.5, 1.0, 2.0], dtype=np.float32)  # aspect-ratio classes in octaves
LN2 = np.float32(math.log(2.0))


def predicting_sources(nbrs):
    """predicting_sources (compress/rate.py:116-128): for neighbours [P, K] (-1 for none), the Gaussians predicting from each one, as CSR
    lists in increasing order (the rows of the valid entries stably sorted by target), and their weights 1 / their neighbour counts."""
    num = len(nbrs)
    valid = nbrs >= 0
    count = valid.sum(axis=1)
    rows = np.repeat(np.arange(num), nbrs.shape[1]).reshape(num, nbrs.shape[1])[valid]
    targets = nbrs[valid]
    sources = rows[np.argsort(targets, kind="stable")]
    offsets = np.zeros(num + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(np.bincount(targets, minlength=num))
    return offsets, sources, (np.float32(1.0) / count[sources].astype(np.float32)).astype(np.float32)


def rate_model(q_xy, feat, log2_scale, q_rot, color_refs, pred_refs, steps, channel_weights, refine_bits=0):
    """A dict of the RateModel fields (neighbors, weights, slope, inv_steps, inv_feat, feat_coeffs, inv_rot, offsets, sources,
    source_weights, pred_channels) from numpy inputs: q_xy [P, 2] int64, feat [P, C], log2_scale [P, 2], q_rot [P] (float32)."""
    f32 = np.float32
    feat, log2_scale = np.asarray(feat, f32), np.asarray(log2_scale, f32)
    q_rot, steps, channel_weights = np.asarray(q_rot, f32).reshape(-1), np.asarray(steps, f32), np.asarray(channel_weights, f32)
    num, channels = feat.shape
    nbrs = nb.bitstream_neighbors(np.asarray(q_xy, np.int64), refine_bits)  # [P, 8], -1 for none
    valid = nbrs >= 0
    count = valid.sum(axis=1)
    weights = (valid.astype(f32) / np.maximum(count.astype(f32), f32(1.0))[:, None]).astype(f32)
    clamped = np.where(valid, nbrs, 0)

    offsets, sources, source_weights = predicting_sources(nbrs)

    # colour-reference subtraction and prediction references
    own = np.arange(channels)
    color = np.asarray(color_refs)
    pred = np.asarray(pred_refs)
    pidx = np.where(pred >= 0, pred, own)
    if (color >= 0).any():
        values = feat - feat[:, np.where(color >= 0, color, own)] * (color >= 0).astype(f32)
    else:
        values = feat
    values = values.astype(f32)

    # neighbour means, covariances with the reference channel and variances, summed over the neighbours in order
    mean = np.zeros((num, channels), f32)
    cov = np.zeros((num, channels), f32)
    var = np.zeros((num, channels), f32)
    vf = valid.astype(f32)
    for k in range(nb.NUM_NEIGHBORS):
        nv = (values[clamped[:, k]] * vf[:, k:k + 1]).astype(f32)
        w = weights[:, k:k + 1]
        mean = (mean + (nv * w).astype(f32)).astype(f32)
        cov = (cov + ((nv * nv[:, pidx]).astype(f32) * w).astype(f32)).astype(f32)
        var = (var + ((nv[:, pidx] * nv[:, pidx]).astype(f32) * w).astype(f32)).astype(f32)
    cov = (cov - (mean * mean[:, pidx]).astype(f32)).astype(f32)
    var = (var - (mean[:, pidx] * mean[:, pidx]).astype(f32)).astype(f32)
    ratio = (cov / (var + (steps * steps).astype(f32)).astype(f32)).astype(f32)
    has_ref = (pred >= 0).astype(f32)
    slope = (np.clip(ratio, -MAX_SLOPE, MAX_SLOPE) * has_ref).astype(f32) * (count >= MIN_CCLM).astype(f32)[:, None]
    slope = slope.astype(f32)

    # rounded residuals of the prediction in steps, and the Laplace scales of the channels
    inv_steps = (f32(1.0) / steps).astype(f32)
    dev = (values[:, pidx] - mean[:, pidx]).astype(f32)
    resid = ((((values - mean).astype(f32) - (slope * dev).astype(f32)).astype(f32)) * inv_steps).astype(f32)
    mean_abs = (np.abs(np.rint(resid)).astype(np.float64).sum(axis=0).astype(f32) / f32(num)).astype(f32)  # integer sums: exact
    inv_feat = (f32(1.0) / (np.maximum(mean_abs, MIN_SCALE) * LN2).astype(f32)).astype(f32)

    # rotation scales by aspect-ratio class
    classes = np.searchsorted(BOUNDARIES, np.abs((log2_scale[:, 0] - log2_scale[:, 1]).astype(f32)), side="left")
    abs_rot = np.abs(q_rot).astype(np.float64)
    sums = np.bincount(classes, weights=abs_rot, minlength=len(BOUNDARIES) + 1)
    counts = np.bincount(classes, minlength=len(BOUNDARIES) + 1)
    overall = f32(f32(abs_rot.sum()) / f32(num))
    scales = np.where(counts > 0, (sums.astype(f32) / np.maximum(counts, 1).astype(f32)).astype(f32), overall).astype(f32)
    inv_class = (f32(1.0) / (np.maximum(scales, MIN_SCALE) * LN2).astype(f32)).astype(f32)
    return dict(neighbors=clamped.astype(np.int32), weights=weights, slope=slope, inv_steps=inv_steps, inv_feat=inv_feat,
                feat_coeffs=(inv_feat * channel_weights).astype(f32), inv_rot=inv_class[classes][:, None], offsets=offsets.astype(np.int32),
                sources=sources.astype(np.int32), source_weights=source_weights,
                pred_channels=tuple(int(c if r < 0 else r) for c, r in enumerate(pred_refs)))
