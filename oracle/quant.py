"""
ORACLE (test infrastructure): PyTorch restatement of the straight-through "step" quantization of the training step
(model.py:993-1006 with compress/quantization.py: quantize_step 36-42, dequantize 45-46, canonicalize 61-74, get_step_symbols 151-172,
dequantize_symbols 188-199), quarter turns off and scales in the log2 domain as during optimization. Device-agnostic: the tests run it on
the CPU, and on CUDA tensors to obtain ATen's own GPU arithmetic.
"""
import torch


def step_symbols(xy, scale, rot, feat, pos_steps, scale_step, rot_step, feat_steps):
    """Integer-valued float symbols of the canonicalized parameters (scale non-negative, in pixels)."""
    scale_steps = torch.full((2,), scale_step, dtype=xy.dtype, device=xy.device)
    rot_steps = torch.full((1,), rot_step, dtype=xy.dtype, device=xy.device)
    q_xy = torch.round(xy / pos_steps)
    q_scale = torch.round(torch.log2(scale.abs()) / scale_steps)
    q_rot = torch.round(rot / rot_steps)
    q_feat = torch.round(feat / feat_steps)
    return q_xy, q_scale, q_rot, q_feat


def dequantize(q_xy, q_scale, q_rot, q_feat, pos_steps, scale_step, rot_step, feat_steps):
    zeros = lambda s: torch.zeros_like(s)  # noqa: E731  (origins of "step" quantization)
    scale_steps = torch.full((2,), scale_step, dtype=q_xy.dtype, device=q_xy.device)
    rot_steps = torch.full((1,), rot_step, dtype=q_xy.dtype, device=q_xy.device)
    xy = q_xy * pos_steps + zeros(pos_steps)
    scale = torch.exp2(q_scale * scale_steps + zeros(scale_steps))
    rot = q_rot * rot_steps + zeros(rot_steps)
    feat = q_feat * feat_steps + zeros(feat_steps)
    return xy, scale, rot, feat


def quantize_ste(xy, scale, rot, feat, pos_steps, scale_step, rot_step, feat_steps):
    """(values x + (dequantize(q) - x), symbols) with the operation order of the reference."""
    sym = step_symbols(xy, scale, rot, feat, pos_steps, scale_step, rot_step, feat_steps)
    deq = dequantize(*sym, pos_steps, scale_step, rot_step, feat_steps)
    values = [x + (q - x) for x, q in zip((xy, scale, rot, feat), deq)]
    return values, sym
