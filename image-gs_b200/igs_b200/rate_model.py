"""
The rate model's preparation on the GPU: compress.rate.rate_model (compress/rate.py:131-164) with the same arguments and the same fields.
The reference finds the neighbours on host threads (compress/csrc/prediction.cpp) and computes the rest with ATen operations; here the
neighbours come from igs_nearest_neighbors in bitstream order (igs_b200.neighbors.bitstream_neighbors) and the rest from one C-ABI call,
igs_rate_model. The result feeds the rate term (igs_rate_fwd / igs_rate_bwd, igs_b200.pipeline.RasterStep's rate stage) as the
reference's RateModel feeds its rate_loss.
"""
import ctypes
from typing import NamedTuple, Optional

import numpy as np
import torch

from . import _lib
from ._lib import ptr
from .neighbors import NUM_NEIGHBORS, bitstream_neighbors


class RateModel(NamedTuple):
    """The fields of compress.rate.RateModel (compress/rate.py:26-42), for P Gaussians with C channels and K = 8 neighbours."""
    neighbors: torch.Tensor       # [P, K] int32, missing ones clamped to 0
    weights: torch.Tensor         # [P, K]: 1 / the number of neighbours, 0 for missing ones
    slope: torch.Tensor           # [P, C]: CCLM slopes
    inv_steps: torch.Tensor       # [C]
    inv_feat: torch.Tensor        # [C]: 1 / (scale ln 2) of the feature channels
    feat_coeffs: torch.Tensor     # [C]: inv_feat times the channel weights
    inv_rot: torch.Tensor         # [P, 1]: 1 / (scale ln 2) of each Gaussian's rotation
    offsets: torch.Tensor         # [P + 1] int32
    sources: torch.Tensor         # [E] int32: the Gaussians predicting from Gaussian j are sources[offsets[j]:offsets[j + 1]]
    source_weights: torch.Tensor  # [E]
    operands: tuple               # channel_operands, for the reference's Python rate_bits
    color_refs: tuple
    pred_channels: tuple


def channel_operands(color_refs, pred_refs, device):
    """The channel references in the index-tensor form of the reference's RateModel.operands (compress/rate.py:69-78), for its Python
    rate_bits: (colour reference of each channel with the mask of channels that have one, or None when none has) and the prediction
    reference of each channel, a channel without one standing for itself."""
    fill = lambda refs: [int(r) if int(r) >= 0 else c for c, r in enumerate(refs)]  # noqa: E731
    pred_idx = torch.tensor(fill(pred_refs), device=device)
    if not any(int(r) >= 0 for r in color_refs):
        return None, pred_idx
    mask = torch.tensor([int(r) >= 0 for r in color_refs], device=device)
    return (torch.tensor(fill(color_refs), device=device), mask), pred_idx


def rate_model(q_xy, feat, log2_scale, q_rot, color_refs, pred_refs, steps, channel_weights, dtype=torch.float32,
               device: Optional[torch.device] = None, refine_bits: int = 0) -> RateModel:
    """compress.rate.rate_model on the GPU: q_xy [P, 2] integer positions (numpy int64), feat [P, C] dequantized features, log2_scale
    [P, 2] canonical log2 scales, q_rot [P] rotation indices, color_refs / pred_refs [C] (-1 for none), steps [C] feature steps,
    channel_weights [C]; float32 CUDA tensors (device: the features' device when not given)."""
    if dtype != torch.float32:
        raise ValueError("rate_model computes in float32")
    device = torch.device(device) if device is not None else feat.device
    if device.type != "cuda":
        raise RuntimeError("rate_model runs on a CUDA device")
    as_f32 = lambda t: torch.as_tensor(t, dtype=torch.float32, device=device).contiguous()
    feat, log2_scale, steps, channel_weights = as_f32(feat), as_f32(log2_scale), as_f32(steps), as_f32(channel_weights)
    q_rot = as_f32(q_rot).reshape(-1)
    num, channels = feat.shape
    if log2_scale.shape != (num, 2) or q_rot.numel() != num or steps.numel() != channels or channel_weights.numel() != channels:
        raise ValueError("rate_model: inconsistent shapes")
    if len(color_refs) != channels or len(pred_refs) != channels:
        raise ValueError("rate_model: one colour and one prediction reference per channel")
    neighbors = torch.from_numpy(bitstream_neighbors(np.asarray(q_xy, dtype=np.int64), refine_bits, device)).to(device)
    lib = _lib.load()
    f32, i32 = torch.float32, torch.int32
    out_neighbors = torch.empty(num, NUM_NEIGHBORS, dtype=i32, device=device)
    weights = torch.empty(num, NUM_NEIGHBORS, dtype=f32, device=device)
    slope = torch.empty(num, channels, dtype=f32, device=device)
    inv_steps, inv_feat, feat_coeffs = (torch.empty(channels, dtype=f32, device=device) for _ in range(3))
    inv_rot = torch.empty(num, 1, dtype=f32, device=device)
    offsets = torch.empty(num + 1, dtype=i32, device=device)
    sources = torch.empty(max(1, num * NUM_NEIGHBORS), dtype=i32, device=device)
    source_weights = torch.empty(max(1, num * NUM_NEIGHBORS), dtype=f32, device=device)
    ws_bytes = lib.igs_rate_model_workspace(num)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    crefs = (ctypes.c_int32 * channels)(*[int(r) for r in color_refs])
    prefs = (ctypes.c_int32 * channels)(*[int(r) for r in pred_refs])
    with torch.cuda.device(device):
        _lib.check(lib.igs_rate_model(num, channels, ptr(neighbors), ptr(feat), ptr(log2_scale), ptr(q_rot),
                                      ctypes.cast(crefs, ctypes.c_void_p), ctypes.cast(prefs, ctypes.c_void_p), ptr(steps),
                                      ptr(channel_weights), ptr(out_neighbors), ptr(weights), ptr(slope), ptr(inv_steps), ptr(inv_feat),
                                      ptr(feat_coeffs), ptr(inv_rot), ptr(offsets), ptr(sources), ptr(source_weights), ptr(ws), ws_bytes,
                                      ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)), "rate_model")
    edges = int(offsets[-1].item())
    pred_channels = tuple(c if int(r) < 0 else int(r) for c, r in enumerate(pred_refs))
    return RateModel(out_neighbors, weights, slope, inv_steps, inv_feat, feat_coeffs, inv_rot, offsets, sources[:edges],
                     source_weights[:edges], channel_operands(color_refs, pred_refs, device), tuple(int(r) for r in color_refs),
                     pred_channels)


MAX_CHANNELS = 12  # IGS_MAX_CHANNELS of include/igs_b200.h: feature channels igs_rate_model handles


def runs_on_gpu(feat, device, dtype=torch.float32) -> bool:
    """Whether rate_model's arguments are ones the GPU version handles: float32, a CUDA device and at most MAX_CHANNELS feature channels.
    Anything else (a texture stack of more channels, the CPU) is the reference's own code's."""
    if dtype != torch.float32 or not torch.cuda.is_available():
        return False
    dev = torch.device(device) if device is not None else getattr(feat, "device", torch.device("cpu"))
    channels = feat.shape[-1] if hasattr(feat, "shape") and len(feat.shape) == 2 else MAX_CHANNELS + 1
    return dev.type == "cuda" and channels <= MAX_CHANNELS


def routed_rate_model(original):
    """compress.rate.rate_model with the reference's signature, on the GPU where runs_on_gpu holds and by `original` otherwise"""

    def rate_model_routed(q_xy, feat, log2_scale, q_rot, color_refs, pred_refs, steps, channel_weights, dtype, device, refine_bits=0):
        if runs_on_gpu(feat, device, dtype):
            return rate_model(q_xy, feat, log2_scale, q_rot, color_refs, pred_refs, steps, channel_weights, dtype, device, refine_bits)
        return original(q_xy, feat, log2_scale, q_rot, color_refs, pred_refs, steps, channel_weights, dtype, device, refine_bits)

    rate_model_routed.original = original
    return rate_model_routed


def routed_bitstream_neighbors(original):
    """compress.rate.bitstream_neighbors with the reference's signature, on the GPU when there is one and by `original` otherwise"""

    def bitstream_neighbors_routed(q_xy, refine_bits=0):
        if torch.cuda.is_available():
            return bitstream_neighbors(q_xy, refine_bits)
        return original(q_xy, refine_bits)

    bitstream_neighbors_routed.original = original
    return bitstream_neighbors_routed


def install(*module_names):
    """Route the reference's calls of compress.rate.rate_model and bitstream_neighbors to the GPU versions (same signatures): the names
    are replaced in each named module that is imported or importable (default: compress.rate and model, which binds rate_model when it is
    imported, model.py:43). Calls the GPU versions do not handle (more than MAX_CHANNELS feature channels, a CPU device or no GPU, a
    dtype other than float32) go to the replaced functions, so training that ran with the reference runs the same. Returns
    {(module, name): original} for restore()."""
    import importlib

    routes = {"rate_model": routed_rate_model, "bitstream_neighbors": routed_bitstream_neighbors}
    replaced = {}
    for name in module_names or ("compress.rate", "model"):
        try:
            module = importlib.import_module(name)
        except ImportError:
            continue
        for attr, route in routes.items():
            if hasattr(module, attr):
                original = getattr(module, attr)
                replaced[(name, attr)] = original
                setattr(module, attr, route(getattr(original, "original", original)))
    return replaced


def restore(replaced):
    """Undo install()."""
    import importlib

    for (name, attr), original in replaced.items():
        setattr(importlib.import_module(name), attr, original)
