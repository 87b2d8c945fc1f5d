"""
The neighbour search of the rate model's preparation on the GPU: compress.rate.bitstream_neighbors (compress/rate.py:56-66), whose
k nearest earlier Gaussians in bitstream order the reference finds on host threads (compress/csrc/prediction.cpp:69-166) before each
CUDA-graph capture. The bitstream order itself (the Morton curve of the coarse positions, then of the fine ones; compress/__init__.py:43-58
and compress/common.py:87-131) is a sort of 64-bit codes on the host, as in the reference; the search runs in igs_nearest_neighbors.
"""
import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import ptr

NUM_NEIGHBORS = 8


def nearest_neighbors(positions: torch.Tensor, causal: bool = True, return_dist2: bool = False):
    """The NUM_NEIGHBORS nearest earlier (causal) or other Gaussians of each of the integer positions [P, 2] (int64, CUDA), by squared
    distance and then by index: indices [P, NUM_NEIGHBORS] int64 (-1 where there are fewer) and optionally the squared distances."""
    if not isinstance(positions, torch.Tensor) or not positions.is_cuda or positions.dtype != torch.int64:
        raise RuntimeError("positions must be a CUDA int64 tensor")
    if positions.ndim != 2 or positions.size(1) != 2:
        raise ValueError("positions must be [P, 2]")
    positions = positions.contiguous()
    num = positions.size(0)
    dev = positions.device
    lib = _lib.load()
    neighbors = torch.empty(num, NUM_NEIGHBORS, device=dev, dtype=torch.int64)
    dist2 = torch.empty_like(neighbors) if return_dist2 else None
    ws_bytes = lib.igs_neighbors_workspace(num)
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        _lib.check(lib.igs_nearest_neighbors(num, ptr(positions), int(bool(causal)), ptr(neighbors), ptr(dist2), ptr(ws), ws_bytes,
                                             ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)), "nearest_neighbors")
    return (neighbors, dist2) if return_dist2 else neighbors


def causal_neighbors(positions: torch.Tensor) -> torch.Tensor:
    """igs_prediction.causal_neighbors (prediction.cpp:161-166) on the GPU."""
    return nearest_neighbors(positions, causal=True)


def _part1by1(x):
    # the lower 32 bits of x spread to the even bit positions (the Morton interleave of compress/common.py:87-97, a standard bit trick)
    x = x & np.uint64(0x00000000FFFFFFFF)
    for shift, mask in ((16, 0x0000FFFF0000FFFF), (8, 0x00FF00FF00FF00FF), (4, 0x0F0F0F0F0F0F0F0F), (2, 0x3333333333333333),
                        (1, 0x5555555555555555)):
        x = (x | (x << np.uint64(shift))) & np.uint64(mask)
    return x


def morton_encode(x, y):
    return _part1by1(np.asarray(x).astype(np.uint64)) | (_part1by1(np.asarray(y).astype(np.uint64)) << np.uint64(1))


def bitstream_order(positions, refine_bits: int = 0):
    """The order of the Gaussians in the bitstream (compress/__init__.py:43-58): along the Morton curve of positions >> refine_bits, ties
    by the Morton code of the positions, then by index (stable)."""
    positions = np.asarray(positions, dtype=np.int64)
    coarse = positions >> refine_bits if refine_bits else positions
    values = coarse - coarse.min(axis=0)
    if values.max() >= 2 ** 32:
        raise ValueError("The position must have at most 2^32 quantization levels per coordinate")
    codes = morton_encode(values[:, 0], values[:, 1])
    if refine_bits == 0:
        return np.argsort(codes, kind="stable")
    fine = morton_encode(*(positions - positions.min(axis=0)).T)
    return np.lexsort((fine, codes))


def bitstream_neighbors(q_xy, refine_bits: int = 0, device="cuda") -> np.ndarray:
    """compress.rate.bitstream_neighbors: for the integer positions q_xy [P, 2] (numpy int64), the indices [P, NUM_NEIGHBORS] (int64) of
    the NUM_NEIGHBORS nearest earlier Gaussians in bitstream order, into the Gaussians in their given order, -1 for none."""
    q_xy = np.asarray(q_xy, dtype=np.int64)
    num = len(q_xy)
    out = np.full((num, NUM_NEIGHBORS), -1, dtype=np.int64)
    if num == 0:
        return out
    order = bitstream_order(q_xy, refine_bits)
    sorted_neighbors = causal_neighbors(torch.from_numpy(np.ascontiguousarray(q_xy[order])).to(device)).cpu().numpy()
    out[order] = np.where(sorted_neighbors >= 0, order[sorted_neighbors.clip(min=0)], -1)
    return out
