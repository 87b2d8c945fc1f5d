"""
The neighbour search of the rate model's preparation on the GPU: compress.rate.bitstream_neighbors (compress/rate.py:56-66), whose
k nearest earlier Gaussians in bitstream order the reference finds on host threads (compress/csrc/prediction.cpp:69-166) before each
CUDA-graph capture. The bitstream order itself (the Morton curve of the coarse positions, then of the fine ones; compress/__init__.py:43-58
and compress/common.py:87-131) is a stable radix sort of 64-bit keys on the GPU (igs_bitstream_order; bitstream_order below is the host
version, used when the key would be wider); the search runs in igs_nearest_neighbors.
"""
import ctypes
from typing import Optional

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


def bitstream_order_device(positions: torch.Tensor, refine_bits: int = 0) -> Optional[torch.Tensor]:
    """bitstream_order of the integer positions [P, 2] (int64, CUDA) on the GPU: the order [P] (int64, on the device), or None when the
    sort key would be wider than 64 bits (then bitstream_order sorts on the host)."""
    if not isinstance(positions, torch.Tensor) or not positions.is_cuda or positions.dtype != torch.int64 or positions.ndim != 2 or \
            positions.size(1) != 2:
        raise RuntimeError("positions must be a CUDA int64 tensor [P, 2]")
    positions = positions.contiguous()
    num = positions.size(0)
    dev = positions.device
    order = torch.empty(num, dtype=torch.int64, device=dev)
    if num == 0:
        return order
    lib = _lib.load()
    ws_bytes = lib.igs_bitstream_order_workspace(num)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        status = lib.igs_bitstream_order(num, ptr(positions), int(refine_bits), ptr(order), ptr(ws), ws_bytes,
                                         ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    if status == _lib.IGS_ERR_UNSUPPORTED:
        return None
    if status == _lib.IGS_ERR_INVALID:
        raise ValueError(lib.igs_last_error().decode())
    _lib.check(status, "bitstream_order")
    return order


def bitstream_neighbors(q_xy, refine_bits: int = 0, device="cuda") -> np.ndarray:
    """compress.rate.bitstream_neighbors: for the integer positions q_xy [P, 2] (numpy int64), the indices [P, NUM_NEIGHBORS] (int64) of
    the NUM_NEIGHBORS nearest earlier Gaussians in bitstream order, into the Gaussians in their given order, -1 for none."""
    q_xy = np.asarray(q_xy, dtype=np.int64)
    num = len(q_xy)
    if num == 0:
        return np.full((0, NUM_NEIGHBORS), -1, dtype=np.int64)
    positions = torch.from_numpy(np.ascontiguousarray(q_xy)).to(device)
    order = bitstream_order_device(positions, refine_bits)
    if order is None:
        order = torch.from_numpy(bitstream_order(q_xy, refine_bits)).to(positions.device)
    sorted_neighbors = causal_neighbors(positions.index_select(0, order).contiguous())
    # back to the Gaussians' own order: row order[s] holds the neighbours of sorted row s, mapped to original indices
    mapped = torch.where(sorted_neighbors >= 0, order[sorted_neighbors.clamp(min=0)], sorted_neighbors)
    out = torch.empty_like(mapped)
    out[order] = mapped
    return out.cpu().numpy()
