"""rasterize_gaussians_sum of gsplat/gsplat/rasterize_sum.py:14-53, on the igs_b200 kernels (top-K normalized mode)."""
from typing import Optional

from torch import Tensor

from . import _path  # noqa: F401
from igs_b200.autograd import rasterize_gaussians_sum_topk


def rasterize_gaussians_sum(xys: Tensor, radii: Tensor, conics: Tensor, num_tiles_hit: Tensor, colors: Tensor, img_height: int,
                            img_width: int, BLOCK_H: int = 16, BLOCK_W: int = 16, topk_norm: bool = False,
                            capacity: Optional[int] = None) -> Tensor:
    """
    Top-K normalized rendering [H, W, C] (a view of a channel-planar [C, H, W] buffer). With capacity, the tile intersections go to
    fixed-capacity buffers without reading their number back to the CPU (CUDA graph capture), and intersections beyond it are dropped.
    Only topk_norm=True (what Image-GS uses, model.py:970) and 16x16 blocks are provided.
    """
    if not topk_norm:
        raise NotImplementedError("igs_b200 provides the top-K normalized rasterizer only (topk_norm=True)")
    if (BLOCK_H, BLOCK_W) != (16, 16):
        raise ValueError("igs_b200 rasterizes 16x16 tiles (BLOCK_H = BLOCK_W = 16)")
    return rasterize_gaussians_sum_topk(xys, radii, conics, num_tiles_hit, colors, img_height, img_width, capacity)
