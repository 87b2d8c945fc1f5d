"""project_gaussians_2d_scale_rot of gsplat/gsplat/project_gaussians_2d_scale_rot.py:12-28, on the igs_b200 kernels."""
from typing import Tuple

from torch import Tensor

from . import _path  # noqa: F401
from igs_b200.autograd import project_gaussians_2d_scale_rot as _project


def project_gaussians_2d_scale_rot(means2d: Tensor, scales2d: Tensor, rotation: Tensor, img_height: int, img_width: int,
                                   tile_bounds: Tuple[int, int, int]):
    """Pixel centers xys [N,2], radii [N], conics [N,3] and tiles hit [N] of 2D Gaussians with means in [0,1) image coordinates, scales
    in pixels and rotations in radians; differentiable with respect to means2d, scales2d and rotation."""
    return _project(means2d, scales2d, rotation, img_height, img_width, tile_bounds)
