"""
Drop-in replacement of the gsplat fork bundled with Image-GS (gsplat/gsplat/__init__.py of BaylorMultimediaLab/image-gs), for the
operators Image-GS calls, running the igs_b200 sm_100a kernels. Put the directory that holds this package first on sys.path; model.py and
compress/*.py then import it unchanged. Operators of the original extension that Image-GS never calls raise NotImplementedError.
"""
from typing import Any
import warnings

import torch

from .project_gaussians_2d_scale_rot import project_gaussians_2d_scale_rot
from .rasterize_sum import rasterize_gaussians_sum
from .utils import (
    bin_and_sort_gaussians,
    bin_and_sort_gaussians_capacity,
    compute_cov2d_bounds,
    compute_cumulative_intersects,
    get_tile_bin_edges,
    map_gaussian_to_intersects,
    sort_intersects_by_tile,
)

__version__ = "1.4.0+igs_b200"

__all__ = [
    "project_gaussians_2d_scale_rot",
    "rasterize_gaussians_sum",
    "rasterize_gaussians_no_tiles",
    "bin_and_sort_gaussians",
    "compute_cumulative_intersects",
    "compute_cov2d_bounds",
    "get_tile_bin_edges",
    "map_gaussian_to_intersects",
    "ProjectGaussians2dScaleRot",
    "RasterizeGaussiansSum",
]


def rasterize_gaussians_no_tiles(*args, **kwargs):
    raise NotImplementedError("rasterize_gaussians_no_tiles is not used by Image-GS and not provided by igs_b200")


def rasterize_gaussians_simple(*args, **kwargs):
    raise NotImplementedError("rasterize_gaussians_simple is not used by Image-GS and not provided by igs_b200")


class _Deprecated(torch.autograd.Function):
    target = None

    @classmethod
    def forward(cls, ctx, *args, **kwargs):
        warnings.warn(f"{cls.__name__} is deprecated, use {cls.target.__name__} instead", DeprecationWarning)
        return cls.target(*args, **kwargs)

    @staticmethod
    def backward(ctx: Any, *grad_outputs: Any) -> Any:
        raise NotImplementedError


class ProjectGaussians2dScaleRot(_Deprecated):
    target = staticmethod(project_gaussians_2d_scale_rot)


class RasterizeGaussiansSum(_Deprecated):
    target = staticmethod(rasterize_gaussians_sum)


class ComputeCumulativeIntersects(_Deprecated):
    target = staticmethod(compute_cumulative_intersects)
