"""Binning helpers of gsplat/gsplat/utils.py, on the igs_b200 kernels."""
from typing import Tuple

from torch import Tensor

from . import _path  # noqa: F401
from igs_b200 import ops as _ops


def compute_cumulative_intersects(num_tiles_hit: Tensor) -> Tuple[int, Tensor]:
    """(total number of tile intersections as a Python int, inclusive int32 prefix sum); reads the total back to the host
    (utils.py:96-115)."""
    cum, total = _ops.cumulative_intersects(num_tiles_hit.contiguous())
    return int(total.item()), cum


def sort_intersects_by_tile(num_points: int, capacity: int, xys: Tensor, radii: Tensor, cum_tiles_hit: Tensor,
                            tile_bounds: Tuple[int, int, int]) -> Tuple[Tensor, Tensor]:
    """Gaussian IDs of the tile intersections sorted by tile, increasing ID within each tile, in `capacity` slots (beyond the capacity
    dropped, unused slots 0), and tile_bins [T, 2] (utils.py:165-186)."""
    return _ops.sort_intersects_by_tile(num_points, capacity, xys.contiguous(), radii.contiguous(), cum_tiles_hit.contiguous(), tile_bounds)


def bin_and_sort_gaussians_capacity(num_points: int, capacity: int, xys: Tensor, radii: Tensor, num_tiles_hit: Tensor,
                                    tile_bounds: Tuple[int, int, int]) -> Tuple[Tensor, Tensor]:
    """sort_intersects_by_tile from the tiles hit per Gaussian, without host synchronization (utils.py:189-199)."""
    cum, _ = _ops.cumulative_intersects(num_tiles_hit.contiguous())
    return sort_intersects_by_tile(num_points, capacity, xys, radii, cum, tile_bounds)


def _unused(name):
    def fn(*args, **kwargs):
        raise NotImplementedError(f"{name} (the legacy 64-bit key binning) is not used by Image-GS and not provided by igs_b200; "
                                  "use sort_intersects_by_tile")
    fn.__name__ = name
    return fn


map_gaussian_to_intersects = _unused("map_gaussian_to_intersects")
get_tile_bin_edges = _unused("get_tile_bin_edges")
bin_and_sort_gaussians = _unused("bin_and_sort_gaussians")
compute_cov2d_bounds = _unused("compute_cov2d_bounds")
