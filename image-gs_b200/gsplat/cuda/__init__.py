"""The raw operators of gsplat.cuda (gsplat/gsplat/cuda/__init__.py of the reference) that Image-GS calls, on the igs_b200 kernels."""
from .. import _path  # noqa: F401
from igs_b200.ops import (  # noqa: F401
    nd_rasterize_backward_topk_norm,
    nd_rasterize_forward_topk_norm,
    project_gaussians_2d_scale_rot_backward,
    project_gaussians_2d_scale_rot_forward,
    rate_loss_backward,
    rate_loss_forward,
    sort_intersects_by_tile,
    topk_norm_loo_loss_increase,
)


def _unused(name):
    def fn(*args, **kwargs):
        raise NotImplementedError(f"gsplat.cuda.{name} is not used by Image-GS and not provided by igs_b200")
    fn.__name__ = name
    return fn


for _name in ["nd_rasterize_forward", "nd_rasterize_backward", "nd_rasterize_forward_no_tiles", "nd_rasterize_backward_no_tiles",
              "nd_rasterize_forward_simple", "nd_rasterize_backward_simple", "rasterize_forward", "rasterize_backward",
              "compute_cov2d_bounds", "map_gaussian_to_intersects", "get_tile_bin_edges"]:
    globals()[_name] = _unused(_name)
