"""
The C-ABI library without a GPU: it loads, exports every entry point include/igs_b200.h declares, answers its host-side queries, and
rejects invalid arguments on the host (IGS_ERR_INVALID with a message) before any CUDA call. The Python layers reject CPU tensors, and the
gsplat drop-in exposes every name that Image-GS's model.py and compress/*.py import.
"""
import ctypes
import os
import re

import pytest
import torch

from igs_b200 import _lib, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "igs_b200.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+char\s*\*\s*|int\s+|size_t\s+)(igs_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 20, names
    for required in ("igs_project_fwd", "igs_project_bwd", "igs_cumsum", "igs_sort_intersects", "igs_raster_fwd_topk",
                     "igs_raster_bwd_topk", "igs_quantize_ste", "igs_rate_fwd", "igs_rate_bwd", "igs_l1_loss", "igs_loo_loss_increase"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/igs_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_host_queries():
    lib = _lib.load()
    c = _lib.constants()
    assert c == dict(tile=16, top_k=10, max_channels=12, eps=1e-4)
    assert lib.igs_version() >= 1
    assert lib.igs_sort_workspace(1000, 16, 16) >= 1000 * 4 + 256 * 4
    assert lib.igs_sort_workspace(0, 16, 16) >= 256 * 4
    assert lib.igs_l1_workspace(1 << 20) > 0
    assert lib.igs_rate_workspace(4000) >= 4 * 16


def test_invalid_arguments_rejected_on_host():
    lib = _lib.load()
    null, fake = None, ctypes.c_void_p(256)  # fake: a non-null pointer the host checks reject before any use
    assert lib.igs_project_fwd(-1, null, null, null, 8, 8, 1, 1, null, null, null, null, null) == 1
    assert "negative" in lib.igs_last_error().decode()
    assert lib.igs_raster_fwd_topk(1, 1, 16, 16, 13, null, null, null, null, null, null, fake, null) == 1
    assert "channels" in lib.igs_last_error().decode()
    assert lib.igs_raster_fwd_topk(2, 1, 16, 16, 3, null, null, null, null, null, null, fake, null) == 1
    assert "tile grid" in lib.igs_last_error().decode()
    assert lib.igs_raster_fwd_topk_tiles(1, 1, 16, 16, 3, -1, null, null, null, null, null, null, fake, null) == 1
    assert "max_list_len" in lib.igs_last_error().decode()
    assert lib.igs_raster_step_l1(1, 1, 16, 16, 0, 10, null, null, null, null, null, null, 1.0, null, fake, null, null, null, null, null,
                                  0, null) == 1
    assert "channels" in lib.igs_last_error().decode()
    assert lib.igs_raster_step_l1(2, 1, 16, 16, 3, 0, null, null, null, null, null, null, 1.0, null, fake, null, null, null, null, null,
                                  0, null) == 1
    assert "tile grid" in lib.igs_last_error().decode()
    assert lib.igs_raster_step_l1(1, 1, 16, 16, 3, 0, null, null, null, null, null, null, 1.0, null, null, null, null, null, null, null,
                                  0, null) == 1
    assert "null loss" in lib.igs_last_error().decode()
    assert lib.igs_raster_step_l1_band(1, 2, 32, 16, 1, 3, 3, 0, null, null, null, null, null, null, 1.0, null, fake, null, null, null,
                                       null, null, 0, null) == 1
    assert "tile rows" in lib.igs_last_error().decode()
    no_refs = (ctypes.c_int32 * 3)(-1, -1, -1)
    self_ref = (ctypes.c_int32 * 3)(0, 0, 1)  # channel 0 predicting from itself
    as_ptr = lambda a: ctypes.cast(a, ctypes.c_void_p)  # noqa: E731
    assert lib.igs_rate_model(10, 3, *([fake] * 4), as_ptr(no_refs), as_ptr(self_ref), *([fake] * 13), 1 << 20, null) == 1
    assert "prediction reference" in lib.igs_last_error().decode()
    assert lib.igs_rate_model(10, 0, *([fake] * 4), as_ptr(no_refs), as_ptr(no_refs), *([fake] * 13), 1 << 20, null) == 1
    assert "channels" in lib.igs_last_error().decode()
    assert lib.igs_bitstream_order(10, fake, 40, fake, fake, 1 << 20, null) == 1
    assert "refine_bits" in lib.igs_last_error().decode()
    assert lib.igs_bitstream_order(-1, fake, 0, fake, fake, 1 << 20, null) == 1
    assert "negative" in lib.igs_last_error().decode()
    assert lib.igs_bitstream_order(0, null, 0, null, null, 0, null) == 0  # nothing to order
    assert lib.igs_sort_intersects(10, 100, null, null, null, 4, 4, null, null, null, 0, null) == 1
    assert lib.igs_quantize_ste(10, 3, null, null, null, null, null, 0.0, 0.1, null, null, null, null, null, null, null, null, null, null,
                                null, null) == 1
    crefs = (ctypes.c_int32 * 3)(0, 5, 0)
    prefs = (ctypes.c_int32 * 3)(0, 1, 2)
    assert lib.igs_rate_fwd(1, 3, 1, null, null, ctypes.c_void_p(1), null, null, null, ctypes.cast(crefs, ctypes.c_void_p),
                            ctypes.cast(prefs, ctypes.c_void_p), null, null, null, 1.0, 1.0, 1.0, ctypes.c_void_p(1), ctypes.c_void_p(1),
                            null, null, ctypes.c_void_p(1), 1 << 20, null) == 1


def test_python_layer_rejects_cpu_tensors():
    x = torch.zeros(4, 2)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.project_gaussians_2d_scale_rot_forward(4, x, x, torch.zeros(4, 1), 16, 16, (1, 1, 1))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.l1_loss_and_grad(torch.zeros(3, 4, 4), torch.zeros(3, 4, 4))


def test_gsplat_shim_exposes_reference_names():
    import gsplat
    import gsplat.cuda
    import gsplat.utils

    for name in ("compute_cumulative_intersects", "project_gaussians_2d_scale_rot", "rasterize_gaussians_sum"):
        assert callable(getattr(gsplat, name))  # model.py:45-51
    for name in ("nd_rasterize_forward_topk_norm", "rate_loss_forward", "rate_loss_backward", "topk_norm_loo_loss_increase",
                 "nd_rasterize_backward_topk_norm", "project_gaussians_2d_scale_rot_forward", "project_gaussians_2d_scale_rot_backward",
                 "sort_intersects_by_tile"):
        assert callable(getattr(gsplat.cuda, name))  # model.py, compress/rate.py:17, compress/pruning.py:10
    assert callable(gsplat.utils.sort_intersects_by_tile)
    with pytest.raises(NotImplementedError):
        gsplat.rasterize_gaussians_sum(None, None, None, None, torch.zeros(1, 3), 4, 4, topk_norm=False)
    with pytest.raises(NotImplementedError):
        gsplat.cuda.nd_rasterize_forward()
