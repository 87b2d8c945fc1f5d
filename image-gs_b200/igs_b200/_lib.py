"""
ctypes binding of libigs_b200.so (the C ABI declared in include/igs_b200.h). The library is required: importing the ops without it, or
calling them without a CUDA device, raises instead of falling back to any other implementation.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("IGS_B200_LIB", os.path.join(_HERE, "libigs_b200.so"))

c_int, c_float, c_double, c_size_t, c_int64, c_void_p = (ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_size_t, ctypes.c_int64,
                                                         ctypes.c_void_p)
P = c_void_p  # device pointers and the stream

# name -> (restype, argtypes); the order follows include/igs_b200.h
SIGNATURES = {
    "igs_last_error": (ctypes.c_char_p, []),
    "igs_version": (c_int, []),
    "igs_constants": (c_int, [ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_double)]),
    "igs_project_fwd": (c_int, [c_int, P, P, P, c_int, c_int, c_int, c_int, P, P, P, P, P]),
    "igs_project_bwd": (c_int, [c_int, P, P, c_int, c_int, P, P, P, P, P, P, P, P, P]),
    "igs_cumsum_workspace": (c_size_t, [c_int]),
    "igs_cumsum": (c_int, [c_int, P, P, P, P, c_size_t, P]),
    "igs_sort_workspace": (c_size_t, [c_int, c_int, c_int]),
    "igs_sort_intersects": (c_int, [c_int, c_int, P, P, P, c_int, c_int, P, P, P, c_size_t, P]),
    "igs_sort_intersects_noalloc": (c_int, [c_int, c_int, P, P, P, c_int, c_int, P, P, P]),
    "igs_raster_fwd_topk": (c_int, [c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P]),
    "igs_raster_fwd_topk_tiles": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P]),
    "igs_raster_l1_workspace": (c_size_t, [c_int]),
    "igs_raster_fwd_topk_tiles_l1": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, c_float, P, P, P, P, P, c_size_t, P]),
    "igs_raster_bwd_topk": (c_int, [c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P]),
    "igs_raster_bwd_topk_tiles": (c_int, [c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P]),
    "igs_raster_step_l1": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, c_float, P, P, P, P, P, P, P, c_size_t,
                                   P]),
    "igs_raster_step_l1_band": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, c_float, P, P, P,
                                        P, P, P, P, c_size_t, P]),
    "igs_train_step_workspace": (c_size_t, [c_int, c_int, c_int, c_int]),
    "igs_train_step_l1": (c_int, [c_int, c_int, P, P, P, P, P, c_float, c_int, c_int, c_int, c_int, c_int] + [P] * 18 + [c_size_t, P]),
    "igs_band_tiles_hit": (c_int, [c_int, P, P, c_int, c_int, c_int, c_int, P, P]),
    "igs_sort_intersects_band": (c_int, [c_int, c_int, P, P, P, c_int, c_int, c_int, c_int, P, P, P, c_size_t, P]),
    "igs_raster_fwd_topk_tiles_band": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P]),
    "igs_raster_fwd_topk_tiles_l1_band": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, c_float, P, P, P,
                                                  P, P, c_size_t, P]),
    "igs_raster_bwd_topk_tiles_band": (c_int, [c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P]),
    "igs_rans_payload_bound": (c_size_t, [c_int, c_int64]),
    "igs_rans_encode": (c_int, [c_int, c_int64, P, c_int, P, c_size_t, ctypes.POINTER(c_size_t), P, P, P]),
    "igs_rans_decode": (c_int, [c_int, c_int64, P, P, P, c_size_t, P]),
    "igs_estimate_bits_workspace": (c_size_t, [c_int]),
    "igs_estimate_stream_bits": (c_int, [c_int, c_int64, P, P, P, c_size_t, P]),
    "igs_ipc_export": (c_int, [P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "igs_ipc_open": (c_int, [P, ctypes.c_uint64, ctypes.POINTER(c_void_p)]),
    "igs_ipc_close": (c_int, [P, ctypes.c_uint64]),
    "igs_band_sync_bytes": (c_size_t, []),
    "igs_band_results_floats": (c_size_t, [c_int, c_int]),
    "igs_band_reduce": (c_int, [c_int, c_int, c_int, c_int, P, P, P, P, P, c_int, c_int, P, P, c_int, P]),
    "igs_loo_loss_increase": (c_int, [c_int, c_int, c_int, c_int, P, P, P, P, P, c_int, c_float, P, P]),
    "igs_feature_weights": (c_int, [c_int, c_int, c_int, P, P, P, c_double, P, P]),
    "igs_neighbors_workspace": (c_size_t, [c_int]),
    "igs_nearest_neighbors": (c_int, [c_int, P, c_int, P, P, P, c_size_t, P]),
    "igs_l1_workspace": (c_size_t, [c_int64]),
    "igs_l1_loss": (c_int, [c_int64, P, P, c_float, P, P, P, c_size_t, P]),
    "igs_l1_loss_signs": (c_int, [c_int64, P, P, c_float, P, P, P, c_size_t, P]),
    "igs_l1_grad_from_signs": (c_int, [c_int64, P, P, P, P]),
    "igs_quantize_ste": (c_int, [c_int, c_int, P, P, P, P, P, c_float, c_float, P, P, P, P, P, P, P, P, P, P, P, P]),
    "igs_feat_transform_bwd": (c_int, [c_int, c_int, P, P, P, P, P]),
    "igs_bitstream_order_workspace": (c_size_t, [c_int]),
    "igs_bitstream_order": (c_int, [c_int, P, c_int, P, P, c_size_t, P]),
    "igs_rate_model_workspace": (c_size_t, [c_int]),
    "igs_rate_model": (c_int, [c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, c_size_t, P]),
    "igs_rate_workspace": (c_size_t, [c_int]),
    "igs_rate_fwd": (c_int, [c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P, P, c_float, c_float, c_float, P, P, P, P, P, c_size_t,
                             P]),
    "igs_rate_bwd": (c_int, [c_int, c_int, P, P, P, P, P, P, P, P, P, P]),
}

# status codes of include/igs_b200.h
IGS_OK, IGS_ERR_INVALID, IGS_ERR_CUDA, IGS_ERR_UNSUPPORTED = 0, 1, 2, 3

_lib = None


def load():
    """The loaded library (ctypes.CDLL with typed entry points). Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"igs_b200 CUDA library not found at {LIB_PATH}; build it with `python image-gs_b200/build.py` "
                          "(the package has no CPU or PyTorch fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


class IgsError(RuntimeError):
    pass


def check(status, what=""):
    if status != 0:
        msg = load().igs_last_error().decode(errors="replace")
        raise IgsError(f"{what or 'igs_b200'} failed (status {status}): {msg}")


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def constants():
    tile, top_k, max_c, eps = c_int(), c_int(), c_int(), c_double()
    check(load().igs_constants(ctypes.byref(tile), ctypes.byref(top_k), ctypes.byref(max_c), ctypes.byref(eps)), "igs_constants")
    return dict(tile=tile.value, top_k=top_k.value, max_channels=max_c.value, eps=eps.value)
