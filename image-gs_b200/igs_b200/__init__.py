"""
igs_b200: Image-GS's per-step 2D Gaussian rasterization on B200 (sm_100a), hand-written CUDA behind the C ABI of include/igs_b200.h.

Layers: _lib (ctypes binding, no fallback), ops (tensor operators with the reference's pybind signatures), autograd (differentiable
operators), pipeline (a preallocated, CUDA-graph-captured training step), workloads (seeded synthetic inputs), bands (tile-row sharding of
one image over several GPUs). The drop-in `gsplat` package next to this one exposes the reference's Python surface on top of these.
"""
from ._lib import IgsError, LIB_PATH, constants, load  # noqa: F401

__version__ = "0.1.0"
