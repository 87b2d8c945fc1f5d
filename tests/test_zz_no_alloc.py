"""
The allocation-free binning entry point, igs_sort_intersects_noalloc: for callers that cannot call cudaMalloc and have no workspace to lend
(for example a plugin inside a host application that owns all device memory, or code where an allocation would synchronize the device).
It is called here through the C ABI and checked against igs_sort_intersects with a caller-provided workspace, on two calls in a row of
different sizes: both calls use the library's one fixed scratch array, so the second must not see anything the first left in it; and
under several CUDA contexts of one device (the array has one address per context), in a child process.
"""
import ctypes
import os
import re

import pytest
import torch

from common import make_case, to_dev
from igs_b200 import _lib, ops

pytestmark = pytest.mark.gpu

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "igs_b200.h")


def header_constant(name):
    return int(re.search(rf"#define {name} (\d+)", open(HEADER).read()).group(1))


def binning_inputs(h, w, n, seed, device):
    _, inp = make_case(h, w, n, seed=seed)
    d = to_dev(inp, device)
    tb = ops.tile_grid(h, w)
    xys, radii, _, hits = ops.project_gaussians_2d_scale_rot_forward(n, d["means"], d["scales"], d["rotations"], h, w, tb)
    cum, total = ops.cumulative_intersects(hits)
    return tb, xys, radii, cum, int(total.item())


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_binning_matches_workspace_binning(device):
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for h, w, n, seed in ((256, 256, 1000, 1001), (88, 120, 300, 11)):  # two calls in a row
        tb, xys, radii, cum, total = binning_inputs(h, w, n, seed, device)
        capacity = total + 37  # padding slots after the last intersection must come back zero
        ids = torch.full((capacity,), -7, dtype=torch.int32, device=device)
        bins = torch.full((tb[0] * tb[1], 2), -7, dtype=torch.int32, device=device)
        status = lib.igs_sort_intersects_noalloc(n, capacity, ptr(xys), ptr(radii), ptr(cum), tb[0], tb[1], ptr(ids), ptr(bins), stream)
        assert status == 0, lib.igs_last_error().decode()
        want_ids, want_bins = ops.sort_intersects_by_tile(n, capacity, xys, radii, cum, tb)
        torch.cuda.synchronize()
        # integer outputs: the tolerance of every binning test is zero
        assert torch.equal(ids, want_ids)
        assert torch.equal(bins, want_bins)


def test_noalloc_binning_rejects_oversized_requests(device):
    lib = _lib.load()
    tb, xys, radii, cum, _ = binning_inputs(32, 32, 10, 3, device)
    out = torch.zeros(16, dtype=torch.int32, device=device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    too_many = header_constant("IGS_NOALLOC_MAX_CAPACITY") + 1
    assert lib.igs_sort_intersects_noalloc(10, too_many, ptr(xys), ptr(radii), ptr(cum), tb[0], tb[1], ptr(out), ptr(out), stream) == 1
    assert "capacity" in lib.igs_last_error().decode()
    tiles = header_constant("IGS_NOALLOC_MAX_TILES")
    assert lib.igs_sort_intersects_noalloc(10, 16, ptr(xys), ptr(radii), ptr(cum), tiles + 1, 1, ptr(out), ptr(out), stream) == 1
    assert "tiles" in lib.igs_last_error().decode()


def test_noalloc_binning_under_several_contexts(device):
    """The fixed scratch array has one address per CUDA context. A host application may run the library under contexts of its own, or
    destroy a context and create another: the child process drives the C ABI from plain driver-API contexts (two side by side, one
    created after another was destroyed, and the primary one), and every call must match igs_sort_intersects and the CPU oracle."""
    import subprocess
    import sys

    child = os.path.join(os.path.dirname(os.path.abspath(__file__)), "noalloc_contexts_child.py")
    proc = subprocess.run([sys.executable, child], capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0 and proc.stdout.strip().endswith("ok"), proc.stdout[-2000:] + proc.stderr[-4000:]
