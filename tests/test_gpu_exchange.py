"""
The bands' peer-memory exchange (igs_band_reduce) on one GPU, through the C ABI:
  * one rank: the exchange sums its own partials (x + 0 is x) and runs the projection backward on them, so its results must equal
    igs_project_bwd on the same partials bit for bit, and the colour gradients and loss must be the partials themselves;
  * a missing rank: a second rank whose synchronisation words nothing ever writes (a flag that nothing sets, in this GPU's own memory:
    no second process or kernel is involved). The wait must give up after its timeout, record IGS_BAND_TIMEOUT_READY in the rank's error
    word, leave the results untouched, and leave the CUDA context usable; later exchanges on that rank do nothing.
The two-rank exchange across two GPUs is in test_gpu_bands_multi.py.
"""
import ctypes
import time

import pytest
import torch

from common import make_case, to_dev

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def lib_and_bands():
    from igs_b200 import _lib, bands

    return _lib, _lib.load(), bands


def buffers(lib, n, c):
    """A rank's partials, results and zeroed synchronisation words (separate tensors; the kernel takes any addresses)."""
    partials = torch.empty(n * (5 + c) + 1, device=DEV, dtype=torch.float32)
    results = torch.full((int(lib.igs_band_results_floats(n, c)),), -7.0, device=DEV, dtype=torch.float32)
    sync = torch.zeros(int(lib.igs_band_sync_bytes()) // 4, device=DEV, dtype=torch.int32)
    return partials, results, sync


def reduce_call(lib, world, rank, n, c, parts, ress, syncs, step, timeout_ms):
    arr = ctypes.c_void_p * world
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    return lib.igs_band_reduce(world, rank, n, c, arr(*[p.data_ptr() for p in parts]), arr(*[r.data_ptr() for r in ress]),
                               arr(*[s.data_ptr() for s in syncs]), ctypes.c_void_p(step.scales.data_ptr()),
                               ctypes.c_void_p(step.rotations.data_ptr()), step.h, step.w, ctypes.c_void_p(step.radii.data_ptr()),
                               ctypes.c_void_p(step.conics.data_ptr()), timeout_ms, stream)


def band_step(wl, d):
    from igs_b200 import bands

    tiles_y = wl.tile_bounds[1]
    step = bands.BandStep(d["means"], d["scales"], d["rotations"], d["features"], d["target"], wl.height, wl.width, 0, tiles_y)
    step.launch()  # the whole image as one band: partials in step.reduced, the projection backward in v_cov2d ...
    torch.cuda.synchronize()
    return step


def test_single_rank_exchange_equals_projection_backward():
    _lib, lib, bands = lib_and_bands()
    wl, inp = make_case(120, 200, 700, seed=17)
    d = to_dev(inp, DEV)
    step = band_step(wl, d)
    n, c = step.n, step.c
    partials, results, sync = buffers(lib, n, c)
    partials.copy_(step.reduced)
    for rep in range(2):
        _lib.check(reduce_call(lib, 1, 0, n, c, [partials], [results], [sync], step, 5000), "igs_band_reduce")
        torch.cuda.synchronize()
        assert int(sync[bands.SYNC_ERROR]) == 0 and int(sync[bands.SYNC_STEP]) == rep + 1
        got = {"v_cov2d": results[:3 * n], "v_mean2d": results[3 * n:5 * n], "v_scale": results[5 * n:7 * n], "v_rot": results[7 * n:8 * n],
               "v_colors": results[8 * n:(8 + c) * n]}
        for key, val in got.items():
            assert torch.equal(val, getattr(step, key).reshape(-1)), key
        assert torch.equal(results[(8 + c) * n], step.loss)


def test_missing_rank_times_out_and_leaves_the_context_usable():
    _lib, lib, bands = lib_and_bands()
    wl, inp = make_case(64, 96, 200, seed=3)
    d = to_dev(inp, DEV)
    step = band_step(wl, d)
    n, c = step.n, step.c
    mine = buffers(lib, n, c)
    absent = buffers(lib, n, c)  # rank 1: nothing runs for it, so its announcements never come
    mine[0].copy_(step.reduced)
    t0 = time.monotonic()
    _lib.check(reduce_call(lib, 2, 0, n, c, [mine[0], absent[0]], [mine[1], absent[1]], [mine[2], absent[2]], step, 300), "igs_band_reduce")
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 0.25 <= waited < 30.0, waited
    assert int(mine[2][bands.SYNC_ERROR]) & 1  # IGS_BAND_TIMEOUT_READY
    assert int(mine[2][bands.SYNC_STEP]) == 0
    assert bool((mine[1] == -7.0).all()) and bool((absent[1] == -7.0).all())  # no results were stored anywhere
    # this rank's announcement reached rank 1's words (a plain store into memory nobody reads)
    assert int(absent[2][0]) == 1
    # the context still works, and a later exchange on the failed rank returns at once without waiting
    x = torch.arange(1000, device=DEV, dtype=torch.float32)
    assert float(x.sum()) == 499500.0
    t0 = time.monotonic()
    _lib.check(reduce_call(lib, 2, 0, n, c, [mine[0], absent[0]], [mine[1], absent[1]], [mine[2], absent[2]], step, 300), "igs_band_reduce")
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 0.25
    assert bool((mine[1] == -7.0).all())


def test_exchange_rejects_bad_arguments():
    _lib, lib, bands = lib_and_bands()
    wl, inp = make_case(32, 32, 20, seed=1)
    d = to_dev(inp, DEV)
    step = band_step(wl, d)
    p, r, s = buffers(lib, step.n, step.c)
    assert reduce_call(lib, 9, 0, step.n, step.c, [p] * 9, [r] * 9, [s] * 9, step, 100) == _lib.IGS_ERR_INVALID  # more than 8 ranks
    assert reduce_call(lib, 1, 1, step.n, step.c, [p], [r], [s], step, 100) == _lib.IGS_ERR_INVALID  # rank outside the world
    assert reduce_call(lib, 1, 0, step.n, step.c, [p], [r], [s], step, 0) == _lib.IGS_ERR_INVALID  # no timeout
