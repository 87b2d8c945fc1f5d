"""
Child process of tests/test_zz_no_alloc.py::test_noalloc_binning_under_several_contexts (run by that test, not collected by pytest).

A host application that embeds this library may run it under CUDA contexts of its own instead of the device's primary context, and the
allocation-free binning's fixed scratch array has a separate address in each context. This script drives the C ABI from plain driver-API
contexts on device 0 (ctypes on libcuda, no torch CUDA state), with every device buffer allocated by the script itself:
  * two contexts created one after the other, then the first made current again;
  * a context destroyed and a new one created in its place (the driver may hand out the same CUcontext handle again);
  * the device's primary context.
In each, igs_sort_intersects_noalloc must give exactly the tile lists of igs_sort_intersects with a workspace of the script's own and of
the CPU oracle's binning. Prints "ok" and exits 0 on success.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, os.path.join(ROOT, "image-gs_b200"), HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

from common import make_case  # noqa: E402
from igs_b200 import _lib  # noqa: E402
from oracle import cpu as orc  # noqa: E402

cu = ctypes.CDLL("libcuda.so.1")
vp, u64, sz = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t


def check(status, what):
    if status != 0:
        raise RuntimeError(f"{what} failed with CUresult {status}")


class Context:
    """A driver-API context on device 0 with the script's own device buffers."""

    def __init__(self, device, primary=False):
        self.handle = vp()
        self.primary = primary
        if primary:
            check(cu.cuDevicePrimaryCtxRetain(ctypes.byref(self.handle), device), "cuDevicePrimaryCtxRetain")
        else:
            check(cu.cuCtxCreate_v2(ctypes.byref(self.handle), 0, device), "cuCtxCreate")
        self.device = device
        self.buffers = []
        self.make_current()

    def make_current(self):
        check(cu.cuCtxSetCurrent(self.handle), "cuCtxSetCurrent")

    def alloc(self, nbytes):
        ptr = u64()
        check(cu.cuMemAlloc_v2(ctypes.byref(ptr), sz(max(int(nbytes), 4))), "cuMemAlloc")
        self.buffers.append(ptr.value)
        return ptr.value

    def upload(self, array):
        a = np.ascontiguousarray(array)
        ptr = self.alloc(a.nbytes)
        check(cu.cuMemcpyHtoD_v2(u64(ptr), a.ctypes.data_as(vp), sz(a.nbytes)), "cuMemcpyHtoD")
        return ptr

    def download(self, ptr, shape, dtype):
        out = np.empty(shape, dtype=dtype)
        check(cu.cuCtxSynchronize(), "cuCtxSynchronize")
        check(cu.cuMemcpyDtoH_v2(out.ctypes.data_as(vp), u64(ptr), sz(out.nbytes)), "cuMemcpyDtoH")
        return out

    def close(self):
        self.make_current()
        for ptr in self.buffers:
            check(cu.cuMemFree_v2(u64(ptr)), "cuMemFree")
        self.buffers = []
        if self.primary:
            check(cu.cuCtxSetCurrent(vp()), "cuCtxSetCurrent")
            check(cu.cuDevicePrimaryCtxRelease_v2(self.device), "cuDevicePrimaryCtxRelease")
        else:
            check(cu.cuCtxDestroy_v2(self.handle), "cuCtxDestroy")


def case(h, w, n, seed):
    wl, inp = make_case(h, w, n, seed=seed)
    xys, radii, _, hits = orc.project_fwd(inp["means"], inp["scales"], inp["rotations"], h, w)
    cum = np.cumsum(hits, dtype=np.int64).astype(np.int32)
    total = int(cum[-1]) if len(cum) else 0
    capacity = total + 19  # padding slots must come back zero
    tiles_x, tiles_y = (w + 15) // 16, (h + 15) // 16
    want_ids, want_bins = orc.sort_intersects(n, capacity, xys, radii, cum, h, w)
    return dict(n=n, capacity=capacity, tiles=(tiles_x, tiles_y), xys=xys, radii=radii, cum=cum, ids=want_ids, bins=want_bins)


def run_in(ctx, lib, c):
    """Both binning entry points in the current context, against the oracle."""
    ctx.make_current()
    xys, radii, cum = ctx.upload(c["xys"]), ctx.upload(c["radii"]), ctx.upload(c["cum"])
    tx, ty = c["tiles"]
    ids = ctx.upload(np.full(c["capacity"], -7, np.int32))
    bins = ctx.upload(np.full((tx * ty, 2), -7, np.int32))
    status = lib.igs_sort_intersects_noalloc(c["n"], c["capacity"], vp(xys), vp(radii), vp(cum), tx, ty, vp(ids), vp(bins), vp(0))
    if status != 0:
        raise RuntimeError(lib.igs_last_error().decode())
    got_ids = ctx.download(ids, (c["capacity"],), np.int32)
    got_bins = ctx.download(bins, (tx * ty, 2), np.int32)
    ws_bytes = lib.igs_sort_workspace(c["capacity"], tx, ty)
    ws = ctx.alloc(ws_bytes)
    ids2, bins2 = ctx.alloc(4 * c["capacity"]), ctx.alloc(8 * tx * ty)
    status = lib.igs_sort_intersects(c["n"], c["capacity"], vp(xys), vp(radii), vp(cum), tx, ty, vp(ids2), vp(bins2), vp(ws),
                                     ws_bytes, vp(0))
    if status != 0:
        raise RuntimeError(lib.igs_last_error().decode())
    ws_ids = ctx.download(ids2, (c["capacity"],), np.int32)
    ws_bins = ctx.download(bins2, (tx * ty, 2), np.int32)
    # integer outputs: bit-exact, as every binning comparison
    np.testing.assert_array_equal(got_ids, ws_ids)
    np.testing.assert_array_equal(got_bins, ws_bins)
    np.testing.assert_array_equal(got_ids, c["ids"])
    np.testing.assert_array_equal(got_bins, c["bins"])


def main():
    check(cu.cuInit(0), "cuInit")
    device = ctypes.c_int()
    check(cu.cuDeviceGet(ctypes.byref(device), 0), "cuDeviceGet")
    lib = _lib.load()
    small, larger = case(88, 120, 300, 11), case(256, 256, 1000, 1001)
    a = Context(device.value)
    run_in(a, lib, larger)
    b = Context(device.value)  # a second context beside the first
    run_in(b, lib, small)
    run_in(a, lib, small)  # back to the first one
    run_in(b, lib, larger)
    a.close()
    c = Context(device.value)  # created after a context was destroyed: possibly the same handle, a new ID
    run_in(c, lib, larger)
    c.close()
    b.close()
    p = Context(device.value, primary=True)
    run_in(p, lib, small)
    p.close()
    print("ok")


if __name__ == "__main__":
    main()
