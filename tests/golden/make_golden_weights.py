"""
Generates the golden fixtures of the per-Gaussian feature weights from the reference's own Python code: compress.quantization.
feature_weights (compress/quantization.py:218-230) over model.Image_GS._iter_topk_weights (model.py:1404-1421). model.py cannot be
imported here (it imports fused_ssim, lpips and pytorch_msssim at the top), so the method's source is taken from model.py with `ast`,
compiled as is, and called on a small stand-in for the model object that carries the attributes it reads (img_h, img_w, topk, device,
dtype) and a _get_pixel_topk returning the oracle's projection and top-K lists. Runs on the CPU in float32/float64; the fixtures it writes
are committed.

Usage: python tests/golden/make_golden_weights.py [REFERENCE_ROOT] [OUT_DIR]
"""
import ast
import math
import os
import sys
import tempfile
import types

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "image-gs_b200"), HERE]

import numpy as np  # noqa: E402
import torch  # noqa: E402

from igs_b200 import workloads  # noqa: E402
from make_golden_py import build_cpp_modules  # noqa: E402
from oracle import cpu  # noqa: E402

CASES = {
    "weights_ragged_120x88": dict(h=88, w=120, n=300, seed=11),
    "weights_big_64x64": dict(h=64, w=64, n=400, log_scale_mean=math.log(20.0), log_scale_std=0.3, seed=16),
    "weights_cfg1_256": dict(h=256, w=256, n=1000, seed=1001),
}


def reference_method(ref_root, name):
    """The function object of model.Image_GS.<name>, compiled from model.py's own source."""
    with open(os.path.join(ref_root, "model.py")) as f:
        tree = ast.parse(f.read())
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == name:
            module = ast.Module(body=[node], type_ignores=[])
            namespace = {"torch": torch}
            exec(compile(module, os.path.join(ref_root, "model.py"), "exec"), namespace)
            return namespace[name]
    raise LookupError(name)


def main(ref_root, out_dir):
    ext_dir = build_cpp_modules(ref_root, os.path.join(tempfile.gettempdir(), "igs_ref_ext"))
    for p in (ext_dir, ref_root):
        sys.path.insert(0, p)
    from compress.quantization import feature_weights

    iter_topk_weights = reference_method(ref_root, "_iter_topk_weights")
    for name, kw in CASES.items():
        kw = dict(kw)
        h, w, n = kw.pop("h"), kw.pop("w"), kw.pop("n")
        wl = workloads.custom_workload(h, w, n, 3, kw.get("log_scale_mean", math.log(2.0)), kw.get("log_scale_std", 0.5), seed=kw["seed"])
        inp = workloads.make_inputs(wl)
        r = cpu.train_step(*[inp[k].numpy() for k in ("means", "scales", "rotations", "features", "target")], h, w)
        xys, conics, topk = (torch.from_numpy(np.ascontiguousarray(r[k])) for k in ("xys", "conics", "pixel_topk"))
        stand_in = types.SimpleNamespace(img_h=h, img_w=w, topk=10, device=torch.device("cpu"), dtype=torch.float32,
                                         _get_pixel_topk=lambda *a: (xys, conics, topk))
        weights = feature_weights(iter_topk_weights(stand_in, xys, None, None, None), n, 1e-4, "cpu")
        np.savez_compressed(os.path.join(out_dir, f"py_{name}.npz"), xys=xys.numpy(), conics=conics.numpy(), pixel_topk=topk.numpy(),
                            meta=np.array([h, w, n], dtype=np.int64), weights=weights.numpy())
        print(name, "nonzero", int((weights > 0).sum()), "sum", float(weights.sum()))


if __name__ == "__main__":
    from oracle.build_ref import reference_root

    main(reference_root(sys.argv[1] if len(sys.argv) > 1 else None), sys.argv[2] if len(sys.argv) > 2 else HERE)
