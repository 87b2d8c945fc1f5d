"""
Generates the golden fixtures of tests/golden/ from the reference's own CUDA extension (built from its sources by oracle/build_ref.py
into oracle/_ref) on a GPU: seeded inputs -> projection -> prefix sum (torch.cumsum, as utils.py) -> sort_intersects_by_tile ->
nd_rasterize_forward_topk_norm -> L1 gradient -> nd_rasterize_backward_topk_norm -> projection backward, plus the leave-one-out kernel.
Small cases are stored whole (the L1 gradient is recomputed by the tests from image and target); large ones as SHA-256 digests of the
integer outputs, 16x512 crops of the image and top-K lists, the first 1000 Gaussians' values and summary statistics.

Usage (on a GPU machine with oracle/_ref built): python tests/golden/make_golden_ref.py [OUT_DIR, default tests/golden]
"""
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, os.path.join(ROOT, "image-gs_b200"), os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from common import digest, np_, reference_stages  # noqa: E402
from igs_b200 import workloads  # noqa: E402
from oracle import build_ref  # noqa: E402

FULL = {
    "ragged_120x88": dict(h=88, w=120, n=300, seed=11),
    "c9_80x64": dict(h=64, w=80, n=200, c=9, seed=13),
    "c12_40x48": dict(h=48, w=40, n=120, c=12, seed=14),
    "big_64x64": dict(h=64, w=64, n=400, log_scale_mean=math.log(20.0), log_scale_std=0.3, seed=16),
    "aniso_200x100": dict(h=100, w=200, n=600, max_anisotropy=8.0, log_scale_std=0.8, seed=15),
}
LARGE = ["cfg1_256", "cfg3_1080p"]
INT_KEYS = ("radii", "num_tiles_hit", "cum", "gaussian_ids_sorted", "tile_bins", "pixel_topk")
FLOAT_KEYS = ("xys", "conics", "image", "v_xy", "v_conic", "v_colors", "v_cov2d", "v_mean2d", "v_scale", "v_rot")


def l1_grad(image, target):
    # F.l1_loss(image, target).backward(): sign(image - target) / numel
    return (torch.sign(image - target) * (1.0 / image.numel())).contiguous()


def run(ref, wl, inp, capacity=None):
    d = {k: v.cuda() for k, v in inp.items()}
    first = reference_stages(ref, d, wl.height, wl.width, capacity=capacity)
    v_out = l1_grad(first["image"], d["target"])
    out = reference_stages(ref, d, wl.height, wl.width, capacity=capacity, v_output=v_out)
    loo_abs = ref.topk_norm_loo_loss_increase(wl.height, wl.width, out["xys"], out["conics"], d["features"], out["pixel_topk"], d["target"],
                                              False, 1e-4)
    loo_sq = ref.topk_norm_loo_loss_increase(wl.height, wl.width, out["xys"], out["conics"], d["features"], out["pixel_topk"], d["target"],
                                             True, 1e-4)
    out.update(loo_abs=loo_abs, loo_sq=loo_sq)
    torch.cuda.synchronize()
    return out


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    ref = build_ref.load_module()
    for name, kw in FULL.items():
        kw = dict(kw)
        h, w = kw.pop("h"), kw.pop("w")
        n = kw.pop("n")
        c = kw.pop("c", 3)
        wl = workloads.custom_workload(h, w, n, c, seed=kw.pop("seed"), **kw)
        inp = workloads.make_inputs(wl)
        out = run(ref, wl, inp)
        arrays = {k: np_(out[k]) for k in INT_KEYS + FLOAT_KEYS + ("loo_abs", "loo_sq")}
        arrays.update({f"in_{k}": v.numpy() for k, v in inp.items()})
        arrays["meta"] = np.array([h, w, n, c, out["num_intersects"]], dtype=np.int64)
        arrays["input_digest"] = np.array(workloads.input_digest(inp))
        np.savez_compressed(os.path.join(out_dir, f"ref_{name}.npz"), **arrays)
        print(name, out["num_intersects"])
    for name in LARGE:
        wl = workloads.get_workload(name)
        inp = workloads.make_inputs(wl)
        out = run(ref, wl, inp)
        half = run(ref, wl, inp, capacity=out["num_intersects"] // 2)
        arrays = {f"digest_{k}": np.array(digest(out[k])) for k in INT_KEYS + ("xys", "conics", "image")}
        arrays.update({f"half_digest_{k}": np.array(digest(half[k])) for k in ("gaussian_ids_sorted", "tile_bins", "pixel_topk")})
        arrays["image_crop"] = np_(out["image"])[:, :16, :512]
        arrays["pixel_topk_crop"] = np_(out["pixel_topk"])[:16, :512]
        for k in ("xys", "conics", "radii", "num_tiles_hit", "v_xy", "v_conic", "v_colors", "v_scale", "v_rot", "v_mean2d", "loo_abs"):
            arrays[f"first1000_{k}"] = np_(out[k])[:1000]
        for k in ("image", "v_xy", "v_conic", "v_colors", "v_scale", "v_rot"):
            a = np_(out[k]).astype(np.float64)
            arrays[f"stats_{k}"] = np.array([a.sum(), np.abs(a).sum(), (a * a).sum()])
        arrays["meta"] = np.array([wl.height, wl.width, wl.num_gaussians, wl.channels, out["num_intersects"]], dtype=np.int64)
        arrays["input_digest"] = np.array(workloads.input_digest(inp))
        np.savez_compressed(os.path.join(out_dir, f"ref_{name}.npz"), **arrays)
        print(name, out["num_intersects"])


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
