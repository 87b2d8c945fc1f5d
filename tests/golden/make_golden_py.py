"""
Generates the golden fixtures of the quantization and rate term from the reference's own Python code (compress/quantization.py and
compress/rate.py of BaylorMultimediaLab/image-gs), run on the CPU in float32:
  - step symbols and straight-through values (get_step_symbols, dequantize_symbols, x + (q - x)),
  - the rate model (rate_model: causal neighbors in bitstream order through the reference's C++ module igs_prediction, CCLM slopes,
    Laplace scales) and rate_bits with its autograd gradients,
for the 480p YUV workload (4,000 Gaussians, colour references none, prediction references Y <- neighbors, U <- Y, V <- U) and a small RGB
one with subtract-green colour references.

The reference's C++ modules igs_prediction and igs_rans are compiled here from compress/csrc/*.cpp with g++ into a temporary directory
(our recipe; the hash define is what compress/common.py:13-27 checks). Needs the reference tree; the fixtures it writes are committed.

Usage: python tests/golden/make_golden_py.py [REFERENCE_ROOT] [OUT_DIR]
"""
import hashlib
import math
import os
import subprocess
import sys
import sysconfig
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "image-gs_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from igs_b200 import workloads  # noqa: E402


def build_cpp_modules(ref_root, out_dir):
    from torch.utils.cpp_extension import include_paths

    inc = include_paths()[0]
    py_inc = sysconfig.get_paths()["include"]
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    for module, source in (("igs_rans", "rans.cpp"), ("igs_prediction", "prediction.cpp")):
        src = os.path.join(ref_root, "compress", "csrc", source)
        with open(src, "rb") as f:
            digest = hashlib.sha256(f.read()).hexdigest()[:16]
        out = os.path.join(out_dir, module + suffix)
        if not os.path.exists(out):
            subprocess.run([("/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"), "-O3", "-std=c++17", "-shared", "-fPIC", "-pthread", "-ffp-contract=off", f'-DSOURCE_HASH="{digest}"',
                            "-I", inc, "-I", py_inc, src, "-o", out], check=True)
    return out_dir


def quant_case(wl, inp, steps):
    from compress.quantization import dequantize_symbols, get_step_symbols

    xy, scale, rot, feat = inp["means"], inp["scales"].abs(), inp["rotations"], inp["features"]
    symbols = get_step_symbols(xy, scale, rot, feat, steps)
    deq = dequantize_symbols(symbols, log_scale=True)
    values = [x + (q - x) for x, q in zip((xy, scale, rot, feat), deq)]
    return symbols, values


def main(ref_root, out_dir):
    os.makedirs(out_dir, exist_ok=True)
    ext_dir = build_cpp_modules(ref_root, os.path.join(tempfile.gettempdir(), "igs_ref_ext"))
    for p in (ext_dir, ref_root, os.path.join(ref_root, "gsplat")):
        sys.path.insert(0, p)
    from compress.quantization import dequantize, get_channel_refs
    from compress.prediction import get_prediction_refs
    from compress.rate import rate_bits, rate_model

    cases = [("cfg2_480p_yuv", workloads.get_workload("cfg2_480p_yuv"), "yuv"),
             ("rgb_subgreen_320x200", workloads.custom_workload(200, 320, 800, 3, math.log(2.5), 0.5, 6.0, seed=31), "rgb")]
    for name, wl, space in cases:
        inp = workloads.make_inputs(wl)
        pos_step, scale_step, rot_step, feat_step = 0.125, 0.03125, math.radians(0.703125), 0.015625
        steps = [pos_step / torch.tensor([wl.width, wl.height], dtype=torch.float32), torch.full((2,), scale_step, dtype=torch.float32),
                 torch.full((1,), rot_step, dtype=torch.float32), torch.full((wl.channels,), feat_step, dtype=torch.float32)]
        symbols, values = quant_case(wl, inp, steps)
        color_refs = get_channel_refs([3], "none" if space == "yuv" else "subtract-green")[3]
        pred_refs = get_prediction_refs([3], space)
        channel_weights = torch.tensor([1.0, 0.25, 0.25] if space == "yuv" else [1.0, 1.0, 1.0], dtype=torch.float32)
        feat_deq = dequantize(*symbols[3])
        model = rate_model(symbols[0][0].numpy().astype(np.int64), feat_deq, dequantize(*symbols[1]), symbols[2][0][:, 0], color_refs,
                           pred_refs, steps[3], channel_weights, torch.float32, "cpu", 3)
        inv_rot_step = 1.0 / steps[2].item()
        feat = values[3].clone().requires_grad_(True)
        rot = values[2].clone().requires_grad_(True)
        feat_bits, rot_bits = rate_bits(feat, rot, model, inv_rot_step)
        l1, l1_ratio = 0.0625, 1.0
        factor = 0.25 * 57.9 / (2.0 * 255.0 ** 2 * wl.num_pixels)
        weight = factor / max(l1 / l1_ratio, 1e-4)
        loss = weight * (feat_bits + rot_bits)
        loss.backward()
        arrays = dict(
            meta=np.array([wl.height, wl.width, wl.num_gaussians, wl.channels], dtype=np.int64), input_digest=np.array(workloads.input_digest(inp)),
            steps_xy=steps[0].numpy(), scale_step=np.float32(scale_step), rot_step=np.float32(rot_step), feat_steps=steps[3].numpy(),
            q_xy=symbols[0][0].numpy(), q_scale=symbols[1][0].numpy(), q_rot=symbols[2][0].numpy(), q_feat=symbols[3][0].numpy(),
            out_xy=values[0].numpy(), out_scale=values[1].numpy(), out_rot=values[2].detach().numpy(), out_feat=values[3].detach().numpy(),
            neighbors=model.neighbors.numpy(), weights=model.weights.numpy(), slope=model.slope.numpy(), inv_steps=model.inv_steps.numpy(),
            feat_coeffs=model.feat_coeffs.numpy(), inv_rot=model.inv_rot.numpy(), offsets=model.offsets.numpy(), sources=model.sources.numpy(),
            source_weights=model.source_weights.numpy(), color_refs=np.array(model.color_refs, dtype=np.int32),
            pred_channels=np.array(model.pred_channels, dtype=np.int32), inv_rot_step=np.float32(inv_rot_step), l1=np.float32(l1),
            l1_ratio=np.float32(l1_ratio), factor=np.float64(factor), feat_bits=np.float64(feat_bits.item()),
            rot_bits=np.float64(rot_bits.item()), loss=np.float64(loss.item()), grad_feat=feat.grad.numpy(), grad_rot=rot.grad.numpy())
        np.savez_compressed(os.path.join(out_dir, f"py_{name}.npz"), **arrays)
        print(name, "loss", loss.item(), "bits", feat_bits.item(), rot_bits.item())


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    from oracle.build_ref import reference_root

    main(reference_root(sys.argv[1] if len(sys.argv) > 1 else None), sys.argv[2] if len(sys.argv) > 2 else HERE)
