"""
Image-GS's own training code against the drop-in gsplat package, on the CPU: the reference's model.py, compress/rate.py and
compress/pruning.py are imported unchanged, in a fresh interpreter whose sys.path puts image-gs_b200/ (this repository's gsplat) first,
with stand-ins for the third-party packages that are absent here and that the rasterization path does not use (fused_ssim, lpips,
pytorch_msssim, matplotlib, flip_evaluator, imageio) and with the reference's own C++ modules (igs_rans, igs_prediction) built from its
sources into oracle/_ref by oracle/build_ref.py. The test checks that
  * every gsplat name those modules import resolves to this repository's implementation, and
  * every call of those names in their source (found with ast) binds to this repository's function signature, positional and keyword
    arguments alike.
Running the calls needs a GPU: tests/test_gpu_ops.py replays model.forward's calls and tests/test_gpu_model_step.py its CUDA-graph
training step through the same package. Skipped where the reference tree is not available (it is read here only, never on a GPU box).
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

PRELUDE = r'''
import ast, importlib.abc, importlib.machinery, inspect, json, os, sys, types

root, pkg, ref, out_dir = sys.argv[1:5]
sys.path[:0] = [out_dir, pkg, ref]

STUBBED = {"fused_ssim", "lpips", "pytorch_msssim", "matplotlib", "flip_evaluator", "imageio"}


class _Anything:
    def __init__(self, *a, **k):
        pass

    def __call__(self, *a, **k):
        return _Anything()

    def __getattr__(self, name):
        return _Anything()

    def __getitem__(self, key):
        return _Anything()

    def __setitem__(self, key, value):
        pass


class _StubLoader(importlib.abc.Loader):
    def create_module(self, spec):
        m = types.ModuleType(spec.name)
        m.__path__ = []

        def attr(name):
            if name.startswith("__"):
                raise AttributeError(name)
            return _Anything()

        m.__getattr__ = attr
        return m

    def exec_module(self, module):
        pass


class _StubFinder(importlib.abc.MetaPathFinder):
    def find_spec(self, name, path, target=None):
        if name.split(".")[0] in STUBBED:
            return importlib.machinery.ModuleSpec(name, _StubLoader(), is_package=True)
        return None


sys.meta_path.insert(0, _StubFinder())

import gsplat, gsplat.cuda, gsplat.utils  # this repository's package
assert os.path.realpath(gsplat.__file__).startswith(os.path.realpath(pkg)), gsplat.__file__
'''

BIND = r'''
modules = {"model": os.path.join(ref, "model.py"), "compress.rate": os.path.join(ref, "compress", "rate.py"),
           "compress.pruning": os.path.join(ref, "compress", "pruning.py")}
report = {"resolved": [], "calls": []}
for modname, path in modules.items():
    mod = __import__(modname, fromlist=["_"])
    tree = ast.parse(open(path).read())
    imported = {}
    for node in ast.walk(tree):
        if isinstance(node, ast.ImportFrom) and node.module and node.module.split(".")[0] == "gsplat":
            source = importlib.import_module(node.module)
            for alias in node.names:
                name = alias.asname or alias.name
                ours = getattr(source, alias.name)
                assert getattr(mod, name) is ours, (modname, name)
                assert os.path.realpath(inspect.getsourcefile(inspect.unwrap(ours))).startswith(os.path.realpath(pkg)), (modname, name)
                imported[name] = ours
                report["resolved"].append(f"{modname}.{name}")
    for node in ast.walk(tree):
        if isinstance(node, ast.Call) and isinstance(node.func, ast.Name) and node.func.id in imported:
            if any(isinstance(a, ast.Starred) for a in node.args) or any(k.arg is None for k in node.keywords):
                continue
            sig = inspect.signature(imported[node.func.id])
            sig.bind(*[None] * len(node.args), **{k.arg: None for k in node.keywords})
            report["calls"].append(f"{modname}:{node.lineno}:{node.func.id}")
print(json.dumps(report))
'''


def _reference_ready():
    ref = build_ref.reference_root()
    return (os.path.exists(os.path.join(ref, "model.py")) and all(build_ref.cpp_module_path(n) for n in build_ref.CPP_MODULES))


@pytest.mark.skipif(not _reference_ready(), reason="the reference tree or its C++ modules (oracle/build_ref.py) are not available")
def test_reference_training_code_binds_to_the_dropin_package():
    import json

    ref = build_ref.reference_root()
    proc = subprocess.run([sys.executable, "-c", PRELUDE + BIND, ROOT, os.path.join(ROOT, "image-gs_b200"), ref, build_ref.OUT],
                          capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-3000:]
    report = json.loads(proc.stdout.strip().splitlines()[-1])
    resolved = set(report["resolved"])
    for name in ("model.project_gaussians_2d_scale_rot", "model.rasterize_gaussians_sum", "model.compute_cumulative_intersects",
                 "model.nd_rasterize_forward_topk_norm", "model.sort_intersects_by_tile", "compress.rate.rate_loss_forward",
                 "compress.rate.rate_loss_backward", "compress.pruning.topk_norm_loo_loss_increase"):
        assert name in resolved, name
    called = {c.split(":")[0] + "." + c.split(":")[2] for c in report["calls"]}
    for name in ("model.project_gaussians_2d_scale_rot", "model.rasterize_gaussians_sum", "compress.pruning.topk_norm_loo_loss_increase",
                 "compress.rate.rate_loss_forward"):
        assert name in called, (name, sorted(called))


CODEC = r'''
import numpy as np

import compress
import compress.quantization
import model
from igs_b200 import bitstream

originals = {"encode": compress.encode_bitstream, "decode": compress.decode_bitstream}
replaced = bitstream.install()
assert model.encode_bitstream is bitstream.encode_bitstream and model.decode_bitstream is bitstream.decode_bitstream
assert model.bitstream_order is bitstream.bitstream_order and compress.quantization.estimate_bits is bitstream.estimate_bits
assert compress.encode_bitstream is bitstream.encode_bitstream and compress.estimate_bits is bitstream.estimate_bits
rng = np.random.default_rng(5)
n = 700
attrs = [(rng.integers(0, 4096, (n, 2)), np.full(2, 0.125), np.zeros(2)), (rng.integers(-40, 8, (n, 2)), np.full(2, 0.03125), np.zeros(2)),
         (rng.integers(-128, 128, (n, 1)), np.full(1, np.float32(np.pi / 256)), np.zeros(1)),
         (rng.integers(-200, 200, (n, 3)), np.full(3, 1 / 64), np.zeros(3))]
ours = model.encode_bitstream(attrs, b"meta", channel_refs=[None, None, None, [1, -1, 1]])
ref = originals["encode"](attrs, b"meta", channel_refs=[None, None, None, [1, -1, 1]])
assert ours[0] == ref[0] and np.array_equal(ours[1], ref[1]) and ours[2] == ref[2]
decoded, meta = model.decode_bitstream(ref[0])
expected, _ = originals["decode"](ours[0])
assert meta == b"meta" and all(np.array_equal(a[0], b[0]) for a, b in zip(decoded, expected))
bitstream.restore(replaced)
assert model.encode_bitstream is originals["encode"]
print("ok")
'''


@pytest.mark.skipif(not _reference_ready(), reason="the reference tree or its C++ modules (oracle/build_ref.py) are not available")
def test_reference_codec_calls_route_to_the_library():
    """bitstream.install() replaces the names model.py and compress/quantization.py bound from compress; a bitstream written through
    model.encode_bitstream afterwards is byte-identical to the replaced encoder's, and each side decodes the other's."""
    ref = build_ref.reference_root()
    proc = subprocess.run([sys.executable, "-c", PRELUDE + CODEC, ROOT, os.path.join(ROOT, "image-gs_b200"), ref, build_ref.OUT],
                          capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert proc.returncode == 0, proc.stderr[-3000:]
    assert proc.stdout.strip().splitlines()[-1] == "ok"
