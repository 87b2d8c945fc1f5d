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

CHILD = r'''
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
    proc = subprocess.run([sys.executable, "-c", CHILD, ROOT, os.path.join(ROOT, "image-gs_b200"), ref, build_ref.OUT],
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
