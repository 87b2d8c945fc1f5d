"""
Test infrastructure, not product code: builds the reference's own gsplat CUDA extension from its sources, unmodified, into oracle/_ref/, so
that GPU tests and the golden-vector script can run the reference kernels beside ours on the same B200 and compare bit for bit.

Recipe (our own, not the reference's setup.py): torch.utils.cpp_extension compiles every gsplat/gsplat/cuda/csrc/*.cu and ext.cpp where they
lie under the reference tree, with the flags of gsplat/setup.py:45-80 (-O3 --use_fast_math --expt-relaxed-constexpr for nvcc, -O3 for the
host compiler, the vendored glm on the include path), for sm_100a. Objects and the module go to oracle/_ref/ only; the reference tree is
read-only. The resulting module is named gsplat_ref_csrc and exposes the reference's pybind functions (gsplat/gsplat/cuda/csrc/ext.cpp:4-32).

Usage: python oracle/build_ref.py [REFERENCE_ROOT]. The reference tree is the argument, else $IGS_REFERENCE_ROOT, else this recipe's
default location (DEFAULT_REFERENCE_ROOT). Needs nvcc, no GPU.
"""
import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
MODULE = "gsplat_ref_csrc"
DEFAULT_REFERENCE_ROOT = "/root/reference"  # where the build container mounts the reference tree; the GPU machine has none


def reference_root(given=None):
    """The reference tree: the given path, else $IGS_REFERENCE_ROOT, else DEFAULT_REFERENCE_ROOT."""
    return given or os.environ.get("IGS_REFERENCE_ROOT") or DEFAULT_REFERENCE_ROOT


def built_module_path():
    """Path of the built reference module, or None if it has not been built."""
    hits = glob.glob(os.path.join(OUT, MODULE + "*.so"))
    return hits[0] if hits else None


def build(root=None, verbose=False):
    csrc = os.path.join(reference_root(root), "gsplat", "gsplat", "cuda", "csrc")
    if not os.path.isdir(csrc):
        raise FileNotFoundError(f"reference CUDA sources not found at {csrc}")
    os.makedirs(OUT, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from torch.utils.cpp_extension import load

    sources = sorted(glob.glob(os.path.join(csrc, "*.cu"))) + sorted(glob.glob(os.path.join(csrc, "*.cpp")))
    load(
        name=MODULE,
        sources=sources,
        extra_include_paths=[os.path.join(csrc, "third_party", "glm")],
        extra_cflags=["-O3", "-Wno-sign-compare"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "--expt-relaxed-constexpr",
                           "-gencode=arch=compute_100a,code=sm_100a"],
        build_directory=OUT,
        verbose=verbose,
        is_python_module=True,
    )
    return built_module_path()


def load_module():
    """Import the built reference module (raises ImportError when oracle/_ref holds no build)."""
    path = built_module_path()
    if path is None:
        raise ImportError("reference extension not built (python oracle/build_ref.py)")
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    spec = importlib.util.spec_from_file_location(MODULE, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


PREDICTION = "igs_prediction"
RANS = "igs_rans"
# the reference's two pybind11 modules of compress/csrc (compress/csrc/setup.py:22-28): module name -> source file
CPP_MODULES = {PREDICTION: "prediction.cpp", RANS: "rans.cpp"}


def cpp_module_path(name):
    """Path of one of the reference's C++ modules built into oracle/_ref, or None."""
    hits = glob.glob(os.path.join(OUT, name + "*.so"))
    return hits[0] if hits else None


def prediction_module_path():
    """Path of the reference's C++ prediction module built into oracle/_ref, or None."""
    return cpp_module_path(PREDICTION)


def build_cpp_module(name, root=None):
    """Compiles one of the reference's compress/csrc modules where it lies, with g++ and compress/csrc/setup.py's flags (-O3
    -ffp-contract=off -pthread, and the source hash define that compress/common.py:13-27 checks), into oracle/_ref/: igs_prediction (its
    neighbour search and predictor: the CPU baseline and checker of the GPU neighbour search) and igs_rans (its rANS coder, which
    compress/__init__.py imports, so that the reference's model.py can be imported here)."""
    import hashlib
    import subprocess
    import sysconfig

    from torch.utils.cpp_extension import include_paths

    src = os.path.join(reference_root(root), "compress", "csrc", CPP_MODULES[name])
    if not os.path.exists(src):
        raise FileNotFoundError(src)
    os.makedirs(OUT, exist_ok=True)
    with open(src, "rb") as f:
        digest = hashlib.sha256(f.read()).hexdigest()[:16]
    out = os.path.join(OUT, name + sysconfig.get_config_var("EXT_SUFFIX"))
    gxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
    subprocess.run([gxx, "-O3", "-std=c++17", "-shared", "-fPIC", "-pthread", "-ffp-contract=off", f'-DSOURCE_HASH="{digest}"', "-I",
                    include_paths()[0], "-I", sysconfig.get_paths()["include"], src, "-o", out], check=True)
    return out


def build_prediction(root=None):
    return build_cpp_module(PREDICTION, root)


def load_cpp_module(name):
    """Import one of the built C++ modules (raises ImportError when it has not been built)."""
    path = cpp_module_path(name)
    if path is None:
        raise ImportError(f"reference module {name} not built (python oracle/build_ref.py)")
    import importlib.util

    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def load_prediction():
    """Import the built prediction module (raises ImportError when it has not been built)."""
    return load_cpp_module(PREDICTION)


if __name__ == "__main__":
    root = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    print(build(root, verbose=True))
    for name in CPP_MODULES:
        print(build_cpp_module(name, root))
