"""
Build of the igs_b200 CUDA library: every image-gs_b200/csrc/*.cu compiled by nvcc for sm_100a and linked into
image-gs_b200/igs_b200/libigs_b200.so (static CUDA runtime, no torch dependency), which the Python package loads with ctypes.

Files whose results must match the reference extension bit for bit (projection, binning, rasterization, rate term, leave-one-out) are
compiled with --use_fast_math like the reference (gsplat/setup.py:70); the quantizer and the L1 loss are IEEE (ATen's arithmetic).

Usage: python image-gs_b200/build.py [--force] [--verbose]. Needs nvcc, no GPU.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "igs_b200")
LIB = os.path.join(OUT_DIR, "libigs_b200.so")
OBJ_DIR = os.path.join(HERE, "_build")

FAST_MATH = {"project.cu", "binning.cu", "raster.cu", "rate.cu", "loo.cu", "exchange.cu"}
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", INCLUDE, "-Xptxas", "-v"]


def nvcc():
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda_home, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    os.makedirs(OBJ_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "igs_b200.h"))
    headers.append(os.path.abspath(__file__))
    objects = []
    log_lines = []
    for name in sources():
        src = os.path.join(CSRC, name)
        obj = os.path.join(OBJ_DIR, name.replace(".cu", ".o"))
        objects.append(obj)
        if not force and not _newer(obj, [src] + headers):
            continue
        flags = COMMON + ARCH + (["--use_fast_math"] if name in FAST_MATH else [])
        cmd = [nvcc(), "-c", src, "-o", obj] + flags
        proc = subprocess.run(cmd, capture_output=True, text=True)
        log_lines.append(f"== {name}\n{proc.stdout}{proc.stderr}")
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError(f"nvcc failed on {name}")
    if force or _newer(LIB, objects):
        cmd = [nvcc(), "-shared", "-o", LIB] + objects + ARCH + ["-Xcompiler", "-fPIC", "-cudart", "static"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            sys.stderr.write(proc.stdout + proc.stderr)
            raise RuntimeError("nvcc link failed")
    if log_lines:
        with open(os.path.join(OBJ_DIR, "ptxas.log"), "a") as f:
            f.write("\n".join(log_lines))
        if verbose:
            print("\n".join(log_lines))
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
