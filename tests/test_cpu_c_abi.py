"""
The C ABI from plain C: tests/c_abi/abi_check.c is compiled with the system C compiler against include/igs_b200.h, linked with
libigs_b200.so and run (constants, workspace sizes, host-side argument checks; no GPU needed).
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_DIR = os.path.join(ROOT, "image-gs_b200", "igs_b200")


def test_c_caller(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    if not os.path.exists(os.path.join(LIB_DIR, "libigs_b200.so")):
        pytest.skip("library not built")
    exe = str(tmp_path / "abi_check")
    cuda_include = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I", cuda_include,
                    os.path.join(ROOT, "tests", "c_abi", "abi_check.c"), "-L", LIB_DIR, "-ligs_b200", f"-Wl,-rpath,{LIB_DIR}", "-o", exe],
                   check=True)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr + out.stdout
    assert out.stdout.count("ok:") == 10
