import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "image-gs_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); runs the igs_b200 kernels")
    config.addinivalue_line("markers", "slow: full-size workloads")


@pytest.fixture(scope="session")
def device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ref_module():
    """The reference's own gsplat extension built from source (oracle/_ref), or skip when it has not been built."""
    from oracle import build_ref

    if build_ref.built_module_path() is None:
        pytest.skip("reference extension not built (python oracle/build_ref.py)")
    return build_ref.load_module()
