import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "ptx-std_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")
    config.addinivalue_line("markers", "slow: long-running CPU check")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def ptxstd_lib():
    """libptxstd.so, built in-tree if missing (nvcc cross-compiles without a GPU)."""
    lib_path = os.path.join(ROOT, "ptx-std_b200", "libptxstd.so")
    if not os.path.exists(lib_path):
        import subprocess
        subprocess.run([sys.executable, os.path.join(ROOT, "ptx-std_b200", "build.py")],
                       check=True)
    import ptxstd
    return ptxstd


@pytest.fixture(scope="session")
def cuda(ptxstd_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    ptxstd_lib.check(ptxstd_lib.lib().ptxstd_device_supported(torch.cuda.current_device()),
                     "device_supported")
    return torch
