import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


def _ensure_ext():
    try:
        import syntropy_b200._C  # noqa: F401
        return
    except ImportError:
        pass
    subprocess.check_call([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=ROOT,
                          stdout=subprocess.DEVNULL)


@pytest.fixture(scope="session", autouse=True)
def native_ext():
    _ensure_ext()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
