import os
import subprocess
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def _ensure_built():
    """Build the oracle (CPU checker) and the product library if missing.
    The oracle/_ref reference build needs the reference tree and is only
    attempted when it is present."""
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True)
    if not os.path.exists(os.path.join(ROOT, "bnns_to_c_b200", "lib", "libbnn_b200.so")):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "bnns_to_c_b200", "csrc")], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
