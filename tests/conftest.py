import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

# The reference checkout: $HMM_REFERENCE_ROOT, else a directory named
# "reference" beside this repository.  Tests that read it skip when it is absent.
REFERENCE = os.environ.get("HMM_REFERENCE_ROOT") or os.path.join(os.path.dirname(ROOT),
                                                                 "reference")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import heteromm_b200 as hmm
    hmm.load()
    return torch.device("cuda:0")


def reference_checkout_available() -> bool:
    return os.path.isdir(os.path.join(REFERENCE, "toolchain", "frontend", "dev"))
