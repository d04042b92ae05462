import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def _cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    """The CUDA backend.  On a GPU box a missing library is a failure, not a skip."""
    if not _cuda_available():
        pytest.skip("no CUDA device")
    import blocktensor_b200 as bt
    bt.load()  # raises if libbt_cuda.so is missing
    return bt


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def ref():
    from oracle import oracle as O
    if not O.ref_available():
        pytest.skip("oracle/_ref/libbtref.so not built (needs the reference source tree)")
    return O.RefLib()
