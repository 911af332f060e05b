import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def ref_module():
    """The reference's own compiled extension (oracle/_ref), if present."""
    from oracle import build_ref
    if build_ref.built_path() is None:
        pytest.skip("reference extension not built in oracle/_ref")
    return build_ref.load()


@pytest.fixture(scope="session")
def mb():
    import memboost_b200
    return memboost_b200
