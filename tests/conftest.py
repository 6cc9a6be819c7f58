import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def _have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_ctx():
    """One gfd context on cuda:0 for the whole GPU test session."""
    if not _have_gpu():
        pytest.skip("no GPU")
    import torch
    torch.cuda.init()
    import gfd_b200
    ctx = gfd_b200.Context(0)
    yield ctx
    ctx.close()
