import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test collected without a CUDA device (run with -m 'not gpu' on CPU hosts)")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"sm_100a kernels need a B200-class device, got sm_{major}{minor}")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def dsl():
    """The reference DSL (pdum.dsl / pdum.tl) from the shimmed copy in baseline/_ref."""
    from oracle.make_ref_shim import ensure_importable

    if not ensure_importable():
        pytest.skip("reference DSL copy not present (python oracle/make_ref_shim.py)")
    import pdum.tl  # noqa: F401

    return True
