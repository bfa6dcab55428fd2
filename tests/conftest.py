"""Test setup: the package directory `ssengine-glm5.3-flash_b200/` is imported as `ssengine_b200`, the repository
root is on sys.path for the CPU oracle (`oracle/`, test infrastructure), and `-m gpu` tests need a CUDA device."""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

__graft_entry__.import_package()

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device (run with -m 'not gpu' on a CPU box)")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"sm_100a library on a device of capability {major}.{minor}")
    from ssengine_b200 import lib

    lib.load()
    return torch.device("cuda:0")
