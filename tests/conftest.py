"""Test configuration: the ``gpu`` marker and import paths.

``-m "not gpu"`` tests need no GPU (oracle vs golden fixtures, host logic, ABI
export table, gloo multi-process logic).  ``-m gpu`` tests call the CUDA path
through the C ABI and compare it with the oracle.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for p in (str(REPO), str(REPO / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    orc.build()
    return orc


@pytest.fixture(scope="session")
def hb():
    """The product package (loaded from hello-ot_b200/)."""
    import __graft_entry__ as entry
    return entry.load_package()


@pytest.fixture(scope="session")
def cuda(hb):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a gpu-marked test ran without CUDA")
    hb.lib()  # fails loudly when the extension is missing
    return torch.device("cuda", 0)
