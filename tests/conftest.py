import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "qwen-3.5-cuda_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_sessionstart(session):
    # the product library and the oracle must exist; build them if this tree
    # was not built yet (nvcc and gcc cross-compile without a GPU)
    from qmoe import build as qbuild
    if not qbuild.LIB.exists():
        qbuild.build()
    from oracle import oracle as orc
    if not orc.LIB.exists():
        orc.build()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
