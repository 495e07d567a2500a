import os
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA devices")
    config.addinivalue_line("markers", "autograd: runs with gradient recording on (all other tests run the "
                                       "layers as inference, under torch.no_grad)")


@pytest.fixture(autouse=True)
def _inference_unless_autograd(request):
    """The layers are nn.Modules whose parameters require gradients, so with gradient
    recording on their outputs carry a graph (as torch's own layers do).  Tests that only
    read forward outputs run under torch.no_grad; autograd tests opt out."""
    if request.node.get_closest_marker("autograd"):
        yield
    else:
        with torch.no_grad():
            yield


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"
