import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run on the B200 box)")


def bf16_from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).view(torch.bfloat16)


def load_golden(name: str) -> dict:
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: g[k] for k in g.files}


@pytest.fixture(scope="session")
def built_lib():
    """The in-tree shared library, built on demand (nvcc cross-compiles without a GPU)."""
    from freesolo_b200 import lib
    if not os.path.isfile(lib.LIB_PATH):
        import __graft_entry__ as ge
        ge.build()
    return lib.load()


def gpu_only():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
