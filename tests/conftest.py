import glob
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def golden_files(prefix):
    return sorted(glob.glob(os.path.join(GOLDEN, f"{prefix}_*.npz")))


def load_golden(path):
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def unpack_mask(bits, s):
    return np.unpackbits(bits, axis=-1, count=s).astype(bool)


@pytest.fixture(scope="session")
def cuda_lib():
    """The in-tree CUDA library, for GPU tests only (no fallback)."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from tributary_b200 import _lib
    return _lib.load()
