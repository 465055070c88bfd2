import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built libinl_cuda.so")
    config.addinivalue_line("markers", "slow: full-size configuration (seconds to minutes)")


def cosine_rows(a, b):
    import numpy as np

    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    num = (a * b).sum(-1)
    den = np.linalg.norm(a, axis=-1) * np.linalg.norm(b, axis=-1)
    return num / np.maximum(den, 1e-300)


@pytest.fixture(scope="session")
def gpu():
    """Skip cleanly when there is no CUDA device; fail loudly when there is one
    but the library is missing (no silent fallback)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import im_not_llm_b200 as inl
    from im_not_llm_b200 import _native

    _native.lib()  # raises when libinl_cuda.so is missing
    return inl
