import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from oracle import oracle as _oracle  # noqa: E402

_oracle.build()

GOLDEN = ROOT / "tests" / "golden" / "blocks.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def golden_more():
    """F16, Q4_0, Q4_1, Q5_1, Q5_K, MXFP4 (tests/golden/make_golden.py, main_more)."""
    return dict(np.load(GOLDEN.with_name("blocks_more.npz")))


@pytest.fixture(scope="session")
def g4():
    import gemma4_kt_b200

    return gemma4_kt_b200


@pytest.fixture(scope="session")
def ctx(g4):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    c = g4.Context(0)
    yield c
    c.close()


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    n = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (n if n > 0 else 1.0))
