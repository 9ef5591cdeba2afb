import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def packs():
    return np.load(os.path.join(GOLDEN, "packs.npz"))


@pytest.fixture(scope="session")
def wb():
    """The product binding (requires the built library; GPU tests only)."""
    import welvet.cuda_b200 as W
    W.cuda_init()
    return W


def pack_cases(packs):
    names = sorted({k.rsplit(".", 1)[0] for k in packs.files})
    out = []
    for n in names:
        meta = packs[n + ".meta"]
        dt, rows, cols, sbits = (int(v) for v in meta)
        scale = float(np.array([sbits], dtype=np.uint32).view(np.float32)[0])
        out.append((n, dt, rows, cols, scale, packs[n + ".w"], packs[n + ".raw"], packs[n + ".dec"]))
    return out
