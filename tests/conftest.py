import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        with np.load(ROOT / "tests" / "golden" / f"{name}.npz") as z:
            out = {}
            for key in z.files:
                rec, field = key.rsplit("/", 1)
                out.setdefault(rec, {})[field] = z[key]
            return out
    return load
