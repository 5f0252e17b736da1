import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    with np.load(ROOT / "tests" / "golden" / "golden_small.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_extra():
    import numpy as np

    with np.load(ROOT / "tests" / "golden" / "golden_extra.npz") as z:
        return {k: z[k] for k in z.files}
