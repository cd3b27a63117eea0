import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

# A local checkout of the reference project, for the CPU tests that import it: $PQ_REFERENCE_DIR,
# else a checkout named "reference" beside this repository.  Absent on GPU hosts (those tests skip).
REFERENCE = Path(os.environ["PQ_REFERENCE_DIR"]) if os.environ.get("PQ_REFERENCE_DIR") else REPO.parent / "reference"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU check")


def reference_available() -> bool:
    return (REFERENCE / "prismaquant" / "format_registry.py").exists()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(REPO / "tests" / "golden" / "small_cases.npz", allow_pickle=False))


@pytest.fixture(scope="session")
def full_digests():
    import json
    with open(REPO / "tests" / "golden" / "full_digests.json") as f:
        return json.load(f)
