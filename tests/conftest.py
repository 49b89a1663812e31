"""Shared fixtures.  GPU tests carry @pytest.mark.gpu; everything else runs on
the CPU (no device needed).  The oracle (oracle/) is the checker only."""
import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT / "esm-cpp_b200"), str(ROOT / "oracle"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def O():
    import oracle

    oracle.orc()
    return oracle


@pytest.fixture(scope="session")
def R(O):
    if not O.ref_available():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return O.ref()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def record():
    """record(name, **values): appends one JSON line of measured values (a
    parity test's observed Pearson, error or flip counts) to the file named
    by $ESM_B200_RECORD, when it is set; otherwise does nothing."""
    path = os.environ.get("ESM_B200_RECORD")

    def _record(name, **values):
        if path:
            with open(path, "a") as f:
                f.write(json.dumps({"test": name, **values}) + "\n")

    return _record
