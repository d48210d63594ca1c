# SPDX-License-Identifier: Unlicense
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "i.coregistration.opencl_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")
    config.addinivalue_line("markers", "slow: full-size model parity (minutes on CPU)")


@pytest.fixture(scope="session")
def dev():
    import coreg

    d = coreg.Device(0)
    yield d
    d.close()
