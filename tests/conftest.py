import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    data = np.load(ROOT / "tests" / "golden" / "pair_model_cases.npz")
    cases = {}
    for name in data["names"]:
        name = str(name)
        cases[name] = {f: data[f"{name}.{f}"] for f in ("q", "k", "v", "out", "scale")}
    return cases
