import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; parity tests through the C ABI")


@pytest.fixture(scope="session")
def golden():
    import json
    return json.loads((ROOT / "tests" / "golden" / "kquant_golden.json").read_text())


@pytest.fixture(scope="session")
def ctx():
    """One backend context on cuda:0 for the GPU tests."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    from turbocider_b200 import cuda as tcc
    c = tcc.Context(0)
    yield c
    c.close()
