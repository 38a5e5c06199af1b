import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PACKAGE_DIR = ROOT / "dynamic-quantization_b200"
for path in (ROOT, PACKAGE_DIR, ROOT / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


# The reference, installed unmodified with `pip install --target baseline/_ref`.
REF_DIR = ROOT / "baseline" / "_ref"


@pytest.fixture(scope="session")
def reference_install():
    """Make the installed reference importable as ``anchorkv`` for the rest of the
    session (no module of this repository shares its name); skip when it is not
    installed."""
    if not (REF_DIR / "anchorkv").exists():
        pytest.skip("the reference is not installed in baseline/_ref")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    return REF_DIR


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
