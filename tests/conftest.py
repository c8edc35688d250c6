import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "go-fann_b200"), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


@pytest.fixture(scope="session", autouse=True)
def _oracle_built():
    """The CPU oracle is test infrastructure built from oracle/ (gcc)."""
    if not (ROOT / "oracle" / "liboracle.so").exists():
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "oracle"], check=True)
