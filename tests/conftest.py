import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def built_libraries():
    """Builds the oracle and the CUDA engine once (no-ops when up to date)."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    from basalt_b200 import build

    build.build()
    yield


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return ROOT / "tests" / "golden"


@pytest.fixture()
def tmp_weights(tmp_path):
    return tmp_path / "weights.bin"


def gpu_available() -> bool:
    from basalt_b200 import Basalt

    return Basalt.device_count() > 0


@pytest.fixture(scope="session")
def runtime():
    from basalt_b200 import Basalt

    if Basalt.device_count() == 0:
        pytest.fail("GPU tests need a CUDA device; run them with -m gpu on a B200")
    return Basalt.create(int(os.environ.get("BASALT_DEVICE", "0")))
