import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "whisper.go_b200", ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Build the generator, the oracle and the CUDA library (no-ops when fresh)."""
    import wgbuild
    wgbuild.build_gen()
    wgbuild.build_oracle()
    wgbuild.build_lib()
    yield


@pytest.fixture(scope="session")
def kat():
    import json
    return json.loads((ROOT / "tests" / "golden" / "reference_kat.json").read_text())
