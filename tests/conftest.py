import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def built():
    """Builds libsbgen.so, libsbenv.so (cross-compiled for sm_100a) and the oracle in tree."""
    from neurips2026_smart_building_challenge_b200 import build

    build.build_all()
    return True


@pytest.fixture(scope="session")
def scenario_cache(tmp_path_factory, built):
    d = os.environ.get("SB_SCENARIO_CACHE")
    return Path(d) if d else tmp_path_factory.mktemp("sbb")
