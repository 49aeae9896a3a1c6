import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


def pytest_collection_modifyitems(config, items):
    """Skip GPU tests cleanly where no device exists (the CPU suite never selects them)."""
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu or os.environ.get("HELIOS_B200_REQUIRE_GPU"):
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
