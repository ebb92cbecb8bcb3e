import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
os.environ.setdefault("MINT_LOG_LEVEL", "WARNING")
# trainers built by the tests must not write wandb run folders into the working tree
os.environ.setdefault("WANDB_MODE", "disabled")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def _cuda_ok() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_ok():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


REF = ROOT / "baseline" / "_ref"


@pytest.fixture(scope="session")
def reference_mint():
    """The reference package (read-only install under baseline/_ref), or skip."""
    if not (REF / "mint").exists():
        pytest.skip("reference not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import mint  # noqa: F401

    return mint
