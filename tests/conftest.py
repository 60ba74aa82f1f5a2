import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "semantic-ai_b200", ROOT / "oracle", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through libsvl_b200.so)")
    config.addinivalue_line("markers", "slow: full-size model shapes")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle
    oracle.build()
    return oracle.lib()


@pytest.fixture(scope="session")
def svl_lib():
    from svl import _lib
    if not _lib.LIB_PATH.exists():
        sys.path.insert(0, str(ROOT / "semantic-ai_b200"))
        import build as _build
        _build.build()
    return _lib.lib()
