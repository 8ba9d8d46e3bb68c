"""Shared pytest configuration: the ``gpu`` marker and import paths."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) and the built native library")
    # The native library is a build output (not committed): build it once if this checkout has none.
    from lich_b200.build import LIB, build

    if not LIB.exists():
        build()
