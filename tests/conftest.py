"""Test configuration: import paths and the ``gpu`` marker.

Tests marked ``gpu`` need a B200 (sm_100a); everything else runs on CPU.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "techjam-kernel_b200", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a B200 GPU (sm_100a)")
