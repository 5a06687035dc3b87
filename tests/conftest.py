import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# the reference's libonpu (oracle/_ref) must never look for an NPU device build
os.environ.setdefault("OPENNPU_GEMV_DIR", "/nonexistent-opennpu-gemv")
os.environ.setdefault("OPENNPU_GEMM8_DIR", "/nonexistent-opennpu-gemm8")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu on the GPU box)")
    config.addinivalue_line("markers", "slow: long CPU test")


GOLDEN = ROOT / "tests" / "golden"
