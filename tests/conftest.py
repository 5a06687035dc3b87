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


def _ensure_built():
    """Build libonpu.so in-tree if this checkout has none yet (nvcc cross-compiles without a GPU)."""
    lib = ROOT / "opennpu_b200" / "_lib" / "libonpu.so"
    if not lib.exists():
        from opennpu_b200 import build
        build.build()
    oracle_lib = ROOT / "oracle" / "_build" / "liboracle.so"
    if not oracle_lib.exists():
        import subprocess
        subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "all"], check=True)


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu on the GPU box)")
    config.addinivalue_line("markers", "slow: long CPU test")


GOLDEN = ROOT / "tests" / "golden"
