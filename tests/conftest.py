"""Shared pytest setup.

Tests marked `gpu` need a CUDA device (they run on the B200 box with
`pytest -m gpu`); everything else runs on CPU (`pytest -m "not gpu"`).
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu on the B200 box)")
