"""Shared pytest configuration.

Registers the ``gpu`` marker (tests that need a CUDA device and the built
extension) and puts the repository root on ``sys.path`` so ``oracle`` and
``junqi_b200`` import without installation.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built junqi_b200 extension")
    config.addinivalue_line("markers", "slow: long-running CPU test")
