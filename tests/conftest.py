"""Test configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 and call the CUDA kernels through the C ABI;
everything else runs on the CPU (oracle vs golden fixtures, host policy,
ABI exports, gloo multi-process logic).
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and the native library")
