"""Test configuration: register the ``gpu`` marker and put the repo root on
``sys.path`` so ``oracle`` and ``logitfill_b200`` import from the checkout."""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built extension")
