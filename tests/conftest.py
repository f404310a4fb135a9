"""Shared pytest setup: import paths, the ``gpu`` marker and CPU threading."""

from pathlib import Path
import sys

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "cuda-moe-engine_b200", ROOT, ROOT / "tests" / "golden"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    import torch

    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    torch.set_num_threads(1)
