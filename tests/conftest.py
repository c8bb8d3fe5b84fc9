from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "orda-knowledge-distillation-kernel_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built CUDA library")


@pytest.fixture(autouse=True)
def _empty_cuda_cache_after_test():
    yield
    import torch

    if torch.cuda.is_available():
        torch.cuda.empty_cache()
