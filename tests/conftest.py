import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA library's C ABI)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def shield_lib():
    """The CUDA library, loaded through its C ABI; a GPU test fails (not skips)
    when it cannot be loaded, so a silent fallback can never pass."""
    from llm_shield_b200 import binding
    return binding.lib()
