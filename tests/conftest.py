"""Shared test configuration: the `gpu` marker and seeded-input helpers."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and libnpu_b200.so")


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device; GPU tests fail (not skip) when it or the library is absent."""
    import torch
    from llm_compiler_3_b200 import _native
    assert torch.cuda.is_available(), "a GPU test ran without a CUDA device"
    _native.lib()
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"expected sm_100 (B200), got sm_{major}{minor}"
    return torch.device("cuda", 0)


def seeded(shape, seed, std=1.0, dtype=None):
    """FP16 N(0, std^2) from a per-tensor seeded CPU generator."""
    import torch
    g = torch.Generator().manual_seed(seed)
    t = (torch.randn(shape, generator=g) * std).half()
    return t if dtype is None else t.to(dtype)
