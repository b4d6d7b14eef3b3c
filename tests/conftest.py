import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_packing.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def built_lib():
    """Build libkvr.so if it is missing or stale (nvcc cross-compiles here)."""
    from kv_reduce_b200 import build

    return build.build()


def bf16_from_bits(bits: np.ndarray, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)
    return t.to(device)


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
