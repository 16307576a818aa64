"""Shared test setup.

Markers: ``gpu`` tests need a CUDA device (run on a B200 box); everything else
runs on CPU. Golden vectors live in tests/golden (made by make_golden.py from
the reference packer itself).
"""

from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def sha16(a) -> str:
    """First 16 hex digits of sha256 of the array's raw bytes (the golden hash)."""
    if hasattr(a, "numpy"):
        a = a.contiguous().cpu().numpy()
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def fp16_from_hex(s: str, shape) -> np.ndarray:
    return np.frombuffer(bytes.fromhex(s), dtype="<u2").view(np.float16).reshape(shape)


def load_golden(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


def small_inputs(seed: int = 0, n: int = 64, k: int = 512):
    """The golden generator's input recipe (tests/golden/make_golden.py)."""
    import torch

    torch.manual_seed(seed)
    gauss = torch.randn(n, k, dtype=torch.float16) * 0.02
    skew = (torch.rand(n, k) * 0.5 + 2.0).to(torch.float16)
    x = torch.randn(8, k, dtype=torch.float16)
    return gauss, skew, x


def bench_inputs(n: int, k: int):
    """Benchmark-shape recipe: seed 0, w = randn*0.02 drawn before x [1, K]."""
    import torch

    torch.manual_seed(0)
    w = torch.randn(n, k, dtype=torch.float16) * 0.02
    x = torch.randn(1, k, dtype=torch.float16)
    return w, x


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
