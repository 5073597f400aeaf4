"""Shared pytest configuration and fixtures.

Markers
-------
gpu : needs an sm_100 (B200) GPU; run with ``-m gpu``. Everything unmarked runs
      on CPU (oracle vs golden vectors, ABI exports, host logic, gloo ranks).

Fixtures mirror the reference suite (ghostweight_triton tests/conftest.py:20-113)
so the ported kernel/module tests read like the originals.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch
import torch.nn as nn

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an sm_100 (B200) GPU")


def _require_cuda() -> str:
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required - no GPU found.")
    return "cuda"


@pytest.fixture(scope="session")
def device() -> str:
    """'cuda' (skips when no GPU is visible, as the reference's fixture does)."""
    return _require_cuda()


@pytest.fixture()
def sample_linear(device: str) -> nn.Linear:
    torch.manual_seed(42)
    return nn.Linear(768, 3072, bias=True).to(device=device, dtype=torch.float16)


class _ToyMLP(nn.Module):
    """128 -> 512 -> 128 -> 10 MLP (fc3 sits on the min_features border)."""

    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(128, 512, bias=True)
        self.act1 = nn.ReLU()
        self.fc2 = nn.Linear(512, 128, bias=True)
        self.act2 = nn.ReLU()
        self.fc3 = nn.Linear(128, 10, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc3(self.act2(self.fc2(self.act1(self.fc1(x)))))


@pytest.fixture()
def toy_model(device: str) -> nn.Module:
    torch.manual_seed(0)
    return _ToyMLP().to(device=device, dtype=torch.float16)


@pytest.fixture()
def toy_model_cpu() -> nn.Module:
    torch.manual_seed(0)
    return _ToyMLP()


DTYPES = [torch.float16, torch.float32]
SHAPES = [
    (1, 128, 256),
    (1, 768, 3072),
    (16, 768, 3072),
    (128, 768, 3072),
    (128, 3072, 768),
]
SPARSITY_LEVELS = [0.0, 0.3, 0.5, 0.7, 0.95]


def tols(dtype: torch.dtype) -> dict:
    """Parity tolerances: 1e-2 for fp16/bf16 outputs, 1e-4 for fp32 (exact-fp32 accumulate)."""
    if dtype in (torch.float16, torch.bfloat16):
        return {"atol": 1e-2, "rtol": 1e-2}
    return {"atol": 1e-4, "rtol": 1e-4}
