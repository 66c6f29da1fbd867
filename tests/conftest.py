"""Test configuration: import paths, the `gpu` marker and shared helpers.

`-m "not gpu"` runs on a machine without a GPU (oracle vs golden fixtures,
host logic, library loading and exports, gloo multi-process logic).
`-m gpu` runs the CUDA parity tests through the C ABI on a B200.
"""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "triton-fused-ops_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a); run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running case")


def load_golden(name: str) -> dict:
    """{case: {field: array}} from tests/golden/<name>.npz."""
    data = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
    cases: dict = {}
    for key in data.files:
        case, field = key.split("/", 1)
        cases.setdefault(case, {})[field] = data[key]
    return cases


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA not available")
    return torch.device("cuda")


TORCH_DT = {"f16": "float16", "bf16": "bfloat16", "f32": "float32"}
NAME_DT = {"float16": "f16", "bfloat16": "bf16", "float32": "f32"}


def dev_tensor(a, dtype: str, device="cuda"):
    """numpy array (values representable in `dtype`) -> torch tensor of `dtype` on device."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32)))
    return t.to(getattr(torch, TORCH_DT[dtype])).to(device)


def host(t) -> np.ndarray:
    """torch tensor -> float32 numpy (exact for fp16/bf16)."""
    return t.detach().float().cpu().numpy()
