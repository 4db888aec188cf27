"""Shared test configuration.

``-m "not gpu"`` runs everywhere (oracle vs the reference's golden vectors,
host logic, the C ABI's exports and host-side validation). ``-m gpu`` needs a
B200: those tests call the CUDA kernels through the C ABI and compare them
with the CPU oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_ROOT = ROOT / "sglang-restomod_b200"
for p in (str(ROOT), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"

# Tolerance of the GEMM / MoE parity checks (bf16 in, fp32 accumulate).
RTOL = 2e-2
ATOL = 2e-2


def load_golden(name: str):
    return np.load(GOLDEN / name)


def assert_close(got, want, rtol=RTOL, atol=ATOL, what=""):
    import torch

    got = torch.as_tensor(got).float().cpu()
    want = torch.as_tensor(want).float().cpu()
    assert got.shape == want.shape, f"{what}: shape {tuple(got.shape)} != {tuple(want.shape)}"
    bad = (got - want).abs() > atol + rtol * want.abs()
    if bool(bad.any()):
        idx = torch.nonzero(bad)[:5].tolist()
        worst = float(((got - want).abs() - rtol * want.abs()).max())
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.numel()} elements out of tolerance "
            f"(rtol={rtol}, atol={atol}); worst excess {worst:.3e}; first at {idx}"
        )


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda", torch.cuda.current_device())
