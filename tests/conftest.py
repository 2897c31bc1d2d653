"""Shared test setup.

Tests marked ``gpu`` need a CUDA device (a B200) and the built library; the
rest run on the CPU: the oracle against the reference's golden outputs, the
host-side logic, the C-ABI library's exports and argument validation, and the
multi-rank host logic on ``gloo``.
"""

from __future__ import annotations

import hashlib
import importlib
import json
import os
import sys
from typing import Any

import numpy as np
import pytest

REPO = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
# every dequant-GEMM call in the tests reads the kernels' fault word and raises
# if a bounded wait expired (checked mode of weight-quantizer_b200._kernels)
os.environ.setdefault("WQ_CHECK_FAULTS", "1")
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def package() -> Any:
    return importlib.import_module("weight-quantizer_b200")


def sha(a: Any) -> str:
    try:
        import torch

        if isinstance(a, torch.Tensor):
            a = a.detach().cpu().contiguous().numpy()
    except ImportError:
        pass
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


_small: dict[str, np.ndarray] | None = None


def small_cases() -> tuple[dict[str, np.ndarray], list[dict[str, Any]]]:
    global _small
    if _small is None:
        with np.load(os.path.join(GOLDEN, "small_cases.npz")) as z:
            _small = {k: z[k] for k in z.files}
    with open(os.path.join(GOLDEN, "small_cases.json")) as f:
        meta = json.load(f)
    return _small, meta


def workload_digests() -> dict[str, Any]:
    with open(os.path.join(GOLDEN, "workload_digests.json")) as f:
        return json.load(f)


def assert_close_y(got: np.ndarray, ref: np.ndarray, what: str = "") -> None:
    """The dequant-GEMM tolerance: max|dy| <= 1e-4 * (1 + |y|) elementwise and
    relative Frobenius error <= 1e-5."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    diff = np.abs(got - ref)
    bound = 1e-4 * (1.0 + np.abs(ref))
    worst = float((diff / bound).max()) if diff.size else 0.0
    assert worst <= 1.0, f"{what}: max|dy|/(1e-4(1+|y|)) = {worst:.3g}"
    nref = float(np.linalg.norm(ref))
    if nref > 0:
        rel = float(np.linalg.norm(got - ref)) / nref
        assert rel <= 1e-5, f"{what}: relative Frobenius error {rel:.3g}"


@pytest.fixture(scope="session")
def wq() -> Any:
    return package()


@pytest.fixture(scope="session")
def orc() -> Any:
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda() -> Any:
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    return torch.device("cuda", 0)
