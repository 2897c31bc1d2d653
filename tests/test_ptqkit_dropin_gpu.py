"""ptqkit's own modules running this library: the drop-in, tested where it matters.

ptqkit (the reference package, installed unmodified into baseline/_ref) is
imported as is; ``ptqkit_binding.install`` adds the CUDA branch in front of
the CPU guard of its ``gemm.dequant_gemm`` (src/ptqkit/gemm.py:43-45). Then:

* ptqkit's ``quantize_model(..., kernel=True)`` (convert.py:236-293) quantizes
  a small model with Linear and GPT-2 Conv1D layers on the CPU (its own RTN,
  and its own AWQ search); the model is moved to the GPU and ptqkit's own
  ``QuantizedLinear.forward`` (linear.py:90-101) runs this library's kernels.
  Its outputs are compared with the same ptqkit model run on the CPU by
  ptqkit's compiled kernel (the reference result), at the dequant-GEMM
  tolerance of conftest.assert_close_y.
* ptqkit's ``gemm.dequant_gemm(impl="kernel")`` on CUDA tensors matches
  ptqkit's CPU kernel for int4 groups and int8 per-channel layers at decode
  and prefill batches.

Without the binding ptqkit refuses CUDA tensors, which the last test checks.
Skipped where baseline/_ref holds no ptqkit install.
"""

from __future__ import annotations

import copy
import dataclasses
import importlib
import os
import sys

import pytest
import torch
from torch import nn

from conftest import REPO, assert_close_y

pytestmark = pytest.mark.gpu

_REF = os.path.join(REPO, "baseline", "_ref")


@pytest.fixture(scope="module")
def ptqkit():  # type: ignore[no-untyped-def]
    if not os.path.isdir(os.path.join(_REF, "ptqkit")):
        pytest.skip("ptqkit is not installed in baseline/_ref")
    if _REF not in sys.path:
        sys.path.insert(0, _REF)
    return importlib.import_module("ptqkit")


@pytest.fixture()
def bound(ptqkit):  # type: ignore[no-untyped-def]
    binding = importlib.import_module("weight-quantizer_b200.ptqkit_binding")
    restore = binding.install(ptqkit)
    yield ptqkit
    restore()


class Conv1D(nn.Module):
    """GPT-2's Conv1D: weight [in, out], y = x @ W + b (ptqkit recognises it by name)."""

    def __init__(self, nf: int, nx: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.randn(nx, nf) * 0.02)
        self.bias = nn.Parameter(torch.randn(nf) * 0.1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.weight + self.bias


class Block(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.c_fc = Conv1D(1024, 512)
        self.c_proj = Conv1D(512, 1024)
        self.head = nn.Linear(512, 384, bias=True)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.head(self.c_proj(torch.relu(self.c_fc(x))))


@pytest.mark.parametrize("bits,group,method", [(4, 128, "rtn"), (8, None, "rtn"), (4, 128, "awq")])
def test_ptqkit_quantize_model_runs_on_b200(bound, cuda, bits: int, group, method: str) -> None:  # type: ignore[no-untyped-def]
    ptqkit = bound
    torch.manual_seed(0)
    model = Block()
    cfg = ptqkit.QuantConfig(bits=bits, symmetric=method == "rtn", group_size=group,
                             method=ptqkit.Method(method))
    calib = [torch.randn(4, 16, 512) for _ in range(2)] if method == "awq" else None
    ptqkit.quantize_model(model, cfg, calib, kernel=True)
    layers = [m for m in model.modules() if isinstance(m, ptqkit.QuantizedLinear)]
    assert len(layers) == 3 and all(m.impl == "kernel" for m in layers)
    for batch in (3, 8, 64):
        x = torch.randn(batch, 512)
        with torch.inference_mode():
            y_ref = model(x)                          # ptqkit's compiled CPU kernel
            gpu = copy.deepcopy(model).to(cuda)
            y = gpu(x.to(cuda))                       # ptqkit's QuantizedLinear -> this library
        assert y.device.type == "cuda"
        assert_close_y(y.cpu().numpy(), y_ref.numpy(), f"ptqkit model int{bits} {method} b{batch}")


@pytest.mark.parametrize("bits,group", [(4, 128), (4, 64), (8, None)])
def test_ptqkit_dequant_gemm_kernel_on_cuda(bound, cuda, bits: int, group) -> None:  # type: ignore[no-untyped-def]
    ptqkit = bound
    g = torch.Generator().manual_seed(bits)
    w = torch.randn(640, 2048, generator=g) * 0.02
    qw = ptqkit.quantize_weight(w, ptqkit.QuantConfig(bits=bits, symmetric=False, group_size=group))
    qw_gpu = dataclasses.replace(qw, codes=qw.codes.to(cuda), scales=qw.scales.to(cuda), zeros=qw.zeros.to(cuda))
    for batch in (1, 4, 16, 300):
        x = torch.randn(2, batch, 2048, generator=g)
        y_ref = ptqkit.gemm.dequant_gemm(x, qw, impl="kernel")
        y = ptqkit.gemm.dequant_gemm(x.to(cuda), qw_gpu, impl="kernel")
        assert tuple(y.shape) == (2, batch, 640)
        assert_close_y(y.cpu().numpy().reshape(-1, 640), y_ref.numpy().reshape(-1, 640), f"int{bits} g{group} b{batch}")


def test_ptqkit_refuses_cuda_without_the_binding(ptqkit, cuda) -> None:  # type: ignore[no-untyped-def]
    qw = ptqkit.quantize_weight(torch.randn(64, 128) * 0.02, ptqkit.QuantConfig(bits=4, group_size=128))
    with pytest.raises(RuntimeError, match="runs on CPU"):
        ptqkit.gemm.dequant_gemm(torch.randn(2, 128, device=cuda), qw, impl="kernel")
