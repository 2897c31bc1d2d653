"""quantize_model on the GPU (mirror of src/ptqkit/convert.py:236-293, RTN).

CPU part: target discovery and weight layout for Linear and GPT-2 style
Conv1D modules, and the argument errors. GPU part: a small model converted
in place; every layer's codes/scales/zeros are bit-identical to the oracle's
RTN and the forward (kernel path, bias added in the epilogue) matches the
oracle's dequant-GEMM plus bias within the dequant-GEMM tolerance.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch
from torch import nn

import oracle
from conftest import assert_close_y


class Conv1D(nn.Module):
    """GPT-2's Conv1D layout: weight [in, out], y = x @ W + b."""

    def __init__(self, nf: int, nx: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.randn(nx, nf) * 0.02)
        self.bias = nn.Parameter(torch.randn(nf) * 0.1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.weight + self.bias


class TinyModel(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(256, 384)
        self.proj = Conv1D(128, 384)
        self.head = nn.Linear(128, 96, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.head(torch.relu(self.proj(torch.relu(self.fc1(x)))))


def _wq():  # type: ignore[no-untyped-def]
    return importlib.import_module("weight-quantizer_b200")


def test_targets_and_layout_on_cpu() -> None:
    wq = _wq()
    torch.manual_seed(0)
    model = TinyModel()
    names = [n for n, _ in wq.iter_targets(model)]
    assert names == ["fc1", "proj", "head"]
    assert tuple(wq.weight_out_in(model.fc1).shape) == (384, 256)
    assert tuple(wq.weight_out_in(model.proj).shape) == (128, 384)   # Conv1D transposed to [out, in]
    assert torch.equal(wq.weight_out_in(model.proj), model.proj.weight.detach().t())


def test_quantize_model_argument_errors() -> None:
    wq = _wq()
    model = TinyModel()
    with pytest.raises(RuntimeError, match="quantize_model expects CUDA parameters"):
        wq.quantize_model(model, wq.QuantConfig(bits=4, group_size=128))


@pytest.mark.gpu
def test_quantize_model_kernel_forward_matches_oracle(cuda) -> None:
    wq = _wq()
    torch.manual_seed(1)
    model = TinyModel()
    ref_layers = {n: (wq.weight_out_in(m).clone(), None if getattr(m, "bias", None) is None else m.bias.detach().clone())
                  for n, m in wq.iter_targets(model)}
    model = model.to(cuda)
    cfg = wq.QuantConfig(bits=4, symmetric=False, group_size=128)
    out = wq.quantize_model(model, cfg, kernel=True)
    assert out is model
    for name, (w, b) in ref_layers.items():
        layer = getattr(model, name)
        assert isinstance(layer, wq.QuantizedLinear) and layer.impl == "kernel"
        r = oracle.quantize_stored(w.numpy(), 4, False, 128)
        assert np.array_equal(layer.codes.cpu().numpy(), r["q"]), name
        assert np.array_equal(layer.scales.cpu().numpy().view(np.int32), r["scales"].view(np.int32)), name
        assert np.array_equal(layer.zeros.cpu().numpy().view(np.int32), r["zeros"].view(np.int32)), name
        for batch in (1, 3, 40):
            x = torch.randn(batch, w.shape[1])
            y = layer(x.to(cuda)).cpu().numpy()
            yo = oracle.dequant_gemm(x.numpy(), r["q"], r["scales"], r["zeros"], None, 128, 4)
            if b is not None:
                yo = yo + b.numpy()
            assert_close_y(y, yo, f"{name} batch {batch}")
    # the whole model runs end to end on the kernels
    x = torch.randn(5, 256, device=cuda)
    assert model(x).shape == (5, 96)


@pytest.mark.gpu
@pytest.mark.parametrize("batch,group", [(2, 64), (17, 128), (9, 32)])
def test_bias_epilogue_every_path(cuda, batch: int, group: int) -> None:
    """decode kernel (batch <= 4), tensor-core kernel (G % 64 == 0) and the
    tiled fallback (G = 32): the epilogue's bias add equals y + bias."""
    wq = _wq()
    g = torch.Generator().manual_seed(batch)
    M, K = 200, 512
    w = torch.randn(M, K, generator=g) * 0.02
    r = oracle.quantize_stored(w.numpy(), 4, True, group)
    x = torch.randn(batch, K, generator=g)
    bias = torch.randn(M, generator=g)
    args = (torch.from_numpy(r["q"]).to(cuda), torch.from_numpy(r["scales"]).to(cuda),
            torch.from_numpy(r["zeros"]).to(cuda), None, group, 4)
    y0 = wq._kernels.dequant_gemm(x.to(cuda), *args)
    y1 = wq._kernels.dequant_gemm(x.to(cuda), *args, bias=bias.to(cuda))
    assert torch.equal(y1, y0 + bias.to(cuda))


@pytest.mark.gpu
def test_bias_with_empty_k(cuda) -> None:
    wq = _wq()
    bias = torch.tensor([1.5, -0.0, 2.0], device=cuda)
    q = torch.zeros(3, 0, dtype=torch.uint8, device=cuda)
    s = torch.ones(3, 0, device=cuda)
    y = wq._kernels.dequant_gemm(torch.zeros(2, 0, device=cuda), q, s, s.clone(), None, 8, 4, bias=bias)
    # the reference's zero result plus the bias: 0 + (-0.0) is +0.0
    assert torch.equal(y, torch.zeros(2, 3, device=cuda) + bias)
