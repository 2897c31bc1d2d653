"""AWQ alpha search on the GPU against the reference's fixtures and the oracle.

Per case (tests/golden/make_awq.py): the winning alpha equals the reference's
and the oracle's; every candidate's pre-scale equals the oracle's bit for bit
and is within 5e-7 relative of the reference's (a few fp32 ulp: the
reference's comes from torch's CPU vector math, whose fp32 pow and sqrt are
not correctly rounded and vary with the host's instruction set); its score
within 5e-3 relative of the reference's (a pre-scale a few ulp away can flip a
handful of codes) and within 1e-5 relative of the oracle's fp64 score for the
same codes (the dequant-GEMM's tolerance); and the winner's codes, scales,
zeros and channel scale are bit-exact with the oracle's RTN given the GPU's
own pre-scale, so the whole search agrees with the oracle bit for bit. Plus the reference's two AWQ tests
(tests/test_awq.py:12-41) and its quantize_model AWQ test (tests/test_convert.py:46-63).
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch
from torch import nn

from test_awq import awq_cases, score

import oracle

pytestmark = pytest.mark.gpu


def awq_mod():  # type: ignore[no-untyped-def]
    return importlib.import_module("weight-quantizer_b200.awq")


def test_search_matches_reference_and_oracle(wq, cuda) -> None:
    cases, meta, z = awq_cases()
    awq = awq_mod()
    for c, m in zip(cases, meta):
        name = m["name"]
        cfg = wq.QuantConfig(bits=m["bits"], symmetric=m["symmetric"], group_size=m["group_size"],
                             method=wq.Method.AWQ, awq_alphas=tuple(m["alphas"]))
        ma = None if c["mean_abs"] is None else c["mean_abs"].to(cuda)
        r = awq.awq_search(c["w"].to(cuda), c["x"].to(cuda), cfg, mean_abs=ma)
        assert r["alpha"] == m["alpha"], name
        w, x = c["w"].numpy(), c["x"].numpy()
        # the oracle's search on the same inputs: same alpha, same pre-scales bit for bit
        ro_search = oracle.awq_search(w, x, m["bits"], m["symmetric"], m["group_size"], tuple(m["alphas"]),
                                      None if c["mean_abs"] is None else c["mean_abs"].numpy())
        assert ro_search["alpha"] == r["alpha"], name
        for i, a in enumerate(m["alphas"]):
            got_pre = r["pre_scale"][i].cpu().numpy()
            assert np.array_equal(got_pre.view(np.int32), ro_search["pre_scale"][i].view(np.int32)), (name, a)
        for i, a in enumerate(m["alphas"]):
            pre = r["pre_scale"][i].cpu().numpy()
            np.testing.assert_allclose(pre, z[f"{name}.pre{i}"], rtol=5e-7, err_msg=f"{name} alpha={a}")
            assert abs(r["mse"][i] - m["mse"][i]) <= 5e-3 * m["mse"][i], (name, a, r["mse"][i], m["mse"][i])
            ro = oracle.rtn_quantize(w, m["bits"], m["symmetric"], m["group_size"], pre)
            assert abs(r["mse"][i] - score(w, x, ro)) <= 1e-5 * score(w, x, ro), (name, a)
        qw = r["weight"]
        i = m["alphas"].index(m["alpha"])
        ro = oracle.quantize_stored(w, m["bits"], m["symmetric"], m["group_size"], r["pre_scale"][i].cpu().numpy())
        assert np.array_equal(qw.codes.cpu().numpy(), ro["q"]), name
        assert np.array_equal(qw.scales.cpu().numpy().view(np.int32), ro["scales"].view(np.int32)), name
        assert np.array_equal(qw.zeros.cpu().numpy().view(np.int32), ro["zeros"].view(np.int32)), name
        assert np.array_equal(qw.channel_scale.cpu().numpy().view(np.int32), ro["channel_scale"].view(np.int32)), name
        assert qw.group_size == m["stored_group"]
        # against the reference's own codes: equal but for ulp-level pre-scale flips
        ref_codes = z[f"{name}.q"]
        got = qw.codes.cpu().numpy()
        if m["bits"] == 4:
            got, ref_codes = oracle.unpack_int4(got, w.shape[1]), oracle.unpack_int4(ref_codes, w.shape[1])
        assert (got != ref_codes).mean() <= 1e-3, name


def test_alpha_zero_is_rtn(wq, cuda) -> None:
    # tests/test_awq.py:12-25
    torch.manual_seed(0)
    weight = torch.randn(6, 32)
    inputs = torch.randn(40, 32)
    config = wq.QuantConfig(bits=4, symmetric=True, group_size=16, method=wq.Method.AWQ, awq_alphas=(0.0,))
    quantized, alpha = awq_mod().awq_quantize(weight.to(cuda), inputs.to(cuda), config)
    rtn = wq.quantize_weight(weight.to(cuda), wq.QuantConfig(bits=4, symmetric=True, group_size=16))
    assert alpha == 0.0
    assert torch.allclose(wq.dequantize_weight(quantized), wq.dequantize_weight(rtn), atol=1e-5)


def test_search_is_not_worse_than_rtn_on_search_rows(wq, cuda) -> None:
    # tests/test_awq.py:28-41
    torch.manual_seed(0)
    weight = torch.randn(6, 32) * 0.1
    weight[:, 1] = 3.0
    inputs = torch.randn(48, 32)
    inputs[:, 0] *= 20
    config = wq.QuantConfig(bits=4, symmetric=True, group_size=16, method=wq.Method.AWQ)
    w, x = weight.to(cuda), inputs.to(cuda)
    quantized, _alpha = awq_mod().awq_quantize(w, x, config)
    rtn = wq.quantize_weight(w, wq.QuantConfig(bits=4, symmetric=True, group_size=16))

    def mse(hat: torch.Tensor) -> float:
        return float((x @ (hat - w).transpose(0, 1)).square().mean())

    assert mse(wq.dequantize_weight(quantized)) <= mse(wq.dequantize_weight(rtn)) + 1e-6


def test_reduction_kernels(wq, cuda) -> None:
    k = wq._kernels
    g = torch.Generator().manual_seed(7)
    x = torch.randn(1001, 300, generator=g) * torch.exp(torch.randn(300, generator=g))
    xd = x.to(cuda)
    acc = k.channel_abs_sum(xd)
    np.testing.assert_allclose(acc.cpu().numpy(), np.abs(x.numpy().astype(np.float64)).sum(0), rtol=1e-12)
    # accumulation across calls and strided rows (every third row of a wider buffer)
    wide = torch.randn(90, 512, generator=g).to(cuda)
    view = wide[::3, :300]
    acc2 = k.channel_abs_sum(view, acc.clone())
    expect = np.abs(x.numpy().astype(np.float64)).sum(0) + np.abs(view.cpu().numpy().astype(np.float64)).sum(0)
    np.testing.assert_allclose(acc2.cpu().numpy(), expect, rtol=1e-12)
    a, b = torch.randn(3, 12345, generator=g), torch.randn(3, 12345, generator=g)
    got = float(k.sq_err_sum(a.to(cuda), b.to(cuda)).item())
    ref = float(((a.double() - b.double()) ** 2).sum())
    assert abs(got - ref) <= 1e-12 * ref
    assert float(k.sq_err_sum(a.to(cuda), b.to(cuda)).item()) == got   # deterministic
    # pre-scales bit for bit with the oracle's formula (fp64 power rounded once,
    # fp64 mean rounded once, fp32 division), on LogNormal(0, 1) magnitudes
    # like the activation statistics of the AWQ workload (11008 channels)
    rng = np.random.default_rng(3)
    for mag in (np.maximum(np.abs(rng.standard_normal(777)).astype(np.float32), np.float32(1e-8)),
                np.exp(rng.standard_normal(11008)).astype(np.float32)):
        for alpha in (0.0, 0.25, 0.5, 0.75, 1.0):
            pre = k.awq_pre_scale(torch.from_numpy(mag).to(cuda), alpha).cpu().numpy()
            if alpha == 0.0:
                assert np.all(pre == 1.0)
                continue
            p = (mag.astype(np.float64) ** alpha).astype(np.float32)
            expect = (p / max(np.float32(p.astype(np.float64).mean()), np.float32(1e-8))).astype(np.float32)
            assert np.array_equal(pre.view(np.int32), expect.view(np.int32)), (mag.size, alpha)


class Tiny(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(16, 32)
        self.fc2 = nn.Linear(32, 16)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(torch.relu(self.fc1(x)))


@pytest.mark.parametrize("sequential", [False, True])
@pytest.mark.parametrize("kernel", [False, True])
def test_quantize_model_awq_tiny_mlp(wq, cuda, sequential: bool, kernel: bool) -> None:
    # tests/test_convert.py:46-63 (AWQ row), on the GPU
    torch.manual_seed(0)
    batches = [torch.randn(4, 16).to(cuda) for _ in range(3)]
    config = wq.QuantConfig(bits=4, symmetric=True, group_size=8, method=wq.Method.AWQ)
    model = Tiny().to(cuda)
    w1 = model.fc1.weight.detach().cpu().numpy().copy()
    wq.quantize_model(model, config, batches, sequential=sequential, kernel=kernel)
    out = model(torch.randn(2, 16).to(cuda))
    assert out.shape == (2, 16)
    assert torch.isfinite(out).all()
    for layer in (model.fc1, model.fc2):
        assert isinstance(layer, wq.QuantizedLinear)
        assert layer.awq_alpha in config.awq_alphas
    # fc1 sees the calibration inputs unchanged in both modes: the oracle's search agrees
    x = torch.cat(batches).cpu().numpy()
    r = oracle.awq_search(w1, x, 4, True, 8, config.awq_alphas)
    assert model.fc1.awq_alpha == r["alpha"]
