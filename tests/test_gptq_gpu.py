"""GPTQ on the GPU against the reference's fixtures and the oracle.

Per case (tests/golden/make_gptq.py): codes equal ptqkit's except for weights
within rounding of a grid edge (the device factorization and GEMMs round
differently from CPU LAPACK/BLAS; at most 1e-3 of the codes may differ),
scales within 1e-5 relative, and the output error mean((X W_hat^T - X W^T)^2)
within 1e-3 relative of ptqkit's. A problem of one block of at most 128
columns (no GEMM) is bit-exact with the oracle fed the device's own factor.
Plus the reference's tests/test_gptq.py cases and its quantize_model GPTQ test
(tests/test_convert.py:46-63).
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch
from torch import nn

from test_gptq import gptq_cases, out_err, unpacked

import oracle

pytestmark = pytest.mark.gpu


def gptq_mod():  # type: ignore[no-untyped-def]
    return importlib.import_module("weight-quantizer_b200.gptq")


def test_gptq_matches_reference(wq, cuda) -> None:
    cases, meta, z = gptq_cases()
    g = gptq_mod()
    for c, m in zip(cases, meta):
        name = m["name"]
        cfg = wq.QuantConfig(bits=m["bits"], symmetric=m["symmetric"], group_size=m["group_size"],
                             method=wq.Method.GPTQ, percdamp=m["percdamp"], blocksize=m["blocksize"])
        qw = g.gptq_quantize(c["w"].to(cuda), c["h"].to(cuda), cfg)
        k = c["w"].shape[1]
        got = unpacked(qw.codes.cpu().numpy(), m["bits"], k)
        ref = unpacked(z[f"{name}.q"], m["bits"], k)
        assert (got != ref).mean() <= 1e-3, (name, int((got != ref).sum()))
        np.testing.assert_allclose(qw.scales.cpu().numpy(), z[f"{name}.scales"], rtol=1e-5, err_msg=name)
        assert qw.group_size == m["stored_group"]
        hat = wq.dequantize_weight(qw).cpu().numpy()
        err = out_err(c["x"].numpy(), c["w"].numpy(), hat)
        assert abs(err - m["out_err"]) <= 1e-3 * m["out_err"], (name, err, m["out_err"])


@pytest.mark.parametrize("bits,sym,group", [(4, True, 96), (4, False, 96), (8, True, None), (4, True, 0)])
def test_single_block_sweep_is_bit_exact(wq, cuda, bits: int, sym: bool, group: int | None) -> None:
    g = torch.Generator().manual_seed(40 + bits)
    k = 96
    x = torch.randn(4 * k, 6, generator=g) @ torch.randn(6, k, generator=g) + 0.3 * torch.randn(4 * k, k, generator=g)
    x[:, 5] = 0
    w = torch.randn(40, k, generator=g) * 0.05
    h = x.double().transpose(0, 1) @ x.double() / x.shape[0]
    cfg = wq.QuantConfig(bits=bits, symmetric=sym, group_size=group, method=wq.Method.GPTQ, percdamp=0.01,
                         blocksize=128)
    mod = gptq_mod()
    qw = mod.gptq_quantize(w.to(cuda), h.to(cuda), cfg)
    hd = h.to(cuda)
    dead = torch.diag(hd) == 0
    u = mod._factor_inverse(hd, 0.01).cpu().numpy()
    assert bool(dead.any())
    r = oracle.gptq_quantize(w.numpy(), h.numpy(), bits, sym, group, 0.01, 128, hinv=u)
    assert np.array_equal(unpacked(qw.codes.cpu().numpy(), bits, k), r["codes"])
    assert np.array_equal(qw.scales.cpu().numpy().view(np.int32), r["scales"].view(np.int32))
    assert np.array_equal(qw.zeros.cpu().numpy(), r["zeros"])


def _mse(weight: torch.Tensor, hat: torch.Tensor, inputs: torch.Tensor) -> float:
    err = inputs @ (hat - weight).transpose(0, 1)
    return float(err.square().mean().item())


def test_gptq_matches_rtn_on_identity_hessian(wq, cuda) -> None:
    # tests/test_gptq.py:11-29
    torch.manual_seed(0)
    weight = torch.randn(8, 32).to(cuda)
    inputs = torch.randn(64, 32).to(cuda)
    hessian = torch.eye(32, dtype=torch.float64)
    config = wq.QuantConfig(bits=4, symmetric=True, group_size=16, method=wq.Method.GPTQ, percdamp=0.0)
    gptq = wq.dequantize_weight(gptq_mod().gptq_quantize(weight, hessian.to(cuda), config))
    rtn = wq.dequantize_weight(wq.quantize_weight(weight, wq.QuantConfig(bits=4, symmetric=True, group_size=16)))
    assert int((gptq - rtn).abs().gt(1e-4).sum()) <= 2
    assert _mse(weight, gptq, inputs) <= _mse(weight, rtn, inputs) * 1.05 + 1e-6


def test_gptq_reduces_output_mse(wq, cuda) -> None:
    # tests/test_gptq.py:32-52
    torch.manual_seed(0)
    out, k, n = 8, 32, 2048
    latent = torch.randn(n, 2) @ torch.randn(2, k)
    latent[:, 0] *= 5
    weight = torch.randn(out, k) * 0.1
    weight[:, 3] = 6
    hessian = latent.double().transpose(0, 1) @ latent.double() / n
    config = wq.QuantConfig(bits=4, symmetric=True, group_size=32, method=wq.Method.GPTQ, percdamp=0.01)
    w, lat = weight.to(cuda), latent.to(cuda)
    gptq = wq.dequantize_weight(gptq_mod().gptq_quantize(w, hessian.to(cuda), config))
    rtn = wq.dequantize_weight(wq.quantize_weight(w, wq.QuantConfig(bits=4, symmetric=True, group_size=32)))
    assert _mse(w, gptq, lat) < 0.5 * _mse(w, rtn, lat)
    assert torch.isfinite(gptq).all()


def test_dead_column_is_finite(wq, cuda) -> None:
    # tests/test_gptq.py:55-63
    torch.manual_seed(1)
    inputs = torch.randn(64, 16)
    inputs[:, 3] = 0
    weight = torch.randn(4, 16)
    hessian = inputs.double().transpose(0, 1) @ inputs.double() / inputs.shape[0]
    config = wq.QuantConfig(bits=4, symmetric=False, group_size=None, method=wq.Method.GPTQ)
    hat = wq.dequantize_weight(gptq_mod().gptq_quantize(weight.to(cuda), hessian.to(cuda), config))
    assert torch.isfinite(hat).all()


class Tiny(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.fc1 = nn.Linear(16, 32)
        self.fc2 = nn.Linear(32, 16)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(torch.relu(self.fc1(x)))


@pytest.mark.parametrize("sequential", [False, True])
def test_quantize_model_gptq_tiny_mlp(wq, cuda, sequential: bool) -> None:
    # tests/test_convert.py:46-63 (GPTQ row), on the GPU
    torch.manual_seed(0)
    batches = [torch.randn(4, 16).to(cuda) for _ in range(3)]
    config = wq.QuantConfig(bits=4, symmetric=True, group_size=8, method=wq.Method.GPTQ)
    model = Tiny().to(cuda)
    w1 = model.fc1.weight.detach().cpu().numpy().copy()
    wq.quantize_model(model, config, batches, sequential=sequential, kernel=True)
    out = model(torch.randn(2, 16).to(cuda))
    assert out.shape == (2, 16)
    assert torch.isfinite(out).all()
    # fc1's Hessian is the calibration inputs' in both modes: the oracle agrees up to near-ties
    x = torch.cat(batches).cpu().numpy().astype(np.float64)
    r = oracle.gptq_quantize(w1, x.T @ x / x.shape[0], 4, True, 8, 0.01, 128)
    got = oracle.unpack_int4(model.fc1.codes.cpu().numpy(), 16).astype(np.int32)
    assert (got != r["codes"]).mean() <= 0.01


@pytest.mark.parametrize("group", [32, None])
def test_nonfinite_obs_error_zeroes_the_column(wq, cuda, monkeypatch, group: int | None) -> None:
    """_obs_block (gptq.py:114-115) zeroes a column's OBS error in every row when
    any row's is not finite. A NaN planted on one diagonal entry of the factor
    (and, for the grouped case, a second one in a later block) makes that
    column's error NaN; the device sweep must give the oracle's codes bit for
    bit, i.e. zero those columns' errors and carry on."""
    g = torch.Generator().manual_seed(77)
    k = 192
    x = torch.randn(3 * k, k, generator=g)
    w = torch.randn(24, k, generator=g) * 0.05
    h = x.double().transpose(0, 1) @ x.double() / x.shape[0]
    mod = gptq_mod()
    u = mod._factor_inverse(h.to(cuda), 0.01).clone()
    u[7, 7] = float("nan")
    u[150, 150] = float("nan")
    monkeypatch.setattr(mod, "_factor_inverse", lambda hess, percdamp: u)
    cfg = wq.QuantConfig(bits=4, symmetric=True, group_size=group, method=wq.Method.GPTQ, percdamp=0.01,
                         blocksize=128)
    qw = mod.gptq_quantize(w.to(cuda), h.to(cuda), cfg)
    r = oracle.gptq_quantize(w.numpy(), h.numpy(), 4, True, group, 0.01, 128, hinv=u.cpu().numpy())
    assert np.array_equal(unpacked(qw.codes.cpu().numpy(), 4, k), r["codes"])
    assert np.isfinite(qw.scales.cpu().numpy()).all()


def test_chol_inverse_upper_vs_oracle(wq, cuda) -> None:
    """The GPTQ factor U (U^T U = A^-1) from this library's blocked kernels
    against the oracle's restatement of gptq.py:59-66 (factor, invert, factor
    the inverse upper): sizes from 1 to 1000 (one block, whole 64-column blocks
    and ragged last blocks), relative to max|U| within 1e-10, exactly zero below
    the diagonal, and U^T U A = I to 1e-9; a matrix that is not positive
    definite reports a column in info."""
    rng = np.random.default_rng(5)
    for n in (1, 2, 63, 64, 65, 130, 300, 1000):
        x = rng.standard_normal((2 * n + 3, n))
        a = x.T @ x / (2 * n + 3) + 0.1 * np.eye(n)
        u, info = wq._kernels.chol_inverse_upper(torch.from_numpy(a).to(cuda))
        assert int(info.item()) == 0, n
        u = u.cpu().numpy()
        ref = oracle.gptq_factor(a, 0.0)
        assert np.all(np.tril(u, -1) == 0.0), n
        assert np.abs(u - ref).max() <= 1e-10 * np.abs(ref).max(), n
        assert np.abs(u.T @ u @ a - np.eye(n)).max() <= 1e-9, n
    a = np.eye(70)
    a[40, 40] = -1.0
    _, info = wq._kernels.chol_inverse_upper(torch.from_numpy(a).to(cuda))
    assert int(info.item()) > 0
