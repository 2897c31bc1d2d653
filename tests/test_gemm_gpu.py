"""Dequant-GEMM on the GPU against the oracle and the reference's golden outputs.

Tolerance (written once, in conftest.assert_close_y): max|dy| <= 1e-4 * (1 + |y|)
elementwise and relative Frobenius error <= 1e-5 against the reference kernel's
outputs; the reference's own kernel-vs-dense check (tests/test_gemm.py:62,
rtol = atol = 1e-4) is applied as well.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import assert_close_y, small_cases, workload_digests

pytestmark = pytest.mark.gpu


def dev_t(a: np.ndarray, dev: torch.device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def run_kernel(wq, data, name: str, meta: dict, dev: torch.device, x: np.ndarray | None = None) -> np.ndarray:
    xs = data[f"{name}.x"] if x is None else x
    ch = data.get(f"{name}.channel")
    y = wq._kernels.dequant_gemm(
        dev_t(xs, dev), dev_t(data[f"{name}.q"], dev), dev_t(data[f"{name}.scales"], dev),
        dev_t(data[f"{name}.zeros"], dev), None if ch is None else dev_t(ch, dev),
        meta["stored_group"], meta["bits"], 0)
    return y.cpu().numpy()


def test_nibble_dot_known_answer(wq, cuda) -> None:
    # tests/test_gemm.py:13-32, through the package's own packing and both impls
    codes = torch.tensor([[1, 2], [15, 0]], dtype=torch.int32, device=cuda)
    qw = wq.assemble_quantized(codes, torch.tensor([[1.0], [1.0]]), torch.zeros(2, 1), bits=4,
                               group_size=2, symmetric=True, granularity="channel")
    x = torch.tensor([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]], device=cuda)
    expect = torch.tensor([[1.0, 15.0], [2.0, 0.0], [3.0, 15.0]], device=cuda)
    assert torch.allclose(wq.dequant_gemm(x, qw, impl="reference"), expect, atol=1e-6)
    assert torch.allclose(wq.dequant_gemm(x, qw, impl="kernel"), expect, atol=1e-6)


def test_golden_cases(wq, cuda) -> None:
    data, meta = small_cases()
    rtn = {m["name"]: m for m in meta if m["kind"] in ("rtn", "kat")}
    n = 0
    for m in meta:
        if m["kind"] != "gemm":
            continue
        name = m["name"]
        got = run_kernel(wq, data, name, rtn[name], cuda)
        assert_close_y(got, data[f"{name}.y_kernel"], name)
        assert np.allclose(got, data[f"{name}.y_reference"], rtol=1e-4, atol=1e-4), name
        n += 1
    assert n > 30


def test_reference_test_cases_through_package(wq, cuda) -> None:
    """tests/test_gemm.py:35-65 run through the package API end to end (GPU RTN + GPU GEMM)."""
    cases = [
        (4, 8, 1, 8, True, None, False), (5, 7, 3, 8, True, 0, False), (8, 16, 4, 4, True, 8, False),
        (3, 13, 1, 4, False, 4, False), (6, 32, 5, 4, True, 16, True), (32, 128, 2, 4, True, 128, False),
        (4, 1, 2, 8, True, None, False), (7, 17, 8, 8, False, None, False),
    ]
    data, _ = small_cases()
    g = torch.Generator().manual_seed(0)
    for i, (out, inn, batch, bits, sym, group, use_pre) in enumerate(cases):
        w = torch.randn(out, inn, generator=g)
        pre = torch.rand(inn, generator=g) + 0.25 if use_pre else None
        qw = wq.quantize_weight(w, wq.QuantConfig(bits=bits, symmetric=sym, group_size=group), pre_scale=pre)
        x = torch.randn(batch, inn, generator=g).to(cuda)
        ref = wq.dequant_gemm(x, qw, impl="reference")
        got = wq.dequant_gemm(x, qw, impl="kernel", nthreads=1)
        assert torch.allclose(got, ref, rtol=1e-4, atol=1e-4), i
        assert_close_y(got.cpu().numpy(), data[f"refcase{i}.y_kernel"], f"refcase{i}")
        again = wq.dequant_gemm(x, qw, impl="kernel", nthreads=2)
        assert torch.equal(got, again)


def _rand_layer(wq, g, M, K, bits, sym, group, pre=False):
    w = torch.randn(M, K, generator=g) * 0.02
    s = torch.rand(K, generator=g) + 0.25 if pre else None
    return wq.quantize_weight(w, wq.QuantConfig(bits=bits, symmetric=sym, group_size=group), pre_scale=s)


def _oracle_y(orc, qw, x: torch.Tensor) -> np.ndarray:
    ch = None if qw.channel_scale is None else qw.channel_scale.cpu().numpy()
    return orc.dequant_gemm(x.cpu().numpy(), qw.codes.cpu().numpy(), qw.scales.cpu().numpy(),
                            qw.zeros.cpu().numpy(), ch, qw.group_size, qw.bits)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 17])
def test_shapes_sweep_vs_oracle(wq, orc, cuda, bits: int, batch: int) -> None:
    """Decode-path and tiled-path shapes: odd K, odd groups, per-tensor broadcast,
    channel scale, rows not a multiple of any tile."""
    g = torch.Generator().manual_seed(100 + bits * 10 + batch)
    shapes = [(96, 256, 128, True, False), (130, 1024, 64, False, True), (33, 4095, 64, True, False),
              (64, 768, None, False, False), (50, 300, 0, True, False), (17, 13, 3, False, False),
              (40, 2048, 32, True, True), (257, 512, 512, False, False),
              # int4 batches 1-2 on the integer tensor-core decode kernel: one
              # table for all rows, full 8192-wide K slices at F = 128 and 64,
              # per-channel tables with a partial last row block
              (64, 512, 0, True, False), (48, 8192, 128, True, True), (32, 8192, 64, False, False),
              (20, 1024, None, True, False)]
    for (M, K, group, sym, pre) in shapes:
        qw = _rand_layer(wq, g, M, K, bits, sym, group, pre)
        x = torch.randn(batch, K, generator=g)
        got = wq.dequant_gemm(x.to(cuda), qw, impl="kernel").cpu().numpy()
        assert_close_y(got, _oracle_y(orc, qw, x), f"{M}x{K} g{group} b{batch} bits{bits}")


def test_decode_and_tiled_paths_agree(wq, orc, cuda) -> None:
    """The same problem through the streaming kernel (aligned rows) and through
    the tiled kernel (a copy of the codes at a 1-byte offset, which the
    streaming kernel does not take)."""
    g = torch.Generator().manual_seed(5)
    for bits in (4, 8):
        qw = _rand_layer(wq, g, 300, 2048, bits, True, 128)
        x = torch.randn(3, 2048, generator=g).to(cuda)
        y_fast = wq._kernels.dequant_gemm(x, qw.codes, qw.scales, qw.zeros, None, qw.group_size, bits)
        buf = torch.empty(qw.codes.numel() + 16, dtype=torch.uint8, device=cuda)
        shifted = buf[1:1 + qw.codes.numel()].view(qw.codes.shape)
        shifted.copy_(qw.codes)
        assert shifted.data_ptr() % 16 != 0
        y_tiled = wq._kernels.dequant_gemm(x, shifted, qw.scales, qw.zeros, None, qw.group_size, bits)
        ref = _oracle_y(orc, qw, x)
        assert_close_y(y_fast.cpu().numpy(), ref, "fast")
        assert_close_y(y_tiled.cpu().numpy(), ref, "tiled")


def test_deterministic_repeat(wq, cuda) -> None:
    g = torch.Generator().manual_seed(9)
    qw = _rand_layer(wq, g, 1000, 4096, 4, True, 128)
    for b in (1, 4, 64):
        x = torch.randn(b, 4096, generator=g).to(cuda)
        a = wq.dequant_gemm(x, qw, impl="kernel")
        c = wq.dequant_gemm(x, qw, impl="kernel")
        assert torch.equal(a, c)


def test_edge_sizes(wq, cuda) -> None:
    g = torch.Generator().manual_seed(11)
    qw = _rand_layer(wq, g, 8, 64, 4, True, 32)
    # empty batch
    y = wq.dequant_gemm(torch.zeros(0, 64, device=cuda), qw, impl="kernel")
    assert y.shape == (0, 8)
    # leading dims are kept
    x = torch.randn(2, 3, 64, generator=g).to(cuda)
    y = wq.dequant_gemm(x, qw, impl="kernel")
    assert y.shape == (2, 3, 8)
    assert torch.allclose(y, wq.dequant_gemm(x, qw, impl="reference"), rtol=1e-4, atol=1e-4)
    # all-zero activations and activations with a huge dynamic range
    for xs in (torch.zeros(2, 64), torch.tensor([[1e30] + [1e-30] * 63, [3.0] * 64])):
        y = wq.dequant_gemm(xs.to(cuda), qw, impl="kernel")
        r = wq.dequant_gemm(xs.to(cuda), qw, impl="reference")
        assert torch.allclose(y, r, rtol=1e-5, atol=1e-30)


def test_output_into_strided_view(wq, cuda) -> None:
    g = torch.Generator().manual_seed(12)
    qw = _rand_layer(wq, g, 96, 512, 4, True, 128)
    x = torch.randn(2, 512, generator=g).to(cuda)
    big = torch.full((2, 200), -7.0, device=cuda)
    view = big[:, 50:146]
    wq._kernels.dequant_gemm(x, qw.codes, qw.scales, qw.zeros, None, qw.group_size, 4, out=view)
    assert torch.allclose(view, wq.dequant_gemm(x, qw, impl="reference"), rtol=1e-4, atol=1e-4)
    assert torch.all(big[:, :50] == -7.0) and torch.all(big[:, 146:] == -7.0)


@pytest.mark.parametrize("wname", ["gpt2_c_fc_int4_g128", "gpt2_small_int8_asym", "awq_11008x4096",
                                   "oddk_4096x4095_g64", "sharded_28672x8192"])
def test_workloads_vs_oracle(wq, orc, cuda, wname: str) -> None:
    wl = importlib.import_module("weight-quantizer_b200.workloads")
    layers = wl.WORKLOADS[wname]()
    assert len(layers) == len(workload_digests()[wname])
    for layer in layers:
        qw = wq.quantize_weight(layer.weight, layer.config, pre_scale=layer.pre_scale)
        for b, x in layer.x.items():
            got = wq.dequant_gemm(x.to(cuda), qw, impl="kernel").cpu()
            # every row, batch 4096 of the 28672 x 8192 layer included (the
            # oracle's threads take a few seconds for it)
            ref = _oracle_y(orc, qw, x)
            assert_close_y(got.numpy(), ref, f"{wname}/{layer.name} b{b}")


@pytest.mark.parametrize("batch", [5, 64, 4096])
def test_fractional_zero_points_vs_oracle(wq, orc, cuda, batch: int) -> None:
    """ptqkit's operator takes any fp32 zero point (dequant_gemm.cpp:73-86
    computes (code - zero) * scale in fp32). The tensor-core path builds A from
    the zero's integer part and subtracts the fractional rest times the group's
    sum of x' in its epilogue. Rows mix integer, fractional, negative and
    above-range zeros, so that some warps take the correction and some do not;
    per-tensor tables and a channel scale are covered too. Zeros far outside
    the code range make y a small difference of large terms, so that case uses
    positive activations (a well-conditioned sum; with mixed signs any two fp32
    summation orders differ by more than the tolerance there)."""
    g = torch.Generator().manual_seed(700 + batch)
    cases = ((4, 300, 1024, 128, False, False), (8, 256, 768, 64, True, False), (4, 160, 512, 512, False, False),
             (4, 160, 512, 128, False, True))
    for bits, M, K, group, pre, far in cases:
        qw = _rand_layer(wq, g, M, K, bits, False, group, pre)
        z = qw.zeros.cpu().clone()
        rows = z.shape[0]
        frac = torch.rand(z.shape, generator=g) - 0.5
        z[rows // 3:] += frac[rows // 3:]                       # fractional from row M/3 on
        z[: rows // 8] = torch.tensor(-2.75)                    # negative, fractional
        x = torch.randn(batch, K, generator=g)
        if far:
            z[rows // 8: rows // 6] = torch.tensor(1500.25)     # beyond the integer part's [0, 1023]
            x = x.abs() + 0.1
        ch = None if qw.channel_scale is None else qw.channel_scale
        got = wq._kernels.dequant_gemm(x.to(cuda), qw.codes, qw.scales, z.to(cuda), ch, qw.group_size, bits)
        ref = orc.dequant_gemm(x.numpy(), qw.codes.cpu().numpy(), qw.scales.cpu().numpy(), z.numpy(),
                               None if ch is None else ch.cpu().numpy(), qw.group_size, bits)
        assert_close_y(got.cpu().numpy(), ref, f"bits{bits} {M}x{K} g{group} b{batch} fractional zeros")
        assert wq._kernels.fault_status() == 0
    # per-tensor table with one fractional zero for every row
    qw = _rand_layer(wq, g, 200, 640, 8, False, 0)
    z = qw.zeros.cpu() + 0.375
    x = torch.randn(batch, 640, generator=g)
    got = wq._kernels.dequant_gemm(x.to(cuda), qw.codes, qw.scales, z.to(cuda), None, qw.group_size, 8)
    ref = orc.dequant_gemm(x.numpy(), qw.codes.cpu().numpy(), qw.scales.cpu().numpy(), z.numpy(), None,
                           qw.group_size, 8)
    assert_close_y(got.cpu().numpy(), ref, f"per-tensor fractional zero b{batch}")


def test_integer_zero_points_unchanged_by_correction(wq, cuda) -> None:
    """Adding an exact 0.0 to every zero point must not change a single bit:
    warps whose zeros are all integers skip the fractional-zero term."""
    g = torch.Generator().manual_seed(41)
    qw = _rand_layer(wq, g, 512, 2048, 4, False, 128)
    x = torch.randn(96, 2048, generator=g).to(cuda)
    a = wq._kernels.dequant_gemm(x, qw.codes, qw.scales, qw.zeros, None, 128, 4)
    b = wq._kernels.dequant_gemm(x, qw.codes, qw.scales, (qw.zeros + 0.0).contiguous(), None, 128, 4)
    assert torch.equal(a, b)


def test_wide_batch_tiles_vs_oracle(wq, orc, cuda) -> None:
    """Batches of 1024 and more run the 192-wide tensor-core tile (the tiles of
    the other tests are 32, 64 and 128 wide). Cases with enough output tiles
    that K is not split: int4 g128 symmetric; int4 g64 asymmetric with a
    channel scale and a ragged last batch tile; int8 with an odd number of
    128-row weight tiles; fractional zero points. Each result is checked
    against the oracle and repeated bit for bit."""
    g = torch.Generator().manual_seed(1234)
    cases = ((2048, 1024, 1024, 4, True, 128, False, False),
             (2304, 768, 1200, 4, False, 64, True, False),
             (1664, 2048, 1100, 8, False, 128, False, False),
             (2048, 1024, 1056, 4, False, 128, False, True))
    for M, K, B, bits, sym, group, pre, frac in cases:
        qw = _rand_layer(wq, g, M, K, bits, sym, group, pre)
        z = qw.zeros.cpu().clone()
        if frac:
            z[M // 2:] += torch.rand(z[M // 2:].shape, generator=g) - 0.5
        x = torch.randn(B, K, generator=g)
        ch = qw.channel_scale
        got = wq._kernels.dequant_gemm(x.to(cuda), qw.codes, qw.scales, z.to(cuda), ch, qw.group_size, bits)
        again = wq._kernels.dequant_gemm(x.to(cuda), qw.codes, qw.scales, z.to(cuda), ch, qw.group_size, bits)
        assert torch.equal(got, again)
        ref = orc.dequant_gemm(x.numpy(), qw.codes.cpu().numpy(), qw.scales.cpu().numpy(), z.numpy(),
                               None if ch is None else ch.cpu().numpy(), qw.group_size, bits)
        assert_close_y(got.cpu().numpy(), ref, f"bits{bits} {M}x{K} g{group} b{B} frac{frac}")
        assert wq._kernels.fault_status() == 0
