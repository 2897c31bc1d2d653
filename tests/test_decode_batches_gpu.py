"""Dequant-GEMM at decode batches (3-32) against the oracle.

Batches 3-32 run the integer tensor-core kernel with stream-K over units of
256 rows x one fold block (dq_gemv_wide.cu). The cases cover every group
layout it takes (g64, g128, g256, per-channel, per-tensor; tables by TMA box
or by direct loads), int4 and int8, odd and short K, row counts that are not
multiples of 256, layers small enough that every row block is shared by many
CTAs (the fixed-order fix-up), channel scales with outlier channels,
fractional zero points, the bias epilogue and strided outputs; the
28672 x 8192 layer is checked on all rows. Batches just above 32 run the
tcgen05 kernel, split-K on small layers. Tolerance: conftest.assert_close_y
(max|dy| <= 1e-4 (1 + |y|), relative Frobenius <= 1e-5).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import assert_close_y

pytestmark = pytest.mark.gpu


def _layer(wq, g, M, K, bits, sym, group, pre=False):
    w = torch.randn(M, K, generator=g) * 0.02
    s = torch.rand(K, generator=g) + 0.25 if pre else None
    return wq.quantize_weight(w, wq.QuantConfig(bits=bits, symmetric=sym, group_size=group), pre_scale=s)


def _oracle(orc, qw, x, zeros=None):
    ch = None if qw.channel_scale is None else qw.channel_scale.cpu().numpy()
    z = qw.zeros.cpu().numpy() if zeros is None else zeros
    return orc.dequant_gemm(x.numpy(), qw.codes.cpu().numpy(), qw.scales.cpu().numpy(), z, ch, qw.group_size,
                            qw.bits)


CASES = [
    # M, K, bits, symmetric, group, pre_scale
    (300, 1024, 4, True, 128, False),
    (1000, 4095, 4, True, 64, False),
    (128, 8192, 4, False, 128, True),      # one row tile, long K
    (257, 2048, 4, True, 256, False),
    (200, 1536, 4, False, None, False),    # per-channel
    (96, 1024, 4, True, 0, False),         # per-tensor
    (384, 768, 8, False, None, False),     # int8 per-channel (GPT-2 shapes)
    (130, 3072, 8, True, 64, True),
    (512, 1008, 8, False, 128, False),     # K not a multiple of 128
    (64, 256, 8, True, 0, False),
]


@pytest.mark.parametrize("batch", [3, 5, 8, 16, 17, 25, 32, 33, 64])
def test_decode_batches_vs_oracle(wq, orc, cuda, batch: int) -> None:
    g = torch.Generator().manual_seed(900 + batch)
    for (M, K, bits, sym, group, pre) in CASES:
        qw = _layer(wq, g, M, K, bits, sym, group, pre)
        x = torch.randn(batch, K, generator=g)
        if pre:   # outlier channels, as in the AWQ workload
            idx = torch.randperm(K, generator=g)[: max(1, K // 100)]
            x[:, idx] *= 20.0
        got = wq.dequant_gemm(x.to(cuda), qw, impl="kernel").cpu().numpy()
        assert_close_y(got, _oracle(orc, qw, x), f"{M}x{K} int{bits} g{group} b{batch}")


def test_decode_fractional_zeros_and_bias(wq, orc, cuda) -> None:
    g = torch.Generator().manual_seed(31)
    for bits, group in ((4, 128), (8, None), (4, 64)):
        qw = _layer(wq, g, 520, 2048, bits, False, group)
        z = qw.zeros.cpu().clone()
        z += torch.rand(z.shape, generator=g) - 0.5
        z[:7] = -3.25
        x = torch.randn(24, 2048, generator=g)
        bias = torch.randn(520, generator=g)
        got = wq._kernels.dequant_gemm(x.to(cuda), qw.codes, qw.scales, z.to(cuda), None, qw.group_size, bits,
                                       bias=bias.to(cuda)).cpu().numpy()
        ref = _oracle(orc, qw, x, z.numpy()) + bias.numpy()[None, :]
        assert_close_y(got, ref, f"int{bits} g{group} fractional zeros + bias")


def test_decode_deterministic_and_full_layer(wq, orc, cuda) -> None:
    """The 28672 x 8192 int4 g128 layer at batches 8 and 32: all rows against
    the oracle, and bit-identical repeats."""
    g = torch.Generator().manual_seed(5)
    qw = _layer(wq, g, 28672, 8192, 4, True, 128)
    for b in (8, 32):
        x = torch.randn(b, 8192, generator=g)
        a = wq.dequant_gemm(x.to(cuda), qw, impl="kernel")
        c = wq.dequant_gemm(x.to(cuda), qw, impl="kernel")
        assert torch.equal(a, c)
        assert_close_y(a.cpu().numpy(), _oracle(orc, qw, x), f"28672x8192 b{b}")


def test_decode_into_strided_output(wq, cuda) -> None:
    g = torch.Generator().manual_seed(13)
    qw = _layer(wq, g, 200, 1024, 4, True, 128)
    x = torch.randn(12, 1024, generator=g).to(cuda)
    big = torch.full((12, 300), -7.0, device=cuda)
    view = big[:, 40:240]
    wq._kernels.dequant_gemm(x, qw.codes, qw.scales, qw.zeros, None, 128, 4, out=view)
    assert torch.allclose(view, wq.dequant_gemm(x, qw, impl="reference"), rtol=1e-4, atol=1e-4)
    assert torch.all(big[:, :40] == -7.0) and torch.all(big[:, 240:] == -7.0)
    assert np.isfinite(view.cpu().numpy()).all()
