"""The no-allocation dequant-GEMM entry point, through the C ABI.

wq_dequant_gemm_f32_noalloc serves callers that may not allocate device memory
where they run a layer (a server that reserves all device memory up front, or
a runtime that only owns the buffers it is given): it takes the same inputs
and output as wq_dequant_gemm_f32 but uses a 32 MiB scratch array inside the
library instead of a caller workspace. This file is named to be collected
last, so a run that stops at its first failure has run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close_y

pytestmark = pytest.mark.gpu


def _noalloc(wq, x: torch.Tensor, qw, y: torch.Tensor) -> int:
    lib = wq._kernels.library()
    ch = qw.channel_scale
    stream = ctypes.c_void_p(int(torch.cuda.current_stream(x.device).cuda_stream))
    return int(lib.wq_dequant_gemm_f32_noalloc(
        x.data_ptr(), x.shape[0], x.shape[1],
        qw.codes.data_ptr(), qw.codes.shape[0], qw.codes.shape[1],
        qw.scales.data_ptr(), qw.scales.shape[0], qw.scales.shape[1],
        qw.zeros.data_ptr(), qw.zeros.shape[0], qw.zeros.shape[1],
        None if ch is None else ch.data_ptr(), -1 if ch is None else ch.shape[0],
        qw.group_size, qw.bits, y.data_ptr(), y.shape[1], stream))


def _layer(wq, g, M, K, bits, sym, group, pre=False):
    w = torch.randn(M, K, generator=g) * 0.02
    s = torch.rand(K, generator=g) + 0.25 if pre else None
    return wq.quantize_weight(w, wq.QuantConfig(bits=bits, symmetric=sym, group_size=group), pre_scale=s)


def test_noalloc_matches_regular_entry_point_on_consecutive_calls(wq, cuda) -> None:
    g = torch.Generator().manual_seed(21)
    # tensor-core shapes (the path that needs scratch), then two calls in a row
    # with different inputs and sizes so stale scratch would show
    cases = [(1000, 4096, 4, True, 128, False, 64), (777, 2048, 4, False, 128, True, 200),
             (640, 3072, 8, False, None, False, 37), (512, 4095, 4, True, 64, False, 9)]
    for (M, K, bits, sym, group, pre, B) in cases:
        qw = _layer(wq, g, M, K, bits, sym, group, pre)
        for call in range(2):
            x = torch.randn(B, K, generator=g).to(cuda)
            expect = wq.dequant_gemm(x, qw, impl="kernel")
            y = torch.full((B, M), float("nan"), device=cuda)
            assert _noalloc(wq, x, qw, y) == 0
            torch.cuda.synchronize()
            assert torch.isfinite(y).all()
            assert_close_y(y.cpu().numpy(), expect.cpu().numpy(), f"{M}x{K} b{B} call {call}")
    assert wq._kernels.fault_status() == 0


def test_noalloc_rejects_problems_beyond_its_scratch(wq, cuda) -> None:
    g = torch.Generator().manual_seed(22)
    qw = _layer(wq, g, 64, 8192, 4, True, 128)
    B = 2048  # needs about 4 * 2048 * 8192 bytes > 32 MiB
    x = torch.zeros(B, 8192, device=cuda)
    y = torch.zeros(B, 64, device=cuda)
    status = _noalloc(wq, x, qw, y)
    assert status == 21
    assert "no-allocation" in wq._kernels.status_message(status)
    # decode batches need no scratch at all and are served
    xs = torch.randn(2, 8192, generator=g).to(cuda)
    ys = torch.zeros(2, 64, device=cuda)
    assert _noalloc(wq, xs, qw, ys) == 0
    assert np.allclose(ys.cpu().numpy(), wq.dequant_gemm(xs, qw, impl="kernel").cpu().numpy(), rtol=0, atol=0)
