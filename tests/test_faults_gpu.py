"""Fault reporting of the kernels' bounded waits, exercised without a fault.

Every mbarrier wait in the library's pipelines gives up after a bounded number
of polls, sets bit 0 of the library's device fault word and lets the launch
finish. This test makes such a wait run out on purpose in the library's
self-test kernel (a barrier that nothing ever arrives on; no copy is in flight,
nothing else is touched) and checks that the host sees it: the fault word, and
the checked mode of the Python binding, which raises on the next call.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_expired_wait_sets_fault_word_and_checked_call_raises(wq, cuda) -> None:
    k = wq._kernels
    k.fault_status(reset=True)
    k.selftest_expired_wait(16)
    assert k.fault_status(reset=False) & 1
    prev = k.set_fault_check(True)
    try:
        g = torch.Generator().manual_seed(1)
        qw = wq.quantize_weight(torch.randn(64, 256, generator=g) * 0.02,
                                wq.QuantConfig(bits=4, symmetric=True, group_size=128))
        x = torch.randn(8, 256, generator=g).to(cuda)
        with pytest.raises(RuntimeError, match="fault word"):
            wq.dequant_gemm(x, qw, impl="kernel")
        # the raise cleared the word: the context is usable and the next call is clean
        assert k.fault_status(reset=False) == 0
        y = wq.dequant_gemm(x, qw, impl="kernel")
        assert torch.allclose(y, wq.dequant_gemm(x, qw, impl="reference"), rtol=1e-4, atol=1e-4)
    finally:
        k.set_fault_check(prev)


def test_selftest_argument_range(wq, cuda) -> None:
    with pytest.raises(ValueError):
        wq._kernels.selftest_expired_wait(0)
    assert wq._kernels.fault_status(reset=True) == 0
