"""The C-ABI library without a GPU: it loads, exports every entry point that
include/wq_b200.h declares, and rejects bad arguments on the host with the
reference's messages (src/ptqkit/csrc/dequant_gemm.cpp:235-277) before any
CUDA call is made."""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

from conftest import REPO, package

HEADER = os.path.join(REPO, "include", "wq_b200.h")


def _declared() -> list[str]:
    text = open(HEADER).read()
    return re.findall(r"WQ_API\s+[\w\s\*]+?\b(wq_\w+)\s*\(", text)


def test_header_declares_entry_points() -> None:
    names = _declared()
    assert "wq_dequant_gemm_f32" in names and "wq_rtn_quantize_f32" in names
    assert len(names) == len(set(names)) >= 12


def test_library_exports_every_declared_symbol(wq) -> None:
    lib = wq._kernels.library()
    for name in _declared():
        assert hasattr(lib, name), name
        assert name in wq._kernels.SIGNATURES, f"{name} has no ctypes signature"
    assert set(wq._kernels.SIGNATURES) == set(_declared())


REFERENCE_MESSAGES = {
    1: "x must have shape [B, K]",
    2: "q, scales, and zeros must be rank 2",
    3: "bits must be 4 or 8",
    4: "group_size must be positive",
    5: "negative dimension",
    6: "packed code row length does not match K",
    7: "zeros shape must match scales",
    8: "scale rows must be 1 or M",
    9: "scale groups must equal ceil(K / group_size)",
    10: "channel_scale must have shape [K]",
    15: "weight must be finite",
    16: "pre_scale must have one entry per input channel",
    17: "pre_scale must be finite and positive",
    18: "int4 codes must lie in [0, 15]",
    19: "group_size must be None, 0, or positive",
}


def test_status_strings_match_reference(wq) -> None:
    for code, msg in REFERENCE_MESSAGES.items():
        assert wq._kernels.status_message(code) == msg


def _call(wq, **kw):  # type: ignore[no-untyped-def]
    a = dict(x=None, B=2, K=8, q=None, M=3, q_cols=4, scales=None, scale_rows=3, groups=1, zeros=None,
             zero_rows=3, zero_groups=1, ch=None, ch_len=-1, group_size=8, bits=4, y=None, ldy=3,
             ws=None, ws_bytes=0, stream=None)
    a.update(kw)
    return wq._kernels.library().wq_dequant_gemm_f32(
        a["x"], a["B"], a["K"], a["q"], a["M"], a["q_cols"], a["scales"], a["scale_rows"], a["groups"],
        a["zeros"], a["zero_rows"], a["zero_groups"], a["ch"], a["ch_len"], a["group_size"], a["bits"],
        a["y"], a["ldy"], a["ws"], a["ws_bytes"], a["stream"])


def test_validation_order_and_codes(wq) -> None:
    assert _call(wq, bits=3) == 3
    assert _call(wq, group_size=0) == 4
    assert _call(wq, K=-1) == 5
    assert _call(wq, q_cols=5) == 6                       # int4: (K+1)//2 = 4
    assert _call(wq, bits=8, q_cols=4) == 6               # int8: K = 8
    assert _call(wq, zero_rows=1) == 7
    assert _call(wq, scale_rows=2, zero_rows=2) == 8
    assert _call(wq, group_size=3) == 9                   # ceil(8/3) = 3 != 1
    assert _call(wq, ch=ctypes.c_void_p(16), ch_len=7) == 10
    assert _call(wq, ldy=2) == 20
    assert _call(wq) == 11                                # valid shapes, null pointers
    assert _call(wq, B=0) == 0                            # nothing to do, no CUDA call
    assert _call(wq, K=0, q_cols=0, groups=5, zero_groups=5) == 11  # y is null
    # scale_rows == 1 broadcast is legal
    assert _call(wq, scale_rows=1, zero_rows=1) == 11


def test_multi_output_and_ipc_validation(wq) -> None:
    """The multi-output entry point runs the same validation as the single-output
    one, then checks the output count; the IPC calls reject null arguments."""
    lib = wq._kernels.library()

    def multi(n_out: int, outs=None, bits: int = 4, group_size: int = 8):  # type: ignore[no-untyped-def]
        return lib.wq_dequant_gemm_f32_multi(None, 1, 8, None, 2, 4, None, 2, 1, None, 2, 1, None, -1,
                                             group_size, bits, outs, n_out, 2, None, None, None, 0, None)

    assert multi(1, bits=3) == 3            # reference validation first
    assert multi(0) == 22                   # WQ_E_OUTPUTS
    assert multi(9) == 22
    assert multi(2) == 11                   # null output array
    arr = (ctypes.c_void_p * 2)(None, None)
    assert multi(2, outs=ctypes.cast(arr, ctypes.c_void_p)) == 11
    assert lib.wq_status_string(22).decode() == "output count must be between 1 and WQ_MAX_OUTPUTS"
    assert lib.wq_ipc_handle_bytes() == 64
    off = ctypes.c_int64(0)
    assert lib.wq_ipc_get_handle(None, None, ctypes.byref(off)) == 11
    ptr = ctypes.c_void_p(0)
    assert lib.wq_ipc_open_handle(None, 0, ctypes.byref(ptr)) == 11
    assert lib.wq_ipc_close_handle(None, 0) == 11


def test_rtn_and_pack_validation(wq) -> None:
    lib = wq._kernels.library()
    assert lib.wq_rtn_quantize_f32(None, None, 4, 4, 5, 1, 2, None, None, None, None, None, None, 0, None) == 3
    assert lib.wq_rtn_quantize_f32(None, None, 4, 4, 4, 1, -2, None, None, None, None, None, None, 0, None) == 19
    assert lib.wq_rtn_quantize_f32(None, None, -1, 4, 4, 1, 2, None, None, None, None, None, None, 0, None) == 5
    assert lib.wq_rtn_quantize_f32(None, None, 4, 4, 4, 1, 2, None, None, None, None, None, None, 0, None) == 11
    assert lib.wq_rtn_flags_status(0) == 0
    assert lib.wq_rtn_flags_status(1) == 15
    assert lib.wq_rtn_flags_status(2) == 17
    assert lib.wq_rtn_flags_status(3) == 15
    assert lib.wq_rtn_workspace_bytes(10, 10, 0) > 0
    assert lib.wq_rtn_workspace_bytes(10, 10, 4) == 0
    assert lib.wq_unpack_int4(None, 2, 3, 7, None, None) == 6
    assert lib.wq_pack_int4(None, 2, 3, None, None, None) == 11


def test_python_wrapper_mirrors_reference_errors(wq) -> None:
    k = wq._kernels
    with pytest.raises(ValueError, match=r"x must have shape \[B, K\]"):
        k.dequant_gemm(torch.zeros(3), torch.zeros(2, 2), torch.zeros(2, 1), torch.zeros(2, 1), None, 4, 4)
    with pytest.raises(ValueError, match="q, scales, and zeros must be rank 2"):
        k.dequant_gemm(torch.zeros(1, 4), torch.zeros(2), torch.zeros(2, 1), torch.zeros(2, 1), None, 4, 4)
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        k.dequant_gemm(torch.zeros(1, 4), torch.zeros(2, 2), torch.zeros(2, 1), torch.zeros(2, 1), None, 4, 4)
    qw = wq.QuantizedWeight(
        codes=torch.zeros(2, 2, dtype=torch.uint8), scales=torch.ones(2, 1), zeros=torch.zeros(2, 1), bits=4,
        group_size=4, in_features=4, out_features=2, symmetric=True, packed=True, granularity="channel")
    with pytest.raises(ValueError, match="impl must be 'reference' or 'kernel'"):
        wq.dequant_gemm(torch.zeros(1, 4), qw, impl="fast")
    with pytest.raises(ValueError, match="x has trailing dim 3, weight expects 4"):
        wq.dequant_gemm(torch.zeros(1, 3), qw, impl="kernel")
    with pytest.raises(RuntimeError, match="the dequant kernel runs on CUDA"):
        wq.dequant_gemm(torch.zeros(1, 4), qw, impl="kernel")


def test_kernel_info_without_gpu(wq) -> None:
    info = wq._kernels.kernel_info(0)
    assert info["arch"] == "sm_100a"
    assert info["abi_version"] == 1


def test_package_has_no_oracle_dependency() -> None:
    """The product package must not import or load the oracle (or any CPU fallback)."""
    pkg_dir = os.path.join(REPO, "weight-quantizer_b200")
    for root, _dirs, files in os.walk(pkg_dir):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(root, f)).read()
                assert "import oracle" not in text and "liboracle" not in text and "oracle/" not in text, f
    assert package() is not None
