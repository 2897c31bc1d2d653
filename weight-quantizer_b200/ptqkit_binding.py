"""Run ptqkit's own modules on B200: the binding a ptqkit maintainer adds.

ptqkit's operator ``gemm.dequant_gemm(x, qw, *, impl, nthreads)``
(src/ptqkit/gemm.py:27-59) sends ``impl="kernel"`` to its compiled CPU module
and refuses other devices (gemm.py:44-45). The drop-in is one more branch in
front of that guard: CUDA inputs go to this library's C ABI
(``wq_dequant_gemm_f32`` through ``_kernels.dequant_gemm``, the same
arguments as ptqkit's ``_kernels.dequant_gemm``), everything else to ptqkit's
code as before. ``install(ptqkit)`` adds that branch at run time, to
``ptqkit.gemm.dequant_gemm`` and to the names that imported it
(``ptqkit.linear.dequant_gemm``, ``ptqkit.dequant_gemm``), so ptqkit's own
``QuantizedLinear.forward`` (linear.py:90-101) and the models that
``quantize_model(..., kernel=True)`` (convert.py:236-293) returns run the
sm_100a kernels once they are moved to a CUDA device.
"""

from __future__ import annotations

from collections.abc import Callable
from types import ModuleType
from typing import Any

import torch

from . import _kernels


def dequant_gemm_cuda(x: torch.Tensor, qw: Any, nthreads: int = 0) -> torch.Tensor:
    """y = x @ W_hat^T for ptqkit's QuantizedWeight ``qw`` and a CUDA ``x`` [..., in]."""
    if x.shape[-1] != qw.in_features:
        raise ValueError(f"x has trailing dim {x.shape[-1]}, weight expects {qw.in_features}")
    flat = x.detach().reshape(-1, qw.in_features).to(dtype=torch.float32)
    y = _kernels.dequant_gemm(
        flat, qw.codes.detach(), qw.scales.detach(), qw.zeros.detach(),
        None if qw.channel_scale is None else qw.channel_scale.detach(),
        int(qw.group_size), int(qw.bits), int(nthreads),
    )
    return y.reshape(*x.shape[:-1], qw.out_features)


def install(ptqkit: ModuleType) -> Callable[[], None]:
    """Route ptqkit's ``impl="kernel"`` calls on CUDA tensors to this library.

    Returns a function that puts ptqkit's original operator back."""
    gemm = ptqkit.gemm
    original = gemm.dequant_gemm

    def dequant_gemm(x: torch.Tensor, qw: Any, *, impl: str = "reference", nthreads: int = 0) -> torch.Tensor:
        if impl == "kernel" and x.device.type == "cuda":
            return dequant_gemm_cuda(x, qw, nthreads)
        return original(x, qw, impl=impl, nthreads=nthreads)

    dequant_gemm.__doc__ = original.__doc__
    patched = []
    for mod in (gemm, getattr(ptqkit, "linear", None), ptqkit):
        if mod is not None and getattr(mod, "dequant_gemm", None) is original:
            setattr(mod, "dequant_gemm", dequant_gemm)
            patched.append(mod)

    def restore() -> None:
        for mod in patched:
            setattr(mod, "dequant_gemm", original)

    return restore
