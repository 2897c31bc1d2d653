"""The operator boundary: ``dequant_gemm`` (mirror of src/ptqkit/gemm.py).

Both implementations compute y = x @ W_hat^T for a ``QuantizedWeight``:

* ``impl="kernel"`` runs the sm_100a dequant-GEMM of the C-ABI library on the
  weight as stored (packed codes, group scales/zeros, optional channel scale),
  where ptqkit's ``kernel`` ran its OpenMP/AVX2 CPU kernel (gemm.py:43-58).
  Decode-shaped batches take the streaming kernel, other shapes the tiled one.
* ``impl="reference"`` is ptqkit's reference formulation (gemm.py:41-42): the
  dense W_hat from ``dequantize_weight`` followed by an fp32 matmul.

Inputs must be CUDA tensors (the reference's kernel refused non-CPU tensors,
gemm.py:44-45; this one refuses non-CUDA tensors). Results are written on the
current CUDA stream and returned without a host synchronization.
"""

from __future__ import annotations

from typing import Any

import torch

from . import _kernels
from .quant import QuantizedWeight, dequantize_weight


def kernel_info() -> dict[str, Any]:
    """Build facts of the CUDA library and the current device (gemm.py:22-24)."""
    return _kernels.kernel_info()


def dequant_gemm(
    x: torch.Tensor,
    qw: QuantizedWeight,
    *,
    impl: str = "reference",
    nthreads: int = 0,
    out: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """Apply a quantized weight. ``x`` is [..., in]. Output is [..., out] (gemm.py:27-59).

    ``nthreads`` is accepted for signature compatibility and ignored. ``out``
    (kernel path) may be a preallocated fp32 [N, out] tensor for the flattened
    batch; it is returned reshaped. ``bias`` (an extension: ptqkit adds the
    bias in ``QuantizedLinear.forward``, linear.py:99-100) is added to every
    output row, in the kernels' epilogue on the kernel path; the result is the
    same single fp32 add.
    """
    if impl not in ("reference", "kernel"):
        raise ValueError("impl must be 'reference' or 'kernel'")
    if x.shape[-1] != qw.in_features:
        raise ValueError(f"x has trailing dim {x.shape[-1]}, weight expects {qw.in_features}")
    lead = x.shape[:-1]
    flat = x.detach().reshape(-1, qw.in_features).to(dtype=torch.float32)
    if impl == "reference":
        y = flat @ dequantize_weight(qw).transpose(0, 1)
        if bias is not None:
            y = y + bias
    else:
        if flat.device.type != "cuda":
            raise RuntimeError("the dequant kernel runs on CUDA")
        y = _kernels.dequant_gemm(
            flat,
            qw.codes.detach(),
            qw.scales.detach(),
            qw.zeros.detach(),
            None if qw.channel_scale is None else qw.channel_scale.detach(),
            int(qw.group_size),
            int(qw.bits),
            int(nthreads),
            out=out,
            bias=None if bias is None else bias.detach(),
        )
    return y.reshape(*lead, qw.out_features)
