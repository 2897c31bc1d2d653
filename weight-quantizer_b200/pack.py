"""int4 packing on the GPU (mirror of src/ptqkit/pack.py).

Layout, row-major over the input dimension K:

    packed[m, j] = (q[m, 2j] & 15) | ((q[m, 2j + 1] & 15) << 4)

Index 2j is the low nibble, index 2j+1 the high nibble. An odd K is padded
with a zero code; the pad nibble is not part of the logical row and is never
consumed by the dequant-GEMM.
"""

from __future__ import annotations

import torch

from . import _kernels


def _cuda(t: torch.Tensor) -> torch.Tensor:
    if t.device.type == "cuda":
        return t
    if not torch.cuda.is_available():
        raise RuntimeError("wq_b200 runs on CUDA devices; no CUDA device is available")
    return t.to(torch.device("cuda", torch.cuda.current_device()))


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """Pack integer codes [M, K] into uint8 [M, ceil(K/2)] (pack.py:17-33)."""
    if codes.ndim != 2:
        raise ValueError("codes must have shape [M, K]")
    return _kernels.pack_int4(_cuda(codes))


def unpack_int4(packed: torch.Tensor, in_features: int) -> torch.Tensor:
    """Invert ``pack_int4`` and drop the pad nibble past ``in_features`` (pack.py:36-55)."""
    if packed.ndim != 2 or packed.dtype != torch.uint8:
        raise ValueError("packed int4 storage must be a uint8 matrix")
    return _kernels.unpack_int4(_cuda(packed), in_features)
