"""``QuantizedLinear``: a Linear / GPT-2 Conv1D whose weight stays quantized on the GPU.

The module holds ptqkit's storage (``QuantizedWeight``: codes, scales, zeros,
optional AWQ channel scale) as buffers with ptqkit's names, which is what the
compressed on-disk format (src/ptqkit/convert.py:296-336) keys on, and
computes ``y = x @ W_hat^T + bias``:

* ``impl="kernel"``: the sm_100a dequant-GEMM straight from the stored codes,
  with the bias added in the kernel's epilogue (the same single fp32 add as
  ptqkit's ``y + bias``, src/ptqkit/linear.py:99-100);
* ``impl="reference"``: ptqkit's dense formulation, W_hat then a matmul.

``materialize()`` keeps a dense W_hat so later calls are one fp32 GEMM (what
ptqkit's sequential calibration relies on); moving the module drops it.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any

import torch
from torch import nn

from .gemm import dequant_gemm
from .quant import QuantizedWeight, dequantize_weight

_IMPLS = ("reference", "kernel")
# QuantizedWeight fields that are plain metadata (the tensors become buffers)
_META = ("bits", "group_size", "in_features", "out_features", "symmetric", "packed", "granularity")


class QuantizedLinear(nn.Module):
    """Linear layer over a ``QuantizedWeight`` (see the module docstring)."""

    codes: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    channel_scale: torch.Tensor | None
    bias: torch.Tensor | None

    def __init__(self, qw: QuantizedWeight, bias: torch.Tensor | None, *, impl: str = "reference") -> None:
        super().__init__()
        if impl not in _IMPLS:
            raise ValueError("impl must be 'reference' or 'kernel'")
        self.impl = impl
        self.awq_alpha: float | None = None   # set by the AWQ calibration
        self._meta: dict[str, Any] = {k: getattr(qw, k) for k in _META}
        for name in ("codes", "scales", "zeros", "channel_scale"):
            t = getattr(qw, name)
            self.register_buffer(name, None if t is None else t.detach().contiguous())
        if bias is not None:
            b = bias.detach().to(dtype=torch.float32).reshape(-1).contiguous()
            if int(b.numel()) != qw.out_features:
                raise ValueError("bias does not match out_features")
            bias = b
        self.register_buffer("bias", bias)
        self._dense: torch.Tensor | None = None

    def __getattr__(self, name: str) -> Any:
        meta = self.__dict__.get("_meta")
        if meta is not None and name in meta:
            return meta[name]
        return super().__getattr__(name)

    def quantized_weight(self) -> QuantizedWeight:
        return QuantizedWeight(codes=self.codes, scales=self.scales, zeros=self.zeros,
                               channel_scale=self.channel_scale, **self._meta)

    def materialize(self) -> None:
        """Keep the dense reconstruction W_hat; forward becomes one fp32 GEMM."""
        self._dense = dequantize_weight(self.quantized_weight())

    def clear_cache(self) -> None:
        self._dense = None

    def _apply(self, fn: Callable[..., Any], recurse: bool = True) -> QuantizedLinear:
        self._dense = None   # a moved or cast module rebuilds W_hat on demand
        super()._apply(fn, recurse=recurse)  # type: ignore[no-untyped-call]
        return self

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n_in = self._meta["in_features"]
        if x.shape[-1] != n_in:
            raise ValueError(f"expected in_features={n_in}, got {x.shape[-1]}")
        if self._dense is not None:
            flat = x.reshape(-1, n_in)
            y = nn.functional.linear(flat, self._dense, self.bias)
            return y.reshape(*x.shape[:-1], self._meta["out_features"])
        return dequant_gemm(x, self.quantized_weight(), impl=self.impl, bias=self.bias)

    def extra_repr(self) -> str:
        m = self._meta
        tail = "" if self.awq_alpha is None else f", awq_alpha={self.awq_alpha}"
        return (f"in={m['in_features']}, out={m['out_features']}, bits={m['bits']}, group={m['group_size']}, "
                f"sym={m['symmetric']}, impl={self.impl}{tail}")
