"""Quantized weight storage and RTN quantization on the GPU.

Mirror of ptqkit's ``quant`` module (src/ptqkit/quant.py): the same
``QuantConfig``, ``QuantizedWeight`` (field for field, with the same invariant
checks, quant.py:98-137), ``quantize_weight`` and ``dequantize_weight``
signatures and error messages. The arithmetic runs in the CUDA library:
``quantize_weight`` is one device RTN + pack pass whose codes, scales, zeros and
packed bytes are bit-exact with the reference's (quant.py:146-289), and
``dequantize_weight`` reconstructs W_hat with the reference's per-element
operation order (quant.py:292-308).

Codes are unsigned integers q in [0, 2^bits - 1]; reconstruction is
W_hat[m, k] = scale[m, g] * (q[m, k] - zero[m, g]) * channel_scale[k], g = k // group_size.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Literal

import torch

from . import _kernels
from .pack import pack_int4

Granularity = Literal["tensor", "channel", "group"]


class Method(str, enum.Enum):
    RTN = "rtn"
    GPTQ = "gptq"
    AWQ = "awq"


@dataclass(frozen=True)
class QuantConfig:
    """Weight-only quantization configuration (quant.py:60-82). Activations stay fp32."""

    bits: int = 4
    symmetric: bool = True
    group_size: int | None = 128
    method: Method = Method.RTN
    percdamp: float = 0.01
    blocksize: int = 128
    awq_alphas: tuple[float, ...] = (0.0, 0.25, 0.5, 0.75, 1.0)

    def __post_init__(self) -> None:
        if self.bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        if self.group_size is not None and self.group_size < 0:
            raise ValueError("group_size must be None, 0, or positive")
        if self.percdamp < 0:
            raise ValueError("percdamp must be non-negative")
        if self.blocksize <= 0:
            raise ValueError("blocksize must be positive")
        if not self.awq_alphas:
            raise ValueError("awq_alphas must be non-empty")


def granularity_of(config: QuantConfig) -> Granularity:
    if config.group_size == 0:
        return "tensor"
    if config.group_size is None:
        return "channel"
    return "group"


def qmax_of(bits: int) -> int:
    return (1 << bits) - 1


@dataclass(frozen=True)
class QuantizedWeight:
    """Quantized [out, in] weight in ptqkit's layout (quant.py:97-137).

    ``codes`` is uint8 [out, in] for int8, or packed uint8 [out, ceil(in/2)] for int4.
    ``scales`` and ``zeros`` are float32 [scale_rows, groups] with scale_rows in {1, out}.
    ``group_size`` is the K-stride of a group; per-tensor and per-channel use K.
    ``channel_scale`` is an optional float32 [in] multiplier applied after the affine map.
    """

    codes: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    bits: int
    group_size: int
    in_features: int
    out_features: int
    symmetric: bool
    packed: bool
    granularity: Granularity
    channel_scale: torch.Tensor | None = None

    def __post_init__(self) -> None:
        if self.bits not in (4, 8):
            raise ValueError("bits must be 4 or 8")
        if self.group_size <= 0:
            raise ValueError("group_size must be positive")
        if self.packed != (self.bits == 4):
            raise ValueError("only int4 storage is packed")
        if self.scales.shape != self.zeros.shape:
            raise ValueError("scales and zeros must have the same shape")
        if self.scales.ndim != 2:
            raise ValueError("scales must have shape [rows, groups]")
        rows, groups = int(self.scales.shape[0]), int(self.scales.shape[1])
        if rows not in (1, self.out_features):
            raise ValueError("scale rows must be 1 or out_features")
        n_groups = (self.in_features + self.group_size - 1) // self.group_size
        if groups != n_groups:
            raise ValueError("scale groups do not match group_size")
        if self.channel_scale is not None and int(self.channel_scale.numel()) != self.in_features:
            raise ValueError("channel_scale must have one entry per input channel")

    def to(self, device: torch.device | str) -> QuantizedWeight:
        """Copy of this weight with every tensor on ``device``."""
        move = lambda t: None if t is None else t.to(device)  # noqa: E731
        return QuantizedWeight(
            codes=move(self.codes), scales=move(self.scales), zeros=move(self.zeros),
            bits=self.bits, group_size=self.group_size, in_features=self.in_features,
            out_features=self.out_features, symmetric=self.symmetric, packed=self.packed,
            granularity=self.granularity, channel_scale=move(self.channel_scale),
        )


def absolute_error_bound(scale: torch.Tensor, *, symmetric: bool) -> torch.Tensor:
    """Per-element RTN bound (quant.py:140-143): scale/2 symmetric, scale asymmetric."""
    factor = 0.5 if symmetric else 1.0
    return scale * factor


def _cuda(t: torch.Tensor) -> torch.Tensor:
    if t.device.type == "cuda":
        return t
    if not torch.cuda.is_available():
        raise RuntimeError("wq_b200 runs on CUDA devices; no CUDA device is available")
    return t.to(torch.device("cuda", torch.cuda.current_device()))


def assemble_quantized(
    codes: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    *,
    bits: int,
    group_size: int,
    symmetric: bool,
    granularity: Granularity,
    channel_scale: torch.Tensor | None = None,
) -> QuantizedWeight:
    """Pack ``codes`` [out, in] and attach fp32 scale/zero tensors (quant.py:187-222)."""
    if codes.ndim != 2:
        raise ValueError("codes must have shape [out, in]")
    codes = _cuda(codes)
    dev = codes.device
    out, inn = int(codes.shape[0]), int(codes.shape[1])
    packed = bits == 4
    stored_codes = pack_int4(codes) if packed else codes.to(dtype=torch.uint8)
    cs = None if channel_scale is None else channel_scale.detach().to(device=dev, dtype=torch.float32).contiguous()
    return QuantizedWeight(
        codes=stored_codes.contiguous(),
        scales=scales.detach().to(device=dev, dtype=torch.float32).contiguous(),
        zeros=zeros.detach().to(device=dev, dtype=torch.float32).contiguous(),
        bits=bits,
        group_size=group_size,
        in_features=inn,
        out_features=out,
        symmetric=symmetric,
        packed=packed,
        granularity=granularity,
        channel_scale=cs,
    )


def quantize_weight(
    weight: torch.Tensor,
    config: QuantConfig,
    *,
    pre_scale: torch.Tensor | None = None,
) -> QuantizedWeight:
    """Round-to-nearest quantize ``weight`` [out, in] on the GPU (quant.py:225-289).

    If ``pre_scale`` [in] is set, W diag(pre_scale) is quantized and the stored
    channel_scale is 1/pre_scale. A CPU ``weight`` is copied to the current CUDA
    device; the returned tensors live on the GPU.
    """
    if weight.ndim != 2:
        raise ValueError("weight must have shape [out, in]")
    w = _cuda(weight.detach()).to(dtype=torch.float32)
    pre = None
    if pre_scale is not None:
        pre = pre_scale.detach().to(dtype=torch.float32, device=w.device).reshape(-1)
        if int(pre.numel()) != int(w.shape[1]):
            # the reference checks finiteness first (quant.py:240-246)
            if not bool(torch.isfinite(w).all()):
                raise ValueError("weight must be finite")
            raise ValueError("pre_scale must have one entry per input channel")
    granularity = granularity_of(config)
    inn = int(w.shape[1])
    if granularity == "tensor":
        mode, index_group = 0, inn
    elif granularity == "channel":
        mode, index_group = -1, inn
    else:
        assert config.group_size is not None
        mode, index_group = int(config.group_size), int(config.group_size)
    r = _kernels.rtn_quantize(w, config.bits, config.symmetric, mode, pre)
    return QuantizedWeight(
        codes=r["codes"],
        scales=r["scales"],
        zeros=r["zeros"],
        bits=config.bits,
        group_size=index_group,
        in_features=inn,
        out_features=int(w.shape[0]),
        symmetric=config.symmetric,
        packed=config.bits == 4,
        granularity=granularity,
        channel_scale=r.get("channel_scale"),
    )


def dequantize_weight(qw: QuantizedWeight) -> torch.Tensor:
    """Reconstruct the fp32 [out, in] matrix on the GPU (quant.py:292-308)."""
    return _kernels.dequantize(
        qw.codes, qw.scales, qw.zeros, qw.channel_scale, qw.in_features, qw.group_size, qw.bits
    )


def element_scales(qw: QuantizedWeight) -> torch.Tensor:
    """Broadcast group scales to [out, in] (channel_scale is not included), quant.py:311-316."""
    idx = torch.arange(qw.in_features, device=qw.scales.device) // qw.group_size
    if int(qw.scales.shape[0]) == 1:
        return qw.scales[0, idx].unsqueeze(0).expand(qw.out_features, qw.in_features)
    return qw.scales[:, idx]
