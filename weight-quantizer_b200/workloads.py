"""Seeded synthetic inputs for the five dequant-GEMM workloads.

No dataset or checkpoint is involved: every workload is random data of the
shape, scale and distribution named for it, generated on the CPU with one
``torch.Generator().manual_seed(0)`` per workload in a fixed order (weights
first, then the pre-scale inputs, then the activations; the order ptqkit's
own kernel test uses, tests/test_gemm.py:47-58), so every process that calls
these functions sees the same bytes.

  gpt2_c_fc_int4_g128   W [3072, 768] ~ N(0, 0.02), int4 symmetric g128, x [8, 768] ~ N(0, 1)
  gpt2_small_int8_asym  12 GPT-2-small blocks (c_attn 2304x768, attn c_proj 768x768,
                        c_fc 3072x768, mlp c_proj 768x3072), W ~ N(0, 0.02), int8
                        asymmetric per-channel; x ~ N(0, 1) at batch 1 and 8
  awq_11008x4096        W [11008, 4096] ~ N(0, 0.02), int4 asymmetric g128 with an AWQ
                        pre-scale s = m^0.5 / mean(m^0.5), m ~ LogNormal(0, 1);
                        x [16, 4096] ~ N(0, 1) with 41 (1%) random channels x20
  oddk_4096x4095_g64    W [4096, 4095] ~ N(0, 0.02), int4 symmetric g64; x at batch 1, 4, 32
  sharded_28672x8192    W [28672, 8192] ~ N(0, 0.015), int4 symmetric g128; x ~ N(0, 1)
                        at batch 1, 32, 256, 4096
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .quant import QuantConfig


@dataclass
class Layer:
    name: str
    weight: torch.Tensor                      # fp32 [out, in], CPU
    config: QuantConfig
    pre_scale: torch.Tensor | None = None     # fp32 [in], CPU
    x: dict[int, torch.Tensor] = field(default_factory=dict)  # batch -> fp32 [B, in], CPU


GPT2_SMALL_LINEARS = (("c_attn", 2304, 768), ("attn_c_proj", 768, 768), ("c_fc", 3072, 768), ("mlp_c_proj", 768, 3072))


def gpt2_c_fc_int4_g128() -> list[Layer]:
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3072, 768, generator=g) * 0.02
    x = torch.randn(8, 768, generator=g)
    return [Layer("c_fc", w, QuantConfig(bits=4, symmetric=True, group_size=128), x={8: x})]


def gpt2_small_int8_asym(blocks: int = 12, batches: tuple[int, ...] = (1, 8)) -> list[Layer]:
    g = torch.Generator().manual_seed(0)
    cfg = QuantConfig(bits=8, symmetric=False, group_size=None)
    layers = []
    for blk in range(blocks):
        for name, out_f, in_f in GPT2_SMALL_LINEARS:
            layers.append(Layer(f"h{blk}.{name}", torch.randn(out_f, in_f, generator=g) * 0.02, cfg))
    for b in batches:
        for layer in layers:
            layer.x[b] = torch.randn(b, int(layer.weight.shape[1]), generator=g)
    return layers


def awq_11008x4096() -> list[Layer]:
    g = torch.Generator().manual_seed(0)
    w = torch.randn(11008, 4096, generator=g) * 0.02
    m = torch.empty(4096).log_normal_(0.0, 1.0, generator=g)
    r = m.pow(0.5)
    s = r / r.mean()
    x = torch.randn(16, 4096, generator=g)
    idx = torch.randperm(4096, generator=g)[:41]
    x[:, idx] *= 20.0
    return [Layer("awq", w, QuantConfig(bits=4, symmetric=False, group_size=128), pre_scale=s, x={16: x})]


def oddk_4096x4095_g64(batches: tuple[int, ...] = (1, 4, 32)) -> list[Layer]:
    g = torch.Generator().manual_seed(0)
    w = torch.randn(4096, 4095, generator=g) * 0.02
    xs = {b: torch.randn(b, 4095, generator=g) for b in batches}
    return [Layer("oddk", w, QuantConfig(bits=4, symmetric=True, group_size=64), x=xs)]


def sharded_28672x8192(batches: tuple[int, ...] = (1, 32, 256, 4096)) -> list[Layer]:
    g = torch.Generator().manual_seed(0)
    w = torch.randn(28672, 8192, generator=g) * 0.015
    xs = {}
    for b in (1, 32, 256, 4096):
        x = torch.randn(b, 8192, generator=g)
        if b in batches:
            xs[b] = x
    return [Layer("sharded", w, QuantConfig(bits=4, symmetric=True, group_size=128), x=xs)]


WORKLOADS = {
    "gpt2_c_fc_int4_g128": gpt2_c_fc_int4_g128,
    "gpt2_small_int8_asym": gpt2_small_int8_asym,
    "awq_11008x4096": awq_11008x4096,
    "oddk_4096x4095_g64": oddk_4096x4095_g64,
    "sharded_28672x8192": sharded_28672x8192,
}
