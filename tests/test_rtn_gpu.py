"""RTN quantize + pack on the GPU: bit-exact with the reference's outputs.

Codes, scales, zeros (compared as int32 bit patterns, so -0.0 zero points
count), channel scales and packed bytes must be identical to what ptqkit's
quantize_weight (src/ptqkit/quant.py:225-289) produced for the golden inputs,
at full size for the five workloads (SHA-256 digests).
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from conftest import sha, small_cases, workload_digests

pytestmark = pytest.mark.gpu


def test_pack_known_answer(wq, cuda) -> None:
    # tests/test_pack.py:6-25
    data, _ = small_cases()
    packed = wq.pack_int4(torch.from_numpy(data["kat_pack.codes"]).to(cuda))
    assert packed[0, 0].item() == 0x21 and packed[0, 1].item() == 0x0F and packed[1, 0].item() == 0xF0
    assert torch.equal(wq.unpack_int4(packed, 4).cpu(), torch.from_numpy(data["kat_pack.codes"]).to(torch.uint8))
    odd = wq.pack_int4(torch.from_numpy(data["pack_odd.codes"]).to(cuda))
    assert tuple(odd.shape) == (5, 4)
    assert np.array_equal(odd.cpu().numpy(), data["pack_odd.packed"])
    codes = torch.randint(0, 16, (13, 128), device=cuda, dtype=torch.int32)
    assert torch.equal(wq.unpack_int4(wq.pack_int4(codes), 128), codes.to(torch.uint8))


def test_pack_range_error(wq, cuda) -> None:
    with pytest.raises(ValueError, match=r"int4 codes must lie in \[0, 15\], got \[-1, 16\]"):
        wq.pack_int4(torch.tensor([[0, -1, 16]], device=cuda))
    with pytest.raises(ValueError, match="packed row is shorter than in_features"):
        wq.unpack_int4(torch.zeros(2, 2, dtype=torch.uint8, device=cuda), 5)


def test_rtn_bit_exact_small(wq, cuda) -> None:
    data, meta = small_cases()
    n = 0
    for m in meta:
        if m["kind"] != "rtn":
            continue
        name = m["name"]
        pre = data.get(f"{name}.pre")
        cfg = wq.QuantConfig(bits=m["bits"], symmetric=m["symmetric"], group_size=m["group"])
        qw = wq.quantize_weight(torch.from_numpy(data[f"{name}.w"]).to(cuda), cfg,
                                pre_scale=None if pre is None else torch.from_numpy(pre).to(cuda))
        assert np.array_equal(qw.codes.cpu().numpy(), data[f"{name}.q"]), name
        assert np.array_equal(qw.scales.cpu().numpy().view(np.int32), data[f"{name}.scales"].view(np.int32)), name
        assert np.array_equal(qw.zeros.cpu().numpy().view(np.int32), data[f"{name}.zeros"].view(np.int32)), name
        assert qw.group_size == m["stored_group"]
        if pre is not None:
            assert np.array_equal(qw.channel_scale.cpu().numpy().view(np.int32),
                                  data[f"{name}.channel"].view(np.int32)), name
        n += 1
    assert n > 200


def test_dequantize_bit_exact(wq, cuda) -> None:
    """dequantize_weight: ((code - zero) * scale) * channel in fp32, per element (quant.py:292-308)."""
    data, meta = small_cases()
    for m in meta:
        if m["kind"] != "rtn":
            continue
        name = m["name"]
        w = data[f"{name}.w"]
        M, K = w.shape
        q = data[f"{name}.q"]
        codes = q.astype(np.float32) if m["bits"] == 8 else np.stack(
            [q & 0x0F, q >> 4], axis=2).reshape(M, -1)[:, :K].astype(np.float32)
        G = m["stored_group"]
        idx = np.arange(K) // G
        sc, ze = data[f"{name}.scales"], data[f"{name}.zeros"]
        if sc.shape[0] > 1:
            s, z = sc[:, idx], ze[:, idx]
        else:
            s, z = np.broadcast_to(sc[0, idx], (M, K)), np.broadcast_to(ze[0, idx], (M, K))
        hat = ((codes - z).astype(np.float32) * s).astype(np.float32)
        ch = data.get(f"{name}.channel")
        if ch is not None:
            hat = (hat * ch[None, :]).astype(np.float32)
        qw = wq.QuantizedWeight(
            codes=torch.from_numpy(q).to(cuda), scales=torch.from_numpy(sc).to(cuda),
            zeros=torch.from_numpy(ze).to(cuda), bits=m["bits"], group_size=G, in_features=K, out_features=M,
            symmetric=m["symmetric"], packed=m["bits"] == 4, granularity="group",
            channel_scale=None if ch is None else torch.from_numpy(ch).to(cuda))
        got = wq.dequantize_weight(qw).cpu().numpy()
        assert np.array_equal(got.view(np.int32), hat.view(np.int32)), name


def test_rtn_errors(wq, cuda) -> None:
    cfg = wq.QuantConfig(bits=4, symmetric=True, group_size=4)
    w = torch.randn(3, 8, device=cuda)
    bad = w.clone()
    bad[1, 2] = float("nan")
    with pytest.raises(ValueError, match="weight must be finite"):
        wq.quantize_weight(bad, cfg)
    bad[1, 2] = float("inf")
    with pytest.raises(ValueError, match="weight must be finite"):
        wq.quantize_weight(bad, cfg, pre_scale=torch.ones(8, device=cuda))
    with pytest.raises(ValueError, match="pre_scale must have one entry per input channel"):
        wq.quantize_weight(w, cfg, pre_scale=torch.ones(7, device=cuda))
    with pytest.raises(ValueError, match="pre_scale must be finite and positive"):
        wq.quantize_weight(w, cfg, pre_scale=torch.zeros(8, device=cuda))
    # a later good call is unaffected
    assert wq.quantize_weight(w, cfg).codes.shape == (3, 4)


def test_rtn_error_bounds_and_shapes(wq, cuda) -> None:
    """Properties of tests/test_quant.py:13-60 on the GPU path."""
    g = torch.Generator().manual_seed(0)
    tensors = [torch.randn(17, 32, generator=g), torch.randn(4, 7, generator=g), torch.randn(8, 128, generator=g),
               torch.linspace(-1.5, 2.0, 128).reshape(4, 32), torch.zeros(4, 8), torch.full((3, 16), 0.5)]
    for w in tensors:
        for bits in (4, 8):
            for sym in (True, False):
                for group in (0, None, 16):
                    cfg = wq.QuantConfig(bits=bits, symmetric=sym, group_size=group)
                    qw = wq.quantize_weight(w.to(cuda), cfg)
                    hat = wq.dequantize_weight(qw)
                    err = (w.to(cuda) - hat).abs()
                    limit = wq.absolute_error_bound(wq.element_scales(qw), symmetric=sym) + 1e-4
                    assert torch.all(err <= limit)
    weight = torch.randn(6, 40, generator=g).to(cuda)
    tensor = wq.quantize_weight(weight, wq.QuantConfig(8, True, 0))
    channel = wq.quantize_weight(weight, wq.QuantConfig(8, False, None))
    group = wq.quantize_weight(weight, wq.QuantConfig(4, True, 16))
    assert tensor.scales.shape == (1, 1) and tensor.granularity == "tensor" and tensor.group_size == 40
    assert channel.scales.shape == (6, 1) and channel.granularity == "channel"
    assert group.scales.shape == (6, 3) and group.packed and group.codes.dtype == torch.uint8
    assert group.codes.shape == (6, 20)


@pytest.mark.parametrize("wname", ["gpt2_c_fc_int4_g128", "gpt2_small_int8_asym", "awq_11008x4096",
                                   "oddk_4096x4095_g64", "sharded_28672x8192"])
def test_rtn_workloads_bit_exact(wq, cuda, wname: str) -> None:
    wl = importlib.import_module("weight-quantizer_b200.workloads")
    dig = workload_digests()[wname]
    for layer, d in zip(wl.WORKLOADS[wname](), dig):
        assert sha(layer.weight) == d["w"]
        qw = wq.quantize_weight(layer.weight.to(cuda), layer.config,
                                pre_scale=None if layer.pre_scale is None else layer.pre_scale.to(cuda))
        assert sha(qw.codes) == d["q"], f"{wname}/{layer.name} codes"
        assert sha(qw.scales) == d["scales"], f"{wname}/{layer.name} scales"
        assert sha(qw.zeros) == d["zeros"], f"{wname}/{layer.name} zeros"
        assert qw.group_size == d["group_size"]
        if layer.pre_scale is not None:
            assert sha(qw.channel_scale) == d["channel"]
