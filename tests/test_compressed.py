"""ptqkit's compressed format (version 1) and the GPU loader.

Pinned on files written by ptqkit itself (tests/golden/make_compressed.py runs
its quantize_model + save_compressed, src/ptqkit/convert.py:236-374, and its
compiled kernel for the expected layer outputs). CPU part: the files' format,
the byte counters, the model builder's seeds and the argument errors. GPU
part: the fp16 <-> fp32 passes bit for bit against torch's CPU conversions,
loading every reference file into a model (buffers bit-identical to the file's
values widened to fp32, layer outputs within the dequant-GEMM tolerance of the
reference kernel's), and writing: the file this package saves after its own
GPU quantize_model is byte-identical to ptqkit's for the same model.
"""

from __future__ import annotations

import importlib.util
import json
import os
from typing import Any

import numpy as np
import pytest
import torch
from torch import nn

from conftest import GOLDEN, assert_close_y, package

with open(os.path.join(GOLDEN, "compressed_ref.json")) as _f:
    INFO: dict[str, dict[str, Any]] = json.load(_f)
CASES = sorted(INFO)


def _models() -> Any:
    spec = importlib.util.spec_from_file_location("make_compressed", os.path.join(GOLDEN, "make_compressed.py"))
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MODELS = _models()


def _path(case: str) -> str:
    return os.path.join(GOLDEN, f"compressed_{case}.pt")


def _golden_y() -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, "compressed_ref.npz")) as z:
        return {k: z[k] for k in z.files}


def _cpu_layer(wq: Any, state: dict[str, Any], name: str) -> Any:
    """A CPU QuantizedLinear holding a file's layer (fp16 widened by torch):
    only for the byte counters, which read shapes and dtypes."""
    t, m = state["tensors"], state["meta"][name]
    p = f"{name}." if name else ""
    ch = t.get(p + "channel_scale")
    qw = wq.QuantizedWeight(
        codes=t[p + "codes"], scales=t[p + "scales"].float(), zeros=t[p + "zeros"].float(),
        bits=m["bits"], group_size=m["group_size"], in_features=m["in_features"],
        out_features=m["out_features"], symmetric=m["symmetric"], packed=m["packed"],
        granularity=m["granularity"], channel_scale=None if ch is None else ch.float(),
    )
    layer = wq.QuantizedLinear(qw, t.get(p + "bias"))
    layer.awq_alpha = m["awq_alpha"]
    return layer


# ----------------------------------------------------------------------------- CPU


@pytest.mark.parametrize("case", CASES)
def test_reference_files_format(case: str) -> None:
    wq = package()
    info = INFO[case]
    state = wq.read_compressed(_path(case))
    assert state["version"] == 1
    assert sorted(state["meta"]) == info["layers"]
    assert wq.payload_nbytes(state) == info["payload_nbytes"]
    assert os.path.getsize(_path(case)) == info["file_bytes"]
    for name, m in state["meta"].items():
        assert m["bits"] == info["bits"] and m["symmetric"] == info["symmetric"]
        assert (m["awq_alpha"] is not None) == (info["method"] == "awq")
        t = state["tensors"]
        assert t[f"{name}.codes"].dtype == torch.uint8
        assert t[f"{name}.scales"].dtype == torch.float16
        assert t[f"{name}.zeros"].dtype == torch.float16
        assert (f"{name}.channel_scale" in t) == (info["method"] == "awq")
        if f"{name}.bias" in t:
            assert t[f"{name}.bias"].dtype == torch.float32


@pytest.mark.parametrize("case", CASES)
def test_model_builder_and_byte_counters(case: str) -> None:
    wq = package()
    info = INFO[case]
    model = MODELS.make_model(info["seed"])
    assert MODELS.state_digest(model) == info["state_sha256"]
    state = wq.read_compressed(_path(case))
    for name in state["meta"]:
        setattr(model, name, _cpu_layer(wq, state, name))
    assert wq.matrix_nbytes(model) == info["matrix_nbytes"]
    assert wq.state_dict_nbytes(model) == info["state_dict_nbytes"]


def test_argument_errors(tmp_path: Any) -> None:
    wq = package()
    state = wq.read_compressed(_path("rtn_int4_g32"))
    bad = dict(state, version=2)
    torch.save(bad, tmp_path / "v2.pt")
    with pytest.raises(ValueError, match="version 2"):
        wq.read_compressed(tmp_path / "v2.pt")
    with pytest.raises(ValueError, match="not a compressed state"):
        wq.load_compressed_layers({"tensors": {}}, device="cuda:0")
    with pytest.raises(ValueError, match="CUDA device"):
        wq.load_compressed_layers(state, device="cpu")
    missing = dict(state, tensors={k: v for k, v in state["tensors"].items() if k != "up.zeros"})
    with pytest.raises(ValueError, match="no tensor 'up.zeros'"):
        wq.load_compressed_layers(missing, device="cuda:0")
    wrong = dict(state, tensors=dict(state["tensors"], **{"up.scales": state["tensors"]["up.scales"].float()}))
    with pytest.raises(ValueError, match="must be torch.float16"):
        wq.load_compressed_layers(wrong, device="cuda:0")
    # writing reads the layers' buffers on the GPU only
    model = MODELS.make_model(1)
    model.up = _cpu_layer(wq, state, "up")
    with pytest.raises(RuntimeError, match="CUDA device"):
        wq.compressed_state(model)


# ----------------------------------------------------------------------------- GPU


@pytest.mark.gpu
def test_widen_every_fp16_pattern() -> None:
    wq = package()
    bits = torch.from_numpy(np.arange(65536, dtype=np.uint16).view(np.float16).copy())
    ref = bits.float()
    for src in (bits, bits[1:], bits[3:65531]):  # aligned vector body; unaligned element path
        got = wq._kernels.widen_f16_f32(src.cuda()).cpu()
        want = src.float()
        nan = torch.isnan(want)
        assert torch.equal(torch.isnan(got), nan)
        assert torch.equal(got[~nan].view(torch.int32), want[~nan].view(torch.int32))
    assert ref.numel() == 65536


@pytest.mark.gpu
def test_narrow_matches_cpu_rounding() -> None:
    wq = package()
    g = torch.Generator().manual_seed(7)
    n = 1 << 20
    mag = torch.pow(10.0, torch.empty(n, dtype=torch.float64).uniform_(-9, 6, generator=g))
    sign = torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0).double()
    rand = (torch.randn(n, generator=g, dtype=torch.float64).abs() * mag * sign).float()
    # exact midpoints between adjacent fp16 values (ties), incl. subnormals and the overflow edge
    h = torch.from_numpy(np.arange(0, 0x7BFF, 7, dtype=np.uint16).view(np.float16).copy()).double()
    nxt = torch.from_numpy((np.arange(0, 0x7BFF, 7, dtype=np.uint16) + 1).view(np.float16).copy()).double()
    ties = ((h + nxt) / 2).float()
    edges = torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 65504.0, 65519.99, 65520.0, -65520.0,
                          2.0**-24, 2.0**-25, 3 * 2.0**-26, 2.0**-26, 6.1e-5, 1e-40, -1e-40], dtype=torch.float32)
    vals = torch.cat([rand, ties, -ties, edges])
    for src in (vals, vals[1:], vals[5:-3]):
        got = wq._kernels.narrow_f32_f16(src.cuda()).cpu()
        want = src.to(torch.float16)
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_load_reference_file(case: str) -> None:
    wq = package()
    dev = torch.device("cuda", 0)
    info = INFO[case]
    state = wq.read_compressed(_path(case))
    t = state["tensors"]
    ys = _golden_y()
    model = MODELS.make_model(info["seed"] + 100)  # different values: all must come from the file
    loaded = wq.load_compressed(_path(case), model, device=dev)
    assert loaded is model
    storages = set()
    for name, m in state["meta"].items():
        layer = model.get_submodule(name)
        assert isinstance(layer, wq.QuantizedLinear) and layer.impl == "kernel"
        assert layer.codes.device == dev and layer.awq_alpha == m["awq_alpha"]
        assert (layer.bits, layer.group_size, layer.granularity) == (m["bits"], m["group_size"], m["granularity"])
        assert torch.equal(layer.codes.cpu(), t[f"{name}.codes"])
        for part in ("scales", "zeros", "channel_scale"):
            if f"{name}.{part}" in t:
                got = getattr(layer, part).cpu()
                assert torch.equal(got.view(torch.int32), t[f"{name}.{part}"].float().view(torch.int32)), part
            else:
                assert getattr(layer, part, None) is None
        if f"{name}.bias" in t:
            assert torch.equal(layer.bias.cpu(), t[f"{name}.bias"])
        else:
            assert layer.bias is None
        storages.add(layer.codes.untyped_storage().data_ptr())
        x = torch.from_numpy(ys[f"{case}.x.{name}"])
        y = layer(x.to(dev)).cpu().numpy()
        assert_close_y(y, ys[f"{case}.y.{name}"], f"{case}/{name}")
    assert len(storages) == 1  # every layer's codes live in the one uploaded block
    for key, ref in t.items():
        if key.startswith("param."):
            got = model.get_parameter(key[len("param."):])
        elif key.startswith("buffer."):
            got = model.get_buffer(key[len("buffer."):])
        else:
            continue
        assert got.device == dev and torch.equal(got.cpu(), ref), key
    ids = torch.randint(0, 32, (2, 8)).to(dev)
    assert torch.isfinite(model(ids)).all()


@pytest.mark.gpu
@pytest.mark.parametrize("case", [c for c in CASES if INFO[c]["method"] == "rtn"])
def test_save_is_byte_identical_to_reference(case: str, tmp_path: Any) -> None:
    wq = package()
    info = INFO[case]
    model = MODELS.make_model(info["seed"]).cuda()
    gs = info["group_size"]
    wq.quantize_model(model, wq.QuantConfig(bits=info["bits"], symmetric=info["symmetric"], group_size=gs))
    state = wq.compressed_state(model)
    ref = wq.read_compressed(_path(case))
    assert state["meta"] == ref["meta"]
    assert list(state["tensors"]) == list(ref["tensors"])
    for key, want in ref["tensors"].items():
        got = state["tensors"][key]
        assert got.dtype == want.dtype and torch.equal(got.view(torch.uint8), want.view(torch.uint8)), key
    path = tmp_path / f"compressed_{case}.pt"  # torch.save names the archive after the file
    assert wq.save_compressed(model, str(path)) == info["file_bytes"]
    with open(path, "rb") as a, open(_path(case), "rb") as b:
        assert a.read() == b.read()


@pytest.mark.gpu
@pytest.mark.parametrize("bits,group,bias", [(4, 128, True), (8, 64, False), (4, None, True)])
def test_round_trip_single_layer(bits: int, group: int | None, bias: bool, tmp_path: Any) -> None:
    """A model that is one Linear (root layer ""): quantize on the GPU, save,
    load; the loaded layer equals the quantized one with fp16-rounded scales,
    and its forward equals that layer's forward bit for bit."""
    wq = package()
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(bits * 1000 + (group or 0))
    lin = nn.Linear(1024, 768, bias=bias)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(768, 1024, generator=g) * 0.02)
        if bias:
            lin.bias.copy_(torch.randn(768, generator=g))
    layer = wq.quantize_model(lin.to(dev), wq.QuantConfig(bits=bits, symmetric=True, group_size=group), kernel=True)
    path = tmp_path / "layer.pt"
    wq.save_compressed(layer, str(path))
    loaded = wq.load_compressed(str(path), nn.Linear(1024, 768, bias=bias), device=dev)
    assert isinstance(loaded, wq.QuantizedLinear)
    assert torch.equal(loaded.codes, layer.codes)
    rounded = {p: getattr(layer, p).half().float() for p in ("scales", "zeros")}
    for p, want in rounded.items():
        assert torch.equal(getattr(loaded, p).view(torch.int32), want.view(torch.int32)), p
    qw = layer.quantized_weight()
    twin = wq.QuantizedLinear(
        wq.QuantizedWeight(codes=qw.codes, scales=rounded["scales"], zeros=rounded["zeros"], bits=qw.bits,
                           group_size=qw.group_size, in_features=qw.in_features, out_features=qw.out_features,
                           symmetric=qw.symmetric, packed=qw.packed, granularity=qw.granularity),
        layer.bias, impl="kernel")
    for batch in (1, 3, 64):
        x = torch.randn(batch, 1024, generator=g).to(dev)
        assert torch.equal(loaded(x), twin(x)), batch
