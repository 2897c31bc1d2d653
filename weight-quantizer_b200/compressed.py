"""ptqkit's compressed on-disk format (version 1) and a GPU loader for it.

Format (src/ptqkit/convert.py:296-336), kept identical so that files move
both ways between ptqkit and this package: ``torch.save`` of

    {"version": 1,
     "meta": {layer: {bits, group_size, in_features, out_features, symmetric,
                      packed, granularity, awq_alpha}},
     "tensors": {"<layer>.codes": uint8, "<layer>.scales"/".zeros"/".channel_scale": fp16,
                 "<layer>.bias": fp32, "param.<name>": ..., "buffer.<name>": ...}}

with one entry per QuantizedLinear (layer "" when the model itself is one) and
every other parameter and buffer of the model as it is. fp16 holds every
integer zero point in [0, 255] exactly; scales and channel scales are rounded
to fp16 by the format (convert.py:297-301), so a loaded layer computes with
those rounded values.

ptqkit writes the format and has no loader. ``load_compressed`` here uploads a
file straight into the layout the dequant-GEMM reads: the codes and fp32 biases
of all layers go to the GPU as one block of device memory, the fp16 scales,
zeros and channel scales of all layers as a second block that one kernel
launch widens into a single fp32 block; each layer's buffers are views of
those blocks. Writing (``compressed_state``) narrows each fp32 array to fp16
on the device before it is copied to the host.
"""

from __future__ import annotations

import os
from collections.abc import Iterator
from typing import Any

import torch
from torch import nn

from . import _kernels
from .convert import _set_module, weight_out_in
from .linear import QuantizedLinear
from .quant import QuantizedWeight

FORMAT_VERSION = 1

_ALIGN = 256  # byte alignment of every tensor inside the uploaded blocks
_HALF_ALIGN = _ALIGN // 2  # the same, in fp16 elements (fp32 views land on 512 B)


def _quantized_layers(model: nn.Module) -> Iterator[tuple[str, QuantizedLinear]]:
    for name, module in model.named_modules():
        if isinstance(module, QuantizedLinear):
            yield name, module


def _to_half(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cuda":
        raise RuntimeError("compressed_state expects QuantizedLinear buffers on a CUDA device")
    return _kernels.narrow_f32_f16(t.detach().to(dtype=torch.float32)).cpu()


def compressed_state(model: nn.Module) -> dict[str, Any]:
    """Integer codes, fp16 scales/zeros, fp32 biases, and untouched parameters
    (convert.py:296-336): the same keys, dtypes and values as ptqkit's, with
    the fp16 rounding done on the GPU."""
    tensors: dict[str, torch.Tensor] = {}
    meta: dict[str, dict[str, Any]] = {}
    quantized_buffers: set[str] = set()
    for name, module in _quantized_layers(model):
        meta[name] = {
            "bits": module.bits,
            "group_size": module.group_size,
            "in_features": module.in_features,
            "out_features": module.out_features,
            "symmetric": module.symmetric,
            "packed": module.packed,
            "granularity": module.granularity,
            "awq_alpha": module.awq_alpha,
        }
        prefix = f"{name}." if name else ""
        tensors[prefix + "codes"] = module.codes.detach().cpu()
        tensors[prefix + "scales"] = _to_half(module.scales)
        tensors[prefix + "zeros"] = _to_half(module.zeros)
        if module.channel_scale is not None:
            tensors[prefix + "channel_scale"] = _to_half(module.channel_scale)
        if module.bias is not None:
            tensors[prefix + "bias"] = module.bias.detach().to(dtype=torch.float32).cpu()
        for buffer_name, _buffer in module.named_buffers(recurse=False):
            quantized_buffers.add(f"{name}.{buffer_name}" if name else buffer_name)
    for param_name, param in model.named_parameters():
        tensors["param." + param_name] = param.detach().cpu()
    for buffer_name, buffer in model.named_buffers():
        if buffer_name in quantized_buffers:
            continue
        tensors["buffer." + buffer_name] = buffer.detach().cpu()
    return {"version": FORMAT_VERSION, "meta": meta, "tensors": tensors}


def payload_nbytes(state: dict[str, Any]) -> int:
    """Bytes of every tensor in a compressed state (convert.py:339-344)."""
    return sum(int(t.nbytes) for t in state["tensors"].values())


def matrix_nbytes(model: nn.Module) -> int:
    """Packed codes plus fp16 scales, zeros, and channel scales; no biases
    (convert.py:347-358)."""
    total = 0
    for _, module in _quantized_layers(model):
        total += int(module.codes.nbytes)
        total += int(module.scales.numel()) * 2
        total += int(module.zeros.numel()) * 2
        if module.channel_scale is not None:
            total += int(module.channel_scale.numel()) * 2
    return total


def save_compressed(model: nn.Module, path: str) -> int:
    """Write ``compressed_state(model)`` with torch.save; returns the file size
    (convert.py:361-367)."""
    state = compressed_state(model)
    parent = os.path.dirname(path)
    if parent:
        os.makedirs(parent, exist_ok=True)
    torch.save(state, path)
    return os.path.getsize(path)


def state_dict_nbytes(model: nn.Module) -> int:
    """Bytes of ``model.state_dict()`` (convert.py:370-374)."""
    return sum(int(t.nbytes) for t in model.state_dict().values())


def _check_state(state: Any) -> dict[str, Any]:
    if not isinstance(state, dict) or "tensors" not in state or "meta" not in state:
        raise ValueError("not a compressed state: expected a dict with 'version', 'meta' and 'tensors'")
    version = state.get("version")
    if version != FORMAT_VERSION:
        raise ValueError(f"unsupported compressed format version {version!r} (expected {FORMAT_VERSION})")
    if not isinstance(state["meta"], dict) or not isinstance(state["tensors"], dict):
        raise ValueError("not a compressed state: 'meta' and 'tensors' must be dicts")
    return state


def read_compressed(path: str | os.PathLike[str]) -> dict[str, Any]:
    """Open a compressed file on the host without executing code from it
    (``weights_only``); tensors are memory-mapped from the file."""
    state = torch.load(os.fspath(path), map_location="cpu", weights_only=True, mmap=True)
    return _check_state(state)


def _tensor(tensors: dict[str, torch.Tensor], key: str, dtype: torch.dtype, ndim: int | None) -> torch.Tensor:
    if key not in tensors:
        raise ValueError(f"compressed state has no tensor {key!r}")
    t = tensors[key]
    if not isinstance(t, torch.Tensor) or t.dtype != dtype:
        raise ValueError(f"compressed tensor {key!r} must be {dtype}")
    if ndim is not None and t.ndim != ndim:
        raise ValueError(f"compressed tensor {key!r} must have {ndim} dimensions")
    return t


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def _device(device: torch.device | str | int | None) -> torch.device:
    dev = torch.device("cuda") if device is None else torch.device(device)
    if dev.type != "cuda":
        raise ValueError("load_compressed uploads to a CUDA device")
    return dev


def _indexed(dev: torch.device) -> torch.device:
    return dev if dev.index is not None else torch.device("cuda", torch.cuda.current_device())


def load_compressed_layers(
    source: str | os.PathLike[str] | dict[str, Any],
    *,
    device: torch.device | str | int | None = None,
    impl: str = "kernel",
) -> dict[str, QuantizedLinear]:
    """Every quantized layer of a compressed file (or state dict) as a
    QuantizedLinear on ``device``, keyed by module name.

    Two host-to-device copies from one pinned staging buffer move the whole
    payload: block A holds the uint8 codes and fp32 biases, block B the fp16
    scales, zeros and channel scales, each tensor at a 256-byte boundary. One
    widening launch turns block B into the fp32 block the layers' scales,
    zeros and channel scales are views of (exact: fp16 -> fp32 loses nothing).
    """
    dev = _device(device)
    state = _check_state(source) if isinstance(source, dict) else read_compressed(source)
    tensors: dict[str, torch.Tensor] = state["tensors"]
    meta: dict[str, dict[str, Any]] = state["meta"]

    # plan: (layer, name, tensor, block, offset); offsets in bytes (A) or fp16 elements (B)
    plan: list[tuple[str, str, torch.Tensor, str, int]] = []
    a_bytes = 0
    b_elems = 0
    for layer, m in meta.items():
        prefix = f"{layer}." if layer else ""
        parts: list[tuple[str, torch.Tensor, str]] = [
            ("codes", _tensor(tensors, prefix + "codes", torch.uint8, 2), "A"),
            ("scales", _tensor(tensors, prefix + "scales", torch.float16, 2), "B"),
            ("zeros", _tensor(tensors, prefix + "zeros", torch.float16, 2), "B"),
        ]
        if prefix + "channel_scale" in tensors:
            parts.append(("channel_scale", _tensor(tensors, prefix + "channel_scale", torch.float16, 1), "B"))
        if prefix + "bias" in tensors:
            parts.append(("bias", _tensor(tensors, prefix + "bias", torch.float32, 1), "A"))
        for key in ("bits", "group_size", "in_features", "out_features", "symmetric", "packed", "granularity"):
            if key not in m:
                raise ValueError(f"compressed layer {layer!r} has no {key!r} entry")
        for part, t, block in parts:
            if block == "A":
                a_bytes = _round_up(a_bytes, _ALIGN)
                plan.append((layer, part, t, "A", a_bytes))
                a_bytes += int(t.nbytes)
            else:
                b_elems = _round_up(b_elems, _HALF_ALIGN)
                plan.append((layer, part, t, "B", b_elems))
                b_elems += int(t.numel())
    a_bytes = _round_up(a_bytes, _ALIGN)
    b_elems = _round_up(b_elems, _HALF_ALIGN)

    dev = _indexed(dev)
    staging = torch.empty(a_bytes + 2 * b_elems, dtype=torch.uint8, pin_memory=True)
    for _, _, t, block, off in plan:
        start = off if block == "A" else a_bytes + 2 * off
        src = t.contiguous().reshape(-1).view(torch.uint8)
        staging[start : start + src.numel()].copy_(src)

    with torch.cuda.device(dev):
        block_a = torch.empty(a_bytes, dtype=torch.uint8, device=dev)
        block_a.copy_(staging[:a_bytes], non_blocking=True)
        wide = torch.empty(b_elems, dtype=torch.float32, device=dev)
        if b_elems:
            block_b = torch.empty(b_elems, dtype=torch.float16, device=dev)
            block_b.view(torch.uint8).copy_(staging[a_bytes:], non_blocking=True)
            _kernels.widen_f16_f32(block_b, wide)
            del block_b  # the caching allocator reuses it only after the widening, in stream order

    views: dict[str, dict[str, torch.Tensor]] = {layer: {} for layer in meta}
    for layer, part, t, block, off in plan:
        if block == "A":
            v = block_a[off : off + int(t.nbytes)].view(t.dtype).view(t.shape)
        else:
            v = wide[off : off + int(t.numel())].view(t.shape)
        views[layer][part] = v

    layers: dict[str, QuantizedLinear] = {}
    for layer, m in meta.items():
        v = views[layer]
        qw = QuantizedWeight(
            codes=v["codes"],
            scales=v["scales"],
            zeros=v["zeros"],
            bits=int(m["bits"]),
            group_size=int(m["group_size"]),
            in_features=int(m["in_features"]),
            out_features=int(m["out_features"]),
            symmetric=bool(m["symmetric"]),
            packed=bool(m["packed"]),
            granularity=m["granularity"],
            channel_scale=v.get("channel_scale"),
        )
        module = QuantizedLinear(qw, v.get("bias"), impl=impl)
        module.awq_alpha = m.get("awq_alpha")
        layers[layer] = module
    return layers


def _matches(module: nn.Module, layer: QuantizedLinear) -> bool:
    if isinstance(module, QuantizedLinear):
        return (module.out_features, module.in_features) == (layer.out_features, layer.in_features)
    try:
        shape = tuple(weight_out_in(module).shape)
    except TypeError:
        return False
    return shape == (layer.out_features, layer.in_features)


def _slots(model: nn.Module, kind: str) -> list[tuple[str, list[tuple[nn.Module, str]], torch.Tensor]]:
    """(file key, owning (module, attribute) pairs, current tensor) for every
    distinct parameter or buffer outside the QuantizedLinear layers. A tensor
    registered under several names is one slot, keyed by its first name, the
    name ``named_parameters()`` / ``named_buffers()`` report for it."""
    table: dict[int, tuple[str, list[tuple[nn.Module, str]], torch.Tensor]] = {}
    for module_name, module in model.named_modules(remove_duplicate=False):
        if isinstance(module, QuantizedLinear):
            continue
        store = module._parameters if kind == "param" else module._buffers
        for leaf, t in store.items():
            if t is None:
                continue
            full = f"{module_name}.{leaf}" if module_name else leaf
            entry = table.setdefault(id(t), (f"{kind}.{full}", [], t))
            entry[1].append((module, leaf))
    return list(table.values())


def load_compressed(
    source: str | os.PathLike[str] | dict[str, Any],
    model: nn.Module,
    *,
    device: torch.device | str | int | None = None,
    impl: str = "kernel",
) -> nn.Module:
    """Rebuild a quantized model from a compressed file on ``device``.

    ``model`` has the architecture the file was written from, before
    quantization (its values are overwritten; it may live on any device). Every
    layer named in the file replaces the nn.Linear / Conv1D of that name
    (``load_compressed_layers``); every other parameter and buffer is set from
    the file's ``param.*`` / ``buffer.*`` tensors, parameters shared between
    modules staying shared. Returns the model, or the layer itself when the
    file holds a single layer that was the whole model (convert.py:253-263).
    """
    dev = _device(device)
    state = _check_state(source) if isinstance(source, dict) else read_compressed(source)
    tensors: dict[str, torch.Tensor] = state["tensors"]
    layers = load_compressed_layers(state, device=dev, impl=impl)
    dev = _indexed(dev)
    if "" in layers:
        if len(layers) != 1:
            raise ValueError("a compressed state with a root layer holds no other layer")
        if not _matches(model, layers[""]):
            raise ValueError("model does not match the compressed layer's shape")
        return layers[""]

    for name, layer in layers.items():
        try:
            target = model.get_submodule(name)
        except AttributeError as err:
            raise ValueError(f"model has no module {name!r}") from err
        if not _matches(target, layer):
            raise ValueError(f"module {name!r} does not match the compressed layer's shape")
        _set_module(model, name, layer)

    used: set[str] = set()
    for kind in ("param", "buffer"):
        for key, owners, old in _slots(model, kind):
            if key not in tensors:
                raise ValueError(f"compressed state has no tensor {key!r}")
            t = tensors[key]
            if tuple(t.shape) != tuple(old.shape):
                raise ValueError(f"compressed tensor {key!r} has shape {tuple(t.shape)}, the model {tuple(old.shape)}")
            new = t.to(device=dev)
            if kind == "param":
                new = nn.Parameter(new, requires_grad=old.requires_grad)
            for owner, leaf in owners:
                getattr(owner, "_parameters" if kind == "param" else "_buffers")[leaf] = new
            used.add(key)

    extra = sorted(k for k in tensors if k.startswith(("param.", "buffer.")) and k not in used)
    if extra:
        raise ValueError(f"compressed state has tensors the model does not: {extra[:4]}")
    return model
