"""Replace nn.Linear and GPT-2 Conv1D modules with QuantizedLinear on the GPU.

Mirror of ptqkit's ``quantize_model`` (src/ptqkit/convert.py:236-293) for the
RTN method, with the model's parameters on a CUDA device instead of the CPU
(ptqkit's ``_check_cpu``, convert.py:122-126, becomes a CUDA check): every
target weight is quantized by the GPU RTN kernel (bit-exact with ptqkit's
quantize_weight) and the module is replaced by a QuantizedLinear whose
``impl="kernel"`` forward runs the dequant-GEMM with the bias added in the
kernel's epilogue.

Conv1D stores its weight as [in, out] and computes x @ W; the quantizer stores
[out, in] for both layouts, so the forward is always x @ W_hat^T + bias
(convert.py:1-4). AWQ and GPTQ need calibration passes that are not part of
this hot path and raise NotImplementedError.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import nn

from .linear import QuantizedLinear
from .quant import Method, QuantConfig, quantize_weight

Batch = torch.Tensor | dict[str, torch.Tensor]


def _is_conv1d(module: nn.Module) -> bool:
    return module.__class__.__name__ == "Conv1D" and hasattr(module, "weight")


def iter_targets(model: nn.Module) -> list[tuple[str, nn.Module]]:
    """Every nn.Linear / Conv1D with a 2-D weight, in named_modules order
    (convert.py:73-82); modules that are already QuantizedLinear are skipped."""
    found: list[tuple[str, nn.Module]] = []
    for name, module in model.named_modules():
        if isinstance(module, QuantizedLinear):
            continue
        if isinstance(module, nn.Linear) or _is_conv1d(module):
            weight = getattr(module, "weight", None)
            if isinstance(weight, torch.Tensor) and weight.ndim == 2:
                found.append((name, module))
    return found


def weight_out_in(module: nn.Module) -> torch.Tensor:
    """The module's weight as [out, in] (convert.py:85-93)."""
    weight = getattr(module, "weight", None)
    if not isinstance(weight, torch.Tensor) or weight.ndim != 2:
        raise TypeError(f"unsupported module {module.__class__.__name__}")
    if isinstance(module, nn.Linear):
        return weight.detach()
    if _is_conv1d(module):
        return weight.detach().transpose(0, 1).contiguous()
    raise TypeError(f"unsupported module {module.__class__.__name__}")


def _bias_of(module: nn.Module) -> torch.Tensor | None:
    bias = getattr(module, "bias", None)
    if not isinstance(bias, torch.Tensor):
        return None
    return bias.detach()


def _replace(root: nn.Module, name: str, new: nn.Module) -> None:
    parent: nn.Module = root
    parts = name.split(".")
    for part in parts[:-1]:
        child = getattr(parent, part)
        if not isinstance(child, nn.Module):
            raise TypeError(f"{part} is not a module")
        parent = child
    setattr(parent, parts[-1], new)


def _check_cuda(model: nn.Module) -> None:
    for param in model.parameters():
        if param.device.type != "cuda":
            raise RuntimeError("quantize_model expects CUDA parameters")


def _prepare(model: nn.Module) -> None:
    model.eval()
    config = getattr(model, "config", None)
    if config is not None and getattr(config, "use_cache", None) is not None:
        config.use_cache = False


def quantize_model(
    model: nn.Module,
    config: QuantConfig,
    calibration_batches: Sequence[Batch] | None = None,
    *,
    sequential: bool = False,
    kernel: bool = False,
    cache_weights: bool = False,
) -> nn.Module:
    """Quantize every Linear and Conv1D in ``model`` in place (convert.py:236-293).

    ``kernel=True`` makes the layers run the sm_100a dequant-GEMM; otherwise
    they use ptqkit's reference dense reconstruction. ``cache_weights`` keeps a
    dense W_hat on every layer (a plain fp32 GEMM forward). Returns the model,
    or the replacement layer when the model itself is the only target.
    """
    del sequential  # only meaningful for the calibration methods
    _check_cuda(model)
    _prepare(model)
    targets = iter_targets(model)
    if config.method is not Method.RTN:
        if calibration_batches is None:
            raise ValueError(f"{config.method.value} requires calibration_batches")
        raise NotImplementedError(f"{config.method.value} calibration is not part of this build; use RTN")
    impl = "kernel" if kernel else "reference"

    with torch.inference_mode():
        if len(targets) == 1 and targets[0][0] == "":
            module = targets[0][1]
            layer = QuantizedLinear(quantize_weight(weight_out_in(module), config), _bias_of(module), impl=impl)
            if cache_weights:
                layer.materialize()
            return layer
        for name, module in targets:
            qw = quantize_weight(weight_out_in(module), config)
            _replace(model, name, QuantizedLinear(qw, _bias_of(module), impl=impl))
        for module in model.modules():
            if isinstance(module, QuantizedLinear):
                if cache_weights:
                    module.materialize()
                else:
                    module.clear_cache()
    return model
