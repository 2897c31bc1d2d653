"""Replace nn.Linear and GPT-2 Conv1D modules with QuantizedLinear on the GPU.

Mirror of ptqkit's ``quantize_model`` (src/ptqkit/convert.py:236-293) for the
RTN, AWQ and GPTQ methods, with the model's parameters on a CUDA device instead of
the CPU (ptqkit's ``_check_cpu``, convert.py:122-126, becomes a CUDA check):
every target weight is quantized by the GPU RTN kernel (bit-exact with
ptqkit's quantize_weight), the GPU AWQ search (``awq.awq_quantize``) or the
GPU GPTQ sweep (``gptq.gptq_quantize``), and
the module is replaced by a QuantizedLinear whose ``impl="kernel"`` forward
runs the dequant-GEMM with the bias added in the kernel's epilogue.

AWQ calibration follows convert.py:26-254: forward pre-hooks collect each
target's inputs, either as running statistics over one pass of the
calibration set (channel |x| sums in fp64 and the first 2048 rows,
ActivationStats) or, with ``sequential=True``, as every input row of one
target at a time with the earlier targets already replaced. GPTQ takes its
Hessian X^T X / n from the same capture (an fp64 Gram matrix on the device)
and runs ``gptq.gptq_quantize``.

Conv1D stores its weight as [in, out] and computes x @ W; the quantizer stores
[out, in] for both layouts, so the forward is always x @ W_hat^T + bias
(convert.py:1-4).
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch
from torch import nn

from . import _kernels
from .awq import awq_quantize, channel_mean_abs
from .gptq import gptq_quantize
from .linear import QuantizedLinear
from .quant import Method, QuantConfig, QuantizedWeight, quantize_weight

Batch = torch.Tensor | dict[str, torch.Tensor]
_SAMPLE_ROWS = 2048


class ActivationStats:
    """Running statistics of one target's inputs (convert.py:35-70), on the device:
    the fp64 Gram matrix X^T X (for GPTQ's Hessian; kept only when asked for),
    the fp64 sum of |x| per input channel, the row count and the first 2048 rows."""

    def __init__(self, gram: bool = True) -> None:
        self.keep_gram = gram
        self.xtx: torch.Tensor | None = None
        self.abs_sum: torch.Tensor | None = None
        self.count: int = 0
        self.sample: torch.Tensor | None = None

    def update(self, hidden: torch.Tensor) -> None:
        x = hidden.detach().reshape(-1, hidden.shape[-1]).to(dtype=torch.float32)
        if self.keep_gram:
            x64 = x.double()
            gram = x64.transpose(0, 1) @ x64
            self.xtx = gram if self.xtx is None else self.xtx + gram
        self.abs_sum = _kernels.channel_abs_sum(x, self.abs_sum)
        self.count += int(x.shape[0])
        if self.sample is None:
            self.sample = x[:_SAMPLE_ROWS].clone()
        elif int(self.sample.shape[0]) < _SAMPLE_ROWS:
            need = _SAMPLE_ROWS - int(self.sample.shape[0])
            self.sample = torch.cat((self.sample, x[:need].clone()), dim=0)

    def hessian(self) -> torch.Tensor:
        if self.xtx is None or self.count == 0:
            raise RuntimeError("no calibration rows")
        return self.xtx / self.count

    def mean_abs(self) -> torch.Tensor:
        if self.abs_sum is None or self.count == 0:
            raise RuntimeError("no calibration rows")
        return (self.abs_sum / self.count).to(dtype=torch.float32)

    def rows(self) -> torch.Tensor:
        if self.sample is None:
            raise RuntimeError("no calibration rows")
        return self.sample


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


def _forward(model: nn.Module, batch: Batch) -> None:
    if isinstance(batch, dict):
        model(**batch)
    else:
        model(batch)


def _as_batches(batches: Sequence[Batch]) -> list[Batch]:
    if len(batches) == 0:
        raise ValueError("calibration_batches is empty")
    return list(batches)


def _capture_all(model: nn.Module, names: list[tuple[str, nn.Module]],
                 batches: Sequence[Batch], gram: bool = True) -> dict[str, ActivationStats]:
    """One pass of the calibration set with a statistics hook on every target (convert.py:140-162)."""
    stats = {name: ActivationStats(gram) for name, _ in names}
    handles = []
    for name, module in names:

        def hook(mod: nn.Module, args: tuple[Any, ...], *, name: str = name) -> None:
            del mod
            if not args or not isinstance(args[0], torch.Tensor):
                raise TypeError(f"{name} did not receive a tensor input")
            stats[name].update(args[0])

        handles.append(module.register_forward_pre_hook(hook))
    try:
        for batch in batches:
            _forward(model, batch)
    finally:
        for handle in handles:
            handle.remove()
    return stats


def _capture_one(model: nn.Module, name: str, module: nn.Module, batches: Sequence[Batch]) -> torch.Tensor:
    """Every input row of one target over the calibration set (convert.py:165-189)."""
    chunks: list[torch.Tensor] = []

    def hook(mod: nn.Module, args: tuple[Any, ...]) -> None:
        del mod
        if not args or not isinstance(args[0], torch.Tensor):
            raise TypeError(f"{name} did not receive a tensor input")
        chunks.append(args[0].detach().reshape(-1, args[0].shape[-1]).to(dtype=torch.float32))

    handle = module.register_forward_pre_hook(hook)
    try:
        for batch in batches:
            _forward(model, batch)
    finally:
        handle.remove()
    if not chunks:
        raise RuntimeError(f"no activations captured for {name}")
    return torch.cat(chunks, dim=0)


def _module_from(qw: QuantizedWeight, source: nn.Module, *, kernel: bool, alpha: float | None) -> QuantizedLinear:
    layer = QuantizedLinear(qw, _bias_of(source), impl="kernel" if kernel else "reference")
    layer.awq_alpha = alpha
    return layer


def _quantize_one(weight: torch.Tensor, config: QuantConfig, stats: ActivationStats | None,
                  rows: torch.Tensor | None) -> tuple[QuantizedWeight, float | None]:
    """RTN, or AWQ from captured statistics or rows (convert.py:206-233)."""
    if config.method is Method.RTN:
        return quantize_weight(weight, config), None
    if config.method is Method.GPTQ:
        if stats is None and rows is None:
            raise ValueError("GPTQ requires calibration activations")
        if rows is not None and stats is None:
            r64 = rows.double()
            hessian = r64.transpose(0, 1) @ r64 / float(rows.shape[0])
        else:
            assert stats is not None
            hessian = stats.hessian()
        return gptq_quantize(weight, hessian, config), None
    if config.method is Method.AWQ:
        if rows is None and stats is None:
            raise ValueError("AWQ requires calibration activations")
        if stats is not None and rows is None:
            sample = stats.rows()
            mean_abs = stats.mean_abs()
        else:
            assert rows is not None
            sample = rows[:_SAMPLE_ROWS]
            mean_abs = channel_mean_abs(rows)
        return awq_quantize(weight, sample, config, mean_abs=mean_abs)
    raise ValueError(f"unknown method {config.method}")


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
    _check_cuda(model)
    _prepare(model)
    targets = iter_targets(model)
    if config.method is not Method.RTN and calibration_batches is None:
        raise ValueError(f"{config.method.value} requires calibration_batches")
    batches = [] if calibration_batches is None else _as_batches(calibration_batches)

    with torch.inference_mode():
        if len(targets) == 1 and targets[0][0] == "":
            module = targets[0][1]
            stats = None
            rows = None
            if config.method is not Method.RTN:
                if sequential:
                    rows = _capture_one(model, "root", module, batches)
                else:
                    stats = _capture_all(model, [("root", module)], batches, config.method is Method.GPTQ)["root"]
            qw, alpha = _quantize_one(weight_out_in(module), config, stats, rows)
            layer = _module_from(qw, module, kernel=kernel, alpha=alpha)
            if cache_weights:
                layer.materialize()
            return layer
        if config.method is Method.RTN or not sequential:
            stats_map: dict[str, ActivationStats] | None = None
            if config.method is not Method.RTN:
                stats_map = _capture_all(model, targets, batches, config.method is Method.GPTQ)
            for name, module in targets:
                stats = None if stats_map is None else stats_map[name]
                qw, alpha = _quantize_one(weight_out_in(module), config, stats, None)
                _replace(model, name, _module_from(qw, module, kernel=kernel, alpha=alpha))
        else:
            for name, module in targets:
                rows = _capture_one(model, name, module, batches)
                qw, alpha = _quantize_one(weight_out_in(module), config, None, rows)
                layer = _module_from(qw, module, kernel=kernel, alpha=alpha)
                # a cached reconstruction keeps later calibration passes on the fp32 GEMM
                layer.materialize()
                _replace(model, name, layer)
        for module in model.modules():
            if isinstance(module, QuantizedLinear):
                if cache_weights:
                    module.materialize()
                else:
                    module.clear_cache()
    return model
