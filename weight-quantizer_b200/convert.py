"""``quantize_model`` on the GPU: replace every nn.Linear / GPT-2 Conv1D by a QuantizedLinear.

Same contract as ptqkit's ``quantize_model`` (src/ptqkit/convert.py:236-293):
RTN needs no data; AWQ and GPTQ calibrate on ``calibration_batches``, either
in one pass over the model (each target sees the float model's inputs) or
``sequential=True`` (targets in order, each calibrated with the earlier ones
already quantized); ``kernel=True`` makes the new layers run the sm_100a
dequant-GEMM; ``cache_weights`` keeps a dense W_hat on every layer; a model
that is itself the only target comes back as the replacement layer.

The calibration is built around the device: a ``_Recorder`` context installs
one forward pre-hook per target and folds every input batch, as it arrives,
into that target's statistics on the GPU (``_Stats``), keeping only what the
method needs:

* AWQ: the per-channel sum of |x| (fp64, this library's fixed-order kernel),
  the row count, and the first 2048 rows (the search sample, convert.py:26-63);
* GPTQ: the fp64 Gram matrix X^T X and the row count (Hessian X^T X / n);
* sequential mode: every input row of the one target being calibrated.

The method itself is one entry of ``_METHODS``: GPU RTN (bit-exact with
ptqkit's quantize_weight), the GPU AWQ search or the GPU GPTQ sweep.
Parameters must already live on a CUDA device (ptqkit requires the CPU,
convert.py:122-126).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from typing import Any

import torch
from torch import nn

from . import _kernels
from .awq import awq_quantize, channel_mean_abs
from .gptq import gptq_quantize
from .linear import QuantizedLinear
from .quant import Method, QuantConfig, QuantizedWeight, quantize_weight

Batch = torch.Tensor | dict[str, torch.Tensor]
_SAMPLE_ROWS = 2048   # AWQ search rows (convert.py:26)


# ---- targets -------------------------------------------------------------------


def _conv1d(module: nn.Module) -> bool:
    # GPT-2's Conv1D (transformers) stores its weight as [in, out]
    return type(module).__name__ == "Conv1D" and hasattr(module, "weight")


def iter_targets(model: nn.Module) -> list[tuple[str, nn.Module]]:
    """(name, module) of every nn.Linear / Conv1D with a 2-D weight, in
    named_modules order; layers that are already quantized are left out."""
    return [
        (name, m) for name, m in model.named_modules()
        if not isinstance(m, QuantizedLinear)
        and (isinstance(m, nn.Linear) or _conv1d(m))
        and isinstance(getattr(m, "weight", None), torch.Tensor) and m.weight.ndim == 2
    ]


def weight_out_in(module: nn.Module) -> torch.Tensor:
    """The module's weight as [out, in] (Conv1D's [in, out] transposed)."""
    w = getattr(module, "weight", None)
    if isinstance(w, torch.Tensor) and w.ndim == 2:
        if isinstance(module, nn.Linear):
            return w.detach()
        if _conv1d(module):
            return w.detach().t().contiguous()
    raise TypeError(f"unsupported module {type(module).__name__}")


def _set_module(root: nn.Module, name: str, new: nn.Module) -> None:
    parent_name, _, leaf = name.rpartition(".")
    setattr(root.get_submodule(parent_name) if parent_name else root, leaf, new)


# ---- calibration ----------------------------------------------------------------


class _Stats:
    """What one target's inputs contribute to its method, kept on the GPU."""

    def __init__(self, *, gram: bool, abs_sum: bool, sample: bool, all_rows: bool) -> None:
        self.want_gram, self.want_abs, self.want_sample, self.want_all = gram, abs_sum, sample, all_rows
        self.n = 0
        self.gram: torch.Tensor | None = None
        self.abs: torch.Tensor | None = None
        self.sample: list[torch.Tensor] = []
        self.n_sample = 0
        self.rows: list[torch.Tensor] = []

    def add(self, x: torch.Tensor) -> None:
        x = x.detach().reshape(-1, x.shape[-1]).to(dtype=torch.float32)
        self.n += int(x.shape[0])
        if self.want_gram:
            x64 = x.double()
            g = x64.t() @ x64
            self.gram = g if self.gram is None else self.gram + g
        if self.want_abs:
            self.abs = _kernels.channel_abs_sum(x, self.abs)
        if self.want_sample and self.n_sample < _SAMPLE_ROWS:
            take = x[: _SAMPLE_ROWS - self.n_sample].clone()
            self.sample.append(take)
            self.n_sample += int(take.shape[0])
        if self.want_all:
            self.rows.append(x.clone())

    def _need_rows(self) -> None:
        if self.n == 0:
            raise RuntimeError("no calibration rows")

    def hessian(self) -> torch.Tensor:
        self._need_rows()
        if self.want_all:
            r = torch.cat(self.rows).double()
            return r.t() @ r / float(r.shape[0])
        assert self.gram is not None
        return self.gram / self.n

    def awq_inputs(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(search rows, mean |x| per channel)."""
        self._need_rows()
        if self.want_all:
            r = torch.cat(self.rows)
            return r[:_SAMPLE_ROWS], channel_mean_abs(r)
        assert self.abs is not None
        return torch.cat(self.sample), (self.abs / self.n).to(dtype=torch.float32)


class _Recorder:
    """Context manager: forward pre-hooks feeding each target's ``_Stats``."""

    def __init__(self, targets: Sequence[tuple[str, nn.Module]], make: Callable[[], _Stats]) -> None:
        self.targets = list(targets)
        self.stats = {name: make() for name, _ in self.targets}
        self._handles: list[Any] = []

    def __enter__(self) -> _Recorder:
        for name, module in self.targets:
            def hook(_: nn.Module, args: tuple[Any, ...], *, name: str = name) -> None:
                if not args or not isinstance(args[0], torch.Tensor):
                    raise TypeError(f"{name} did not receive a tensor input")
                self.stats[name].add(args[0])
            self._handles.append(module.register_forward_pre_hook(hook))
        return self

    def __exit__(self, *exc: object) -> None:
        for h in self._handles:
            h.remove()
        self._handles.clear()


def _run(model: nn.Module, batches: Sequence[Batch]) -> None:
    for batch in batches:
        if isinstance(batch, dict):
            model(**batch)
        else:
            model(batch)


def _record(model: nn.Module, targets: Sequence[tuple[str, nn.Module]], batches: Sequence[Batch],
            method: Method, all_rows: bool) -> dict[str, _Stats]:
    def make() -> _Stats:
        if all_rows:
            return _Stats(gram=False, abs_sum=False, sample=False, all_rows=True)
        return _Stats(gram=method is Method.GPTQ, abs_sum=method is Method.AWQ, sample=method is Method.AWQ,
                      all_rows=False)

    with _Recorder(targets, make) as rec:
        _run(model, batches)
    return rec.stats


# ---- methods ----------------------------------------------------------------------


def _rtn(w: torch.Tensor, cfg: QuantConfig, st: _Stats | None) -> tuple[QuantizedWeight, float | None]:
    return quantize_weight(w, cfg), None


def _awq(w: torch.Tensor, cfg: QuantConfig, st: _Stats | None) -> tuple[QuantizedWeight, float | None]:
    if st is None:
        raise ValueError("AWQ requires calibration activations")
    rows, mean_abs = st.awq_inputs()
    return awq_quantize(w, rows, cfg, mean_abs=mean_abs)


def _gptq(w: torch.Tensor, cfg: QuantConfig, st: _Stats | None) -> tuple[QuantizedWeight, float | None]:
    if st is None:
        raise ValueError("GPTQ requires calibration activations")
    return gptq_quantize(w, st.hessian(), cfg), None


_METHODS: dict[Method, Callable[[torch.Tensor, QuantConfig, _Stats | None], tuple[QuantizedWeight, float | None]]] = {
    Method.RTN: _rtn, Method.AWQ: _awq, Method.GPTQ: _gptq,
}


def _layer(module: nn.Module, cfg: QuantConfig, st: _Stats | None, impl: str) -> QuantizedLinear:
    qw, alpha = _METHODS[cfg.method](weight_out_in(module), cfg, st)
    bias = getattr(module, "bias", None)
    layer = QuantizedLinear(qw, bias.detach() if isinstance(bias, torch.Tensor) else None, impl=impl)
    layer.awq_alpha = alpha
    return layer


# ---- the model pass -----------------------------------------------------------------


def quantize_model(
    model: nn.Module,
    config: QuantConfig,
    calibration_batches: Sequence[Batch] | None = None,
    *,
    sequential: bool = False,
    kernel: bool = False,
    cache_weights: bool = False,
) -> nn.Module:
    """Quantize every Linear and Conv1D of ``model`` in place on the GPU (see the module docstring)."""
    if any(p.device.type != "cuda" for p in model.parameters()):
        raise RuntimeError("quantize_model expects CUDA parameters")
    model.eval()
    hf_config = getattr(model, "config", None)
    if hf_config is not None and getattr(hf_config, "use_cache", None) is not None:
        hf_config.use_cache = False
    calibrated = config.method is not Method.RTN
    if calibrated and calibration_batches is None:
        raise ValueError(f"{config.method.value} requires calibration_batches")
    batches = [] if calibration_batches is None else list(calibration_batches)
    if calibration_batches is not None and not batches:
        raise ValueError("calibration_batches is empty")
    impl = "kernel" if kernel else "reference"
    targets = iter_targets(model)
    root_only = len(targets) == 1 and targets[0][0] == ""

    done: list[QuantizedLinear] = []
    with torch.inference_mode():
        if calibrated and sequential:
            # one target at a time; the quantized layers before it keep a dense
            # W_hat so that later passes run a plain GEMM through them
            for name, module in targets:
                st = _record(model, [(name, module)], batches, config.method, all_rows=True)[name]
                layer = _layer(module, config, st, impl)
                layer.materialize()
                done.append(layer)
                if not root_only:
                    _set_module(model, name, layer)
        else:
            stats = _record(model, targets, batches, config.method, all_rows=False) if calibrated else {}
            for name, module in targets:
                layer = _layer(module, config, stats.get(name), impl)
                done.append(layer)
                if not root_only:
                    _set_module(model, name, layer)
        for layer in (done if root_only else [m for m in model.modules() if isinstance(m, QuantizedLinear)]):
            if cache_weights:
                layer.materialize()
            else:
                layer.clear_cache()
    return done[0] if root_only else model
