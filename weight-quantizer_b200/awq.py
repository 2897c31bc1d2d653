"""Activation-aware weight scaling (AWQ) on the GPU, then RTN.

Mirror of ptqkit's ``awq`` module (src/ptqkit/awq.py:1-81): for calibration
activations X [n, K] and a weight W [out, K],

    m_k = mean_i |X_ik|                       (clamped to >= 1e-8)
    s(alpha)_k = m_k^alpha / mean(m^alpha)
    alpha* = argmin over config.awq_alphas of || X_s W^T - X_s W_hat(alpha)^T ||^2 / (n_s out)
    W_hat(alpha) = dequant(RTN(W diag(s(alpha)))) diag(s(alpha))^-1

on the deterministic stride subsample X_s of at most 2048 rows (awq.py:31-36);
the stored channel scale is 1/s. Every step runs on the device: the channel
means and the pre-scale in this library's reduction kernels, RTN in its
bit-exact quantizer, the score's X_s W_hat^T in its dequant-GEMM (straight
from the packed codes, so no dense W_hat is formed) and the squared error in a
deterministic fp64 reduction. The fp32 target X_s W^T is one plain GEMM
(cuBLAS through torch, with TF32 off).

ptqkit evaluates the score as ``search @ hat.T - target`` with a dense fp32
reconstruction on the CPU; the scores here agree with it to within the GEMM's
rounding (the tests check 1e-4 relative), so the same alpha wins unless two
candidates tie to that precision. Given the same pre-scale, the codes are
bit-exact with ptqkit's.
"""

from __future__ import annotations

from typing import Any

import torch

from . import _kernels
from .quant import QuantConfig, QuantizedWeight, quantize_weight

_SEARCH_ROWS = 2048


def _subsample(activations: torch.Tensor, limit: int) -> torch.Tensor:
    """The first ``limit`` rows of a stride-``max(n // limit, 1)`` view (awq.py:31-36)."""
    n = int(activations.shape[0])
    if n <= limit:
        return activations
    step = max(n // limit, 1)
    return activations[::step][:limit]


def _gemm_fp32(a: torch.Tensor, b_t: torch.Tensor) -> torch.Tensor:
    """a @ b_t.T in full fp32 (TF32 disabled for the call)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return a @ b_t.transpose(0, 1)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def channel_mean_abs(activations: torch.Tensor) -> torch.Tensor:
    """mean_i |X_ik| as fp32 [K] (awq.py:61), summed in fp64 on the device."""
    n = int(activations.shape[0])
    acc = _kernels.channel_abs_sum(activations)
    if n == 0:   # the mean of no rows, as torch gives it
        return torch.full_like(acc, float("nan"), dtype=torch.float32)
    return (acc / n).to(dtype=torch.float32)


def awq_search(
    weight: torch.Tensor,
    activations: torch.Tensor,
    config: QuantConfig,
    *,
    mean_abs: torch.Tensor | None = None,
) -> dict[str, Any]:
    """The alpha search of awq.py:39-81 with every candidate recorded.

    Returns ``{"weight": QuantizedWeight, "alpha": float, "alphas": [...],
    "mse": [...], "pre_scale": [...]}`` where the lists follow
    ``config.awq_alphas``.
    """
    if weight.ndim != 2:
        raise ValueError("weight must have shape [out, in]")
    if activations.ndim != 2 or int(activations.shape[1]) != int(weight.shape[1]):
        raise ValueError("activations must have shape [n, in]")
    dev = weight.device if weight.device.type == "cuda" else activations.device
    if dev.type != "cuda":
        if not torch.cuda.is_available():
            raise RuntimeError("wq_b200 runs on CUDA devices; no CUDA device is available")
        dev = torch.device("cuda", torch.cuda.current_device())
    w = weight.detach().to(device=dev, dtype=torch.float32).contiguous()
    x_all = activations.detach().to(device=dev, dtype=torch.float32)
    if mean_abs is None:
        mag = channel_mean_abs(x_all).clamp(min=1e-8)
    else:
        mag = mean_abs.detach().to(device=dev, dtype=torch.float32).reshape(-1).clamp(min=1e-8)
        if int(mag.numel()) != int(w.shape[1]):
            raise ValueError("mean_abs must have one entry per input channel")
    search = _subsample(x_all, _SEARCH_ROWS).contiguous()
    target = _gemm_fp32(search, w)
    denom = float(target.numel())
    best: QuantizedWeight | None = None
    best_alpha = float(config.awq_alphas[0])
    best_mse = float("inf")
    mses: list[float] = []
    pres: list[torch.Tensor] = []
    for alpha in config.awq_alphas:
        a = float(alpha)
        pre = _kernels.awq_pre_scale(mag, a)
        qw = quantize_weight(w, config, pre_scale=pre)
        y_hat = _kernels.dequant_gemm(
            search, qw.codes, qw.scales, qw.zeros, qw.channel_scale, qw.group_size, qw.bits, 0
        )
        mse = float(_kernels.sq_err_sum(y_hat, target).item()) / denom if denom > 0 else float("nan")
        mses.append(mse)
        pres.append(pre)
        if mse < best_mse:
            best_mse = mse
            best = qw
            best_alpha = a
    if best is None:
        raise RuntimeError("AWQ search produced no candidate")
    return {"weight": best, "alpha": best_alpha, "alphas": [float(a) for a in config.awq_alphas],
            "mse": mses, "pre_scale": pres}


def awq_quantize(
    weight: torch.Tensor,
    activations: torch.Tensor,
    config: QuantConfig,
    *,
    mean_abs: torch.Tensor | None = None,
) -> tuple[QuantizedWeight, float]:
    """Return the quantized weight and the alpha that won the search (awq.py:39-81)."""
    r = awq_search(weight, activations, config, mean_abs=mean_abs)
    return r["weight"], r["alpha"]
