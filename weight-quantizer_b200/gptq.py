"""GPTQ column quantization on the GPU (fp64).

Mirror of ptqkit's ``gptq`` module (src/ptqkit/gptq.py:1-191). For one linear
map with Hessian H = X^T X / n it quantizes the columns of W left to right
onto the RTN grid and corrects the remaining columns with the OBS step

    err = (w_i - w_hat_i) / U_ii,     W[:, i:] -= err * U[i, i:],

U the upper Cholesky factor of the damped inverse Hessian (gptq.py:44-71:
symmetrize, isolate channels whose diagonal is exactly zero, add
percdamp * mean(diag) to the diagonal, retry with a larger bump if the
factorization fails). Group scales come from the updated weights at the start
of each group, per-channel and per-tensor scales once before the sweep.

Device split: everything runs in this library's kernels. The factor U
(``wq_chol_inverse_upper_f64``) is computed as J M^-1 J with M M^T = J H J
(J reverses rows and columns), one blocked factorization and one blocked
triangular inverse, where the reference factors H, inverts it and factors the
inverse (the same matrix, rounded differently); a pivot that is not positive
retries with more damping as the reference does. The sweep:
``wq_gptq_qparams_f64`` (the grid of quant.py:146-172 in fp64),
``wq_gptq_block_f64`` (one block's column sweep, one warp per weight row,
bit-exact with ptqkit's _obs_block given the same inputs) and
``wq_gptq_tail_f64`` (each block's update of the later columns, the
O(K^2 M) part, an fp64 tile kernel summing in column order). Groups wider
than 128 columns are swept in 128-column blocks whose later columns are
corrected by that update, the same updates as the reference's per-column
ones in a different summation order.

Because the factorization and the tail update round differently from the CPU
LAPACK/BLAS the reference runs on, codes agree with ptqkit's except where a
weight lands within rounding of a grid edge; the tests bound that fraction
and the output error.
"""

from __future__ import annotations

import torch

from . import _kernels
from .quant import Method, QuantConfig, QuantizedWeight, assemble_quantized, granularity_of

_BLOCK = 128   # columns one sweep kernel launch holds


def _factor_inverse(hessian: torch.Tensor, percdamp: float) -> torch.Tensor:
    """The upper Cholesky factor of the damped inverse (gptq.py:44-71)."""
    h = 0.5 * (hessian + hessian.transpose(0, 1))
    diag = torch.diag(h)
    dead = diag == 0
    if bool(torch.any(dead).item()):
        h = h.clone()
        h[dead, :] = 0
        h[:, dead] = 0
        idx = torch.arange(h.shape[0], device=h.device)[dead]
        h[idx, idx] = 1
    damp = percdamp * torch.mean(torch.diag(h))
    if not bool(torch.isfinite(damp).item()) or float(damp.item()) < 0:
        damp = torch.zeros((), dtype=h.dtype, device=h.device)
    eye = torch.arange(h.shape[0], device=h.device)
    h = h.clone()
    h[eye, eye] = h[eye, eye] + damp
    for _ in range(6):
        factor, info = _kernels.chol_inverse_upper(h)
        if int(info.item()) == 0:
            return factor
        bump = torch.mean(torch.diag(h)) * 0.1 + 1e-6
        h[eye, eye] = h[eye, eye] + bump
    raise RuntimeError("damped Hessian Cholesky failed")


_NO_BAD_COLUMN = 2**31 - 1


def _sweep(work: torch.Tensor, hinv: torch.Tensor, codes: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor,
           qp_stride: int, bits: int, start: int, end: int) -> None:
    """Quantize columns [start, end) of ``work`` and correct the later columns
    (gptq.py:86-125), in sweeps of at most 128 columns.

    A column whose OBS error is not finite in some row gets a zero error in
    every row, as _obs_block does (gptq.py:114-115): the sweep kernel reports
    the first such column and the block is swept again with it masked (the
    sweep reads ``work`` without writing it, so a repeat starts clean)."""
    inn = int(work.shape[1])
    rows = int(work.shape[0])
    bad = torch.empty(1, dtype=torch.int32, device=work.device)
    for s0 in range(start, end, _BLOCK):
        s1 = min(s0 + _BLOCK, end)
        err = torch.empty((rows, s1 - s0), dtype=torch.float64, device=work.device)
        mask: torch.Tensor | None = None
        for _ in range(s1 - s0 + 1):
            bad.fill_(_NO_BAD_COLUMN)
            _kernels.gptq_block(work, hinv, s0, s1 - s0, scale, zero, qp_stride, bits, codes, err, mask, bad)
            col = int(bad.item())
            if col == _NO_BAD_COLUMN:
                break
            if mask is None:
                mask = torch.zeros(s1 - s0, dtype=torch.uint8, device=work.device)
            mask[col] = 1
        if s1 < inn:
            _kernels.gptq_tail(work, s1, err, hinv, s0)


def gptq_quantize(weight: torch.Tensor, hessian: torch.Tensor, config: QuantConfig) -> QuantizedWeight:
    """Quantize ``weight`` [out, in] with Hessian ``hessian`` [in, in] (gptq.py:128-191)."""
    if config.method not in (Method.GPTQ, Method.RTN):
        raise ValueError("gptq_quantize expects a GPTQ or RTN grid config")
    if weight.ndim != 2:
        raise ValueError("weight must have shape [out, in]")
    out, inn = int(weight.shape[0]), int(weight.shape[1])
    if hessian.shape != (inn, inn):
        raise ValueError("hessian must have shape [in, in]")
    dev = weight.device if weight.device.type == "cuda" else hessian.device
    if dev.type != "cuda":
        if not torch.cuda.is_available():
            raise RuntimeError("wq_b200 runs on CUDA devices; no CUDA device is available")
        dev = torch.device("cuda", torch.cuda.current_device())
    work = weight.detach().to(device=dev, dtype=torch.float64).clone().contiguous()
    if not bool(torch.isfinite(work).all().item()):
        raise ValueError("weight must be finite")
    h = hessian.detach().to(device=dev, dtype=torch.float64)
    dead = torch.diag(h) == 0
    if bool(torch.any(dead).item()):
        work[:, dead] = 0
    hinv = _factor_inverse(h, config.percdamp).contiguous()
    bits = int(config.bits)
    codes = torch.zeros(out, inn, dtype=torch.int32, device=dev)
    granularity = granularity_of(config)
    if granularity == "group":
        assert config.group_size is not None
        gs = int(config.group_size)
        groups = (inn + gs - 1) // gs
        scales = torch.empty((out, groups), dtype=torch.float64, device=dev)
        zeros = torch.empty((out, groups), dtype=torch.float64, device=dev)
        for g, start in enumerate(range(0, inn, gs)):
            end = min(start + gs, inn)
            _kernels.gptq_qparams(work, start, end, bits, config.symmetric, False, scales[:, g], zeros[:, g], groups)
            _sweep(work, hinv, codes, scales[:, g], zeros[:, g], groups, bits, start, end)
        index_group = gs
    else:
        tensor = granularity == "tensor"
        rows = 1 if tensor else out
        scales = torch.empty((rows, 1), dtype=torch.float64, device=dev)
        zeros = torch.empty((rows, 1), dtype=torch.float64, device=dev)
        _kernels.gptq_qparams(work, 0, inn, bits, config.symmetric, tensor, scales, zeros, 1)
        stride = 0 if tensor else 1
        for start in range(0, inn, int(config.blocksize)):
            end = min(start + int(config.blocksize), inn)
            _sweep(work, hinv, codes, scales, zeros, stride, bits, start, end)
        index_group = inn
    return assemble_quantized(codes, scales, zeros, bits=bits, group_size=index_group,
                              symmetric=config.symmetric, granularity=granularity, channel_scale=None)
