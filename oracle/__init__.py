"""CPU oracle for the dequant-GEMM path (test infrastructure only).

This package is the checker, never the thing measured or shipped: only the test
suite, the smoke check and the benchmark's CPU-baseline leg import it. The
product package does not import it and has no CPU fallback.

Two implementations live here:

* ``liboracle.so`` (``dq_oracle.c``): a plain-C restatement of ptqkit's CPU
  dequant-GEMM (src/ptqkit/csrc/dequant_gemm.cpp:57-218), RTN quantizer
  (src/ptqkit/quant.py:146-184, 225-289) and int4 packing (src/ptqkit/pack.py:17-55).
* ``_ref/_kernels*.so``: ptqkit's own C++ kernel compiled from its single source
  file by ``oracle/Makefile`` (target ``ref``). Present only where it was built.

Both are pinned against outputs of the reference itself in ``tests/golden``.
"""

from __future__ import annotations

import ctypes
import glob
import importlib.util
import os
import subprocess
import sysconfig
from types import ModuleType

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
_lib: ctypes.CDLL | None = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build(with_ref: bool = False) -> None:
    """Compile the C oracle (and, if asked and its source is mounted, the reference kernel)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if with_ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        handle = ctypes.CDLL(_LIB_PATH)
        handle.orc_dequant_gemm.restype = ctypes.c_int
        handle.orc_dequant_gemm.argtypes = [
            _f32p, _u8p, _f32p, _f32p, _f32p, _f32p,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
        ]
        handle.orc_rtn_quantize.restype = ctypes.c_int
        handle.orc_rtn_quantize.argtypes = [
            _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, _i32p, _f32p, _f32p, _f32p,
        ]
        handle.orc_pack_int4.restype = ctypes.c_int
        handle.orc_pack_int4.argtypes = [_i32p, ctypes.c_int, ctypes.c_int, _u8p]
        handle.orc_unpack_int4.restype = None
        handle.orc_unpack_int4.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, _u8p]
        _lib = handle
    return _lib


def _ptr(a: np.ndarray | None, kind: type) -> ctypes._Pointer | None:  # type: ignore[type-arg]
    if a is None:
        return None
    return a.ctypes.data_as(ctypes.POINTER(kind))


def _c(a: np.ndarray, dtype: type) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def dequant_gemm(
    x: np.ndarray,
    q: np.ndarray,
    scales: np.ndarray,
    zeros: np.ndarray,
    channel_scale: np.ndarray | None,
    group_size: int,
    bits: int,
    nthreads: int = 0,
) -> np.ndarray:
    """y = x @ W_hat^T, bitwise equal to ptqkit's AVX2 CPU kernel."""
    x = _c(x, np.float32)
    q = _c(q, np.uint8)
    scales = _c(scales, np.float32)
    zeros = _c(zeros, np.float32)
    ch = None if channel_scale is None else _c(channel_scale, np.float32)
    B, K = x.shape
    M = q.shape[0]
    y = np.zeros((B, M), dtype=np.float32)
    rc = lib().orc_dequant_gemm(
        _ptr(x, ctypes.c_float), _ptr(q, ctypes.c_uint8), _ptr(scales, ctypes.c_float),
        _ptr(zeros, ctypes.c_float), _ptr(ch, ctypes.c_float), _ptr(y, ctypes.c_float),
        B, M, K, scales.shape[0], scales.shape[1], group_size, bits, nthreads,
    )
    if rc != 0:
        raise ValueError(f"oracle dequant_gemm rejected its arguments (status {rc})")
    return y


def rtn_quantize(
    w: np.ndarray,
    bits: int,
    symmetric: bool,
    group_size: int | None,
    pre_scale: np.ndarray | None = None,
) -> dict[str, np.ndarray | int]:
    """RTN of quant.py:225-289. Returns int32 codes, fp32 scales/zeros, the stored
    group_size (K for tensor and channel granularity) and the channel scale."""
    w = _c(w, np.float32)
    M, K = w.shape
    if group_size is None:
        mode, rows, groups, stored = -1, M, 1, K
    elif group_size == 0:
        mode, rows, groups, stored = 0, 1, 1, K
    else:
        mode, rows, groups, stored = group_size, M, (K + group_size - 1) // group_size, group_size
    codes = np.zeros((M, K), dtype=np.int32)
    scales = np.zeros((rows, groups), dtype=np.float32)
    zeros = np.zeros((rows, groups), dtype=np.float32)
    pre = None if pre_scale is None else _c(pre_scale, np.float32)
    channel = None if pre is None else np.zeros(K, dtype=np.float32)
    rc = lib().orc_rtn_quantize(
        _ptr(w, ctypes.c_float), _ptr(pre, ctypes.c_float), M, K, bits, int(symmetric), mode,
        _ptr(codes, ctypes.c_int32), _ptr(scales, ctypes.c_float), _ptr(zeros, ctypes.c_float),
        _ptr(channel, ctypes.c_float),
    )
    if rc == 2:
        raise ValueError("weight must be finite")
    if rc == 3:
        raise ValueError("pre_scale must be finite and positive")
    if rc != 0:
        raise ValueError(f"oracle rtn_quantize rejected its arguments (status {rc})")
    return {"codes": codes, "scales": scales, "zeros": zeros, "group_size": stored, "channel_scale": channel}


def pack_int4(codes: np.ndarray) -> np.ndarray:
    codes = _c(codes, np.int32)
    M, K = codes.shape
    out = np.zeros((M, (K + 1) // 2), dtype=np.uint8)
    if lib().orc_pack_int4(_ptr(codes, ctypes.c_int32), M, K, _ptr(out, ctypes.c_uint8)) != 0:
        raise ValueError("int4 codes must lie in [0, 15]")
    return out


def unpack_int4(packed: np.ndarray, in_features: int) -> np.ndarray:
    packed = _c(packed, np.uint8)
    M = packed.shape[0]
    out = np.zeros((M, in_features), dtype=np.uint8)
    lib().orc_unpack_int4(_ptr(packed, ctypes.c_uint8), M, in_features, _ptr(out, ctypes.c_uint8))
    return out


def quantize_stored(
    w: np.ndarray, bits: int, symmetric: bool, group_size: int | None, pre_scale: np.ndarray | None = None
) -> dict[str, np.ndarray | int]:
    """RTN followed by the storage step of assemble_quantized (quant.py:187-222):
    int4 codes packed, int8 codes as uint8."""
    r = rtn_quantize(w, bits, symmetric, group_size, pre_scale)
    codes = r["codes"]
    assert isinstance(codes, np.ndarray)
    r["q"] = pack_int4(codes) if bits == 4 else codes.astype(np.uint8)
    return r


def reference_kernels() -> ModuleType | None:
    """ptqkit's own compiled CPU kernel module from ``_ref/``, or None if not built."""
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    paths = glob.glob(os.path.join(HERE, "_ref", "_kernels" + suffix))
    if not paths:
        return None
    spec = importlib.util.spec_from_file_location("_kernels", paths[0])
    if spec is None or spec.loader is None:
        return None
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def dequantize(codes: np.ndarray, scales: np.ndarray, zeros: np.ndarray, channel: np.ndarray | None,
               group_size: int) -> np.ndarray:
    """W_hat in fp32 with quant.py:292-308's operation order: (codes - zero) * scale [* channel]."""
    codes = np.asarray(codes, dtype=np.float32)
    idx = np.arange(codes.shape[1]) // group_size
    rows = scales.shape[0]
    sc = scales[0, idx][None, :] if rows == 1 else scales[:, idx]
    zr = zeros[0, idx][None, :] if rows == 1 else zeros[:, idx]
    hat = ((codes - zr).astype(np.float32) * sc).astype(np.float32)
    if channel is not None:
        hat = (hat * channel[None, :]).astype(np.float32)
    return hat


def awq_search(
    w: np.ndarray,
    x: np.ndarray,
    bits: int,
    symmetric: bool,
    group_size: int | None,
    alphas: tuple[float, ...],
    mean_abs: np.ndarray | None = None,
) -> dict[str, object]:
    """The alpha search of src/ptqkit/awq.py:39-81 restated in numpy plus this
    package's C RTN: channel magnitudes and scores in fp64, pre-scales rounded
    to fp32 as the reference does (m^alpha, then the division by the clamped
    mean). Returns the winning alpha, every alpha's score and pre-scale, and the
    winner's RTN outputs."""
    w = _c(w, np.float32)
    x = np.asarray(x, dtype=np.float32)
    if mean_abs is None:
        mag = np.abs(x.astype(np.float64)).mean(axis=0).astype(np.float32)
    else:
        mag = np.asarray(mean_abs, dtype=np.float32).reshape(-1)
    mag = np.maximum(mag, np.float32(1e-8))
    n = x.shape[0]
    search = x if n <= 2048 else x[:: max(n // 2048, 1)][:2048]
    s64 = search.astype(np.float64)
    target = s64 @ w.astype(np.float64).T
    best_alpha, best_mse, best = float(alphas[0]), float("inf"), None
    mses, pres = [], []
    for a in alphas:
        a = float(a)
        if a == 0.0:
            pre = np.ones(w.shape[1], dtype=np.float32)
        else:
            # torch's pow on an fp32 tensor takes the scalar exponent as fp32
            # (0.3 becomes 0.300000012); the power of that exponent is taken
            # in fp64 and rounded once to fp32
            p = (mag.astype(np.float64) ** float(np.float32(a))).astype(np.float32)
            mean = np.float32(p.astype(np.float64).mean())
            mean = max(mean, np.float32(1e-8))
            pre = (p / mean).astype(np.float32)
        r = rtn_quantize(w, bits, symmetric, group_size, pre)
        hat = dequantize(r["codes"], r["scales"], r["zeros"], r["channel_scale"], int(r["group_size"]))
        err = s64 @ hat.astype(np.float64).T - target
        mse = float((err * err).mean()) if err.size else float("nan")
        mses.append(mse)
        pres.append(pre)
        if mse < best_mse:
            best_alpha, best_mse, best = a, mse, r
    return {"alpha": best_alpha, "mse": mses, "pre_scale": pres, "rtn": best, "mag": mag}


def _qparams64(block: np.ndarray, symmetric: bool, bits: int) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:146-172 on an fp64 [rows, cols] block; returns [rows] scale, zero."""
    qmax = (1 << bits) - 1
    if symmetric:
        amax = np.abs(block).max(axis=1)
        scale = np.where(amax > 0, (2 * amax) / qmax, 1.0)
        return scale, np.full_like(scale, (qmax + 1) / 2.0)
    xmin = np.minimum(block.min(axis=1), 0.0)
    xmax = np.maximum(block.max(axis=1), 0.0)
    deg = (xmin == 0) & (xmax == 0)
    xmin = np.where(deg, -1.0, xmin)
    xmax = np.where(deg, 1.0, xmax)
    scale = (xmax - xmin) / qmax
    scale = np.where(scale > 0, scale, 1.0)
    zero = np.clip(np.rint(-xmin / scale), 0, qmax)
    return scale, zero


def gptq_factor(hessian: np.ndarray, percdamp: float) -> np.ndarray:
    """Upper Cholesky factor of the damped inverse Hessian (src/ptqkit/gptq.py:44-71)."""
    import scipy.linalg

    h = 0.5 * (hessian + hessian.T)
    dead = np.diag(h) == 0
    if dead.any():
        h = h.copy()
        h[dead, :] = 0
        h[:, dead] = 0
        idx = np.arange(h.shape[0])[dead]
        h[idx, idx] = 1
    damp = percdamp * np.mean(np.diag(h))
    if not np.isfinite(damp) or damp < 0:
        damp = 0.0
    h = h.copy()
    h[np.diag_indices_from(h)] += damp
    for _ in range(6):
        try:
            low = np.linalg.cholesky(h)
            inv = scipy.linalg.cho_solve((low, True), np.eye(h.shape[0]))
            return np.linalg.cholesky(inv).T
        except np.linalg.LinAlgError:
            h[np.diag_indices_from(h)] += np.mean(np.diag(h)) * 0.1 + 1e-6
    raise RuntimeError("damped Hessian Cholesky failed")


def gptq_quantize(
    w: np.ndarray,
    hessian: np.ndarray,
    bits: int,
    symmetric: bool,
    group_size: int | None,
    percdamp: float = 0.01,
    blocksize: int = 128,
    hinv: np.ndarray | None = None,
) -> dict[str, np.ndarray | int]:
    """src/ptqkit/gptq.py:86-191 restated in numpy fp64 (the OBS sweep column by
    column, as _obs_block). ``hinv`` replaces the factorization when given."""
    work = np.array(w, dtype=np.float64)
    h = np.asarray(hessian, dtype=np.float64)
    dead = np.diag(h) == 0
    work[:, dead] = 0
    u = gptq_factor(h, percdamp) if hinv is None else np.asarray(hinv, dtype=np.float64)
    out, inn = work.shape
    qmax = (1 << bits) - 1
    codes = np.zeros((out, inn), dtype=np.int32)

    def obs_block(sc: np.ndarray, zz: np.ndarray, start: int, end: int) -> None:
        block = work[:, start:end].copy()
        err_block = np.zeros_like(block)
        for i in range(end - start):
            col = block[:, i].copy()
            d = u[start + i, start + i]
            q = np.clip(np.rint(col / sc) + zz, 0, qmax)
            deq = sc * (q - zz)
            codes[:, start + i] = q.astype(np.int32)
            err = (col - deq) / max(d, 1e-8)
            if not np.isfinite(err).all():
                err = np.zeros_like(col)
            block[:, i:] = block[:, i:] - err[:, None] * u[start + i, start + i:end][None, :]
            err_block[:, i] = err
        if end < inn:
            work[:, end:] = work[:, end:] - err_block @ u[start:end, end:]

    if group_size is not None and group_size > 0:
        scs, zzs = [], []
        for start in range(0, inn, group_size):
            end = min(start + group_size, inn)
            sc, zz = _qparams64(work[:, start:end], symmetric, bits)
            obs_block(sc, zz, start, end)
            scs.append(sc)
            zzs.append(zz)
        scales, zeros, stored = np.stack(scs, axis=1), np.stack(zzs, axis=1), group_size
    else:
        if group_size == 0:
            sc, zz = _qparams64(work.reshape(1, -1), symmetric, bits)
            scales, zeros = sc.reshape(1, 1), zz.reshape(1, 1)
            scv, zzv = np.full(out, sc[0]), np.full(out, zz[0])
        else:
            sc, zz = _qparams64(work, symmetric, bits)
            scales, zeros = sc.reshape(-1, 1), zz.reshape(-1, 1)
            scv, zzv = sc, zz
        for start in range(0, inn, blocksize):
            obs_block(scv, zzv, start, min(start + blocksize, inn))
        stored = inn
    return {"codes": codes, "scales": scales.astype(np.float32), "zeros": zeros.astype(np.float32),
            "group_size": stored, "hinv": u}
