"""ctypes binding of ``libwq_b200.so``, the counterpart of ptqkit's native module.

ptqkit's ``_kernels`` (src/ptqkit/_kernels.pyi:3-12, src/ptqkit/csrc/dequant_gemm.cpp:317-331)
exposes ``dequant_gemm(x, q, scales, zeros, channel_scale, group_size, bits, nthreads)``
and ``kernel_info()``. This module exposes the same two with the same argument
names and error behaviour (``ValueError`` with the reference's messages for bad
arguments), operating on CUDA tensors through the library's C ABI
(``include/wq_b200.h``), plus the device RTN, packing and reconstruction entry points.

PyTorch only supplies device memory and the current stream. There is no CPU
path: if the library is missing, every call raises.
"""

from __future__ import annotations

import ctypes
import os
from typing import Any

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwq_b200.so")

WQ_OK = 0
WQ_E_CUDA = 14
_ARG_ERRORS_AS_VALUEERROR = {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 15, 16, 17, 18, 19, 20, 21, 22}

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every symbol declared in include/wq_b200.h
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "wq_status_string": (ctypes.c_char_p, [_int]),
    "wq_last_cuda_error": (ctypes.c_char_p, []),
    "wq_fault_status": (_int, [_int, ctypes.POINTER(ctypes.c_uint32)]),
    "wq_selftest_expired_wait": (_int, [ctypes.c_uint32, _vp]),
    "wq_kernel_info": (_int, [_int, _vp]),
    "wq_dequant_gemm_workspace_bytes": (_sz, [_i64, _i64, _i64, _int, _int]),
    "wq_dequant_gemm_f32": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
         _int, _int, _vp, _i64, _vp, _sz, _vp],
    ),
    "wq_rtn_workspace_bytes": (_sz, [_i64, _i64, _int]),
    "wq_rtn_quantize_f32": (
        _int,
        [_vp, _vp, _i64, _i64, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    ),
    "wq_rtn_flags_status": (_int, [ctypes.c_int32]),
    "wq_pack_int4": (_int, [_vp, _i64, _i64, _vp, _vp, _vp]),
    "wq_unpack_int4": (_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "wq_dequantize_f32": (
        _int, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _int, _int, _vp, _vp]
    ),
    "wq_gather_permute_f32": (_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "wq_dequant_gemm_f32_noalloc": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
         _int, _int, _vp, _i64, _vp],
    ),
    "wq_widen_f16_f32": (_int, [_vp, _vp, _i64, _vp]),
    "wq_narrow_f32_f16": (_int, [_vp, _vp, _i64, _vp]),
    "wq_ipc_handle_bytes": (_sz, []),
    "wq_ipc_get_handle": (_int, [_vp, _vp, ctypes.POINTER(ctypes.c_int64)]),
    "wq_ipc_open_handle": (_int, [_vp, _i64, ctypes.POINTER(ctypes.c_void_p)]),
    "wq_ipc_close_handle": (_int, [_vp, _i64]),
    "wq_channel_abs_sum_f64": (_int, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "wq_awq_pre_scale_f32": (_int, [_vp, _i64, ctypes.c_float, _vp, _vp]),
    "wq_sq_err_workspace_bytes": (_sz, []),
    "wq_sq_err_sum_f64": (_int, [_vp, _vp, _i64, _vp, _vp, _sz, _vp]),
    "wq_gptq_qparams_workspace_bytes": (_sz, [_i64]),
    "wq_gptq_qparams_f64": (_int, [_vp, _i64, _i64, _i64, _i64, _int, _int, _int, _vp, _vp, _i64, _vp, _sz, _vp]),
    "wq_gptq_block_f64": (
        _int, [_vp, _i64, _i64, _vp, _i64, _i64, _int, _vp, _vp, _i64, _int, _vp, _i64, _vp, _vp, _vp, _vp]),
    "wq_gptq_tail_f64": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _int, _vp, _i64, _i64, _vp]),
    "wq_chol_inverse_upper_workspace_bytes": (_sz, [_i64]),
    "wq_chol_inverse_upper_f64": (_int, [_vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp, _vp]),
    "wq_dequant_gemm_f32_multi": (
        _int,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64,
         _int, _int, _vp, _int, _i64, _vp, _vp, _vp, _sz, _vp],
    ),
}

MAX_OUTPUTS = 8


class _KernelInfo(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int),
        ("compiled_sm", ctypes.c_int),
        ("device", ctypes.c_int),
        ("device_cc", ctypes.c_int),
        ("sm_count", ctypes.c_int),
        ("tcgen05", ctypes.c_int),
        ("device_name", ctypes.c_char * 96),
    ]


_lib: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Load the in-tree C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"wq_b200 CUDA library not found at {LIB_PATH}; build it with "
                "`make -C weight-quantizer_b200/csrc` (or __graft_entry__.build())"
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_message(status: int) -> str:
    msg: bytes = library().wq_status_string(status)
    return msg.decode()


def _check(status: int) -> None:
    if status == WQ_OK:
        return
    if status == WQ_E_CUDA:
        detail: bytes = library().wq_last_cuda_error()
        raise RuntimeError(f"wq_b200: {detail.decode()}")
    if status in _ARG_ERRORS_AS_VALUEERROR:
        raise ValueError(status_message(status))
    raise RuntimeError(f"wq_b200: status {status}")


def _stream(device: torch.device) -> int:
    return int(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else int(t.data_ptr())


def _cuda_device(tensors: list[torch.Tensor]) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise ValueError("dequant kernel inputs must be CUDA tensors")
        if t.device != dev:
            raise ValueError("dequant kernel inputs must be on one CUDA device")
    return dev


def fault_status(reset: bool = True) -> int:
    """The current device's fault word (nonzero: a bounded pipeline wait
    expired in some launch since the last reset). Synchronizes the device."""
    v = ctypes.c_uint32(0)
    _check(library().wq_fault_status(int(reset), ctypes.byref(v)))
    return int(v.value)


# Checked mode: after every dequant-GEMM call, read (and clear) the fault word
# and raise if a kernel set it. Reading it synchronizes the device, so it is
# off by default; WQ_CHECK_FAULTS=1 in the environment or set_fault_check(True)
# turns it on. Without it, fault_status() is the way to learn of an expired
# wait (the kernels never hang on one: they stop waiting and finish).
_fault_check = os.environ.get("WQ_CHECK_FAULTS", "") not in ("", "0")


def set_fault_check(on: bool) -> bool:
    """Turn checked mode on or off; returns the previous setting."""
    global _fault_check
    prev = _fault_check
    _fault_check = bool(on)
    return prev


def _raise_on_fault() -> None:
    v = fault_status(reset=True)
    if v:
        raise RuntimeError(
            f"wq_b200: a kernel set the fault word ({v:#x}; bit 0 = a bounded pipeline wait expired), "
            "so its output is not valid")


def selftest_expired_wait(max_polls: int = 16, device: torch.device | None = None) -> None:
    """Launch the library's self-test of fault reporting: a wait on a barrier
    that nothing arrives on, given up after ``max_polls`` polls, which sets bit
    0 of the fault word the way an expired pipeline wait does."""
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    _check(library().wq_selftest_expired_wait(int(max_polls), _stream(dev)))


def kernel_info(device: int | None = None) -> dict[str, Any]:
    """Build and device facts (counterpart of ``_kernels.kernel_info``)."""
    if device is None:
        device = torch.cuda.current_device() if torch.cuda.is_available() else 0
    info = _KernelInfo()
    status = library().wq_kernel_info(int(device), ctypes.byref(info))
    out: dict[str, Any] = {
        "abi_version": info.abi_version,
        "arch": f"sm_{info.compiled_sm}a",
        "tcgen05": bool(info.tcgen05),
    }
    if status == WQ_OK:
        out.update(device=info.device_name.decode(), device_cc=info.device_cc, sm_count=info.sm_count)
    return out


def dequant_gemm(
    x: torch.Tensor,
    q: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    channel_scale: torch.Tensor | None,
    group_size: int,
    bits: int,
    nthreads: int = 0,
    *,
    out: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
) -> torch.Tensor:
    """y[B, M] = x[B, K] @ W_hat^T (+ bias) on the current CUDA stream.

    Same arguments as ptqkit's ``_kernels.dequant_gemm``. Inputs are cast to
    fp32/uint8 and made contiguous like the reference's ``forcecast | c_style``
    arrays (dequant_gemm.cpp:223-226). ``nthreads`` is accepted and ignored.
    ``out`` may be a preallocated fp32 [B, M] view with unit column stride.
    ``bias`` (fp32 [M], no reference counterpart at this level: ptqkit adds it
    in QuantizedLinear.forward) is added in the kernels' epilogue.
    """
    del nthreads
    if x.ndim != 2:
        raise ValueError("x must have shape [B, K]")
    if q.ndim != 2 or scales.ndim != 2 or zeros.ndim != 2:
        raise ValueError("q, scales, and zeros must be rank 2")
    tensors = [x, q, scales, zeros] + ([] if channel_scale is None else [channel_scale])
    dev = _cuda_device(tensors)
    x = x.to(dtype=torch.float32).contiguous()
    q = q.to(dtype=torch.uint8).contiguous()
    scales = scales.to(dtype=torch.float32).contiguous()
    zeros = zeros.to(dtype=torch.float32).contiguous()
    ch_len = -1
    if channel_scale is not None:
        channel_scale = channel_scale.to(dtype=torch.float32).contiguous()
        if channel_scale.ndim != 1:
            raise ValueError("channel_scale must have shape [K]")
        ch_len = int(channel_scale.shape[0])
    B, K = int(x.shape[0]), int(x.shape[1])
    M = int(q.shape[0])
    if out is None:
        y = torch.empty((B, M), dtype=torch.float32, device=dev)
        ldy = M
    else:
        if out.dtype != torch.float32 or out.device != dev or tuple(out.shape) != (B, M):
            raise ValueError("out must be a float32 [B, M] tensor on the inputs' device")
        if M > 0 and B > 1 and out.stride(1) != 1:
            raise ValueError("out must have unit column stride")
        y = out
        ldy = int(out.stride(0)) if B > 1 else M
    lib = library()
    ws_bytes = int(lib.wq_dequant_gemm_workspace_bytes(B, M, K, int(group_size), int(bits)))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
    if bias is None:
        status = lib.wq_dequant_gemm_f32(
            _ptr(x), B, K,
            _ptr(q), M, int(q.shape[1]),
            _ptr(scales), int(scales.shape[0]), int(scales.shape[1]),
            _ptr(zeros), int(zeros.shape[0]), int(zeros.shape[1]),
            _ptr(channel_scale), ch_len,
            int(group_size), int(bits),
            _ptr(y), ldy,
            _ptr(ws), ws_bytes,
            _stream(dev),
        )
    else:
        b = _bias_arg(bias, M, dev)
        arr = (ctypes.c_void_p * 1)(ctypes.c_void_p(y.data_ptr() if y.numel() else 0))
        status = lib.wq_dequant_gemm_f32_multi(
            _ptr(x), B, K,
            _ptr(q), M, int(q.shape[1]),
            _ptr(scales), int(scales.shape[0]), int(scales.shape[1]),
            _ptr(zeros), int(zeros.shape[0]), int(zeros.shape[1]),
            _ptr(channel_scale), ch_len,
            int(group_size), int(bits),
            ctypes.cast(arr, ctypes.c_void_p), 1, ldy, None, _ptr(b),
            _ptr(ws), ws_bytes,
            _stream(dev),
        )
    _check(status)
    if _fault_check:
        _raise_on_fault()
    return y


def rtn_quantize(
    w: torch.Tensor,
    bits: int,
    symmetric: bool,
    group_mode: int,
    pre_scale: torch.Tensor | None = None,
) -> dict[str, torch.Tensor]:
    """Device RTN + pack. ``group_mode``: >0 group size, 0 per-tensor, -1 per-channel.

    Returns stored codes (packed for int4), fp32 scales/zeros and, with
    ``pre_scale``, the stored channel scale 1/s. Reads the status flags back
    (one host synchronization), as the reference raises before returning."""
    if w.ndim != 2:
        raise ValueError("weight must have shape [out, in]")
    dev = _cuda_device([w] + ([] if pre_scale is None else [pre_scale]))
    w = w.to(dtype=torch.float32).contiguous()
    M, K = int(w.shape[0]), int(w.shape[1])
    if pre_scale is not None:
        pre_scale = pre_scale.to(dtype=torch.float32).reshape(-1).contiguous()
        if int(pre_scale.numel()) != K:
            raise ValueError("pre_scale must have one entry per input channel")
    if group_mode > 0:
        rows, groups = M, (K + group_mode - 1) // group_mode
    elif group_mode == 0:
        rows, groups = 1, 1
    else:
        rows, groups = M, 1
    cols = (K + 1) // 2 if bits == 4 else K
    q = torch.empty((M, cols), dtype=torch.uint8, device=dev)
    scales = torch.empty((rows, groups), dtype=torch.float32, device=dev)
    zeros = torch.empty((rows, groups), dtype=torch.float32, device=dev)
    channel = torch.empty(K, dtype=torch.float32, device=dev) if pre_scale is not None else None
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = library()
    ws_bytes = int(lib.wq_rtn_workspace_bytes(M, K, int(group_mode)))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
    status = lib.wq_rtn_quantize_f32(
        _ptr(w), _ptr(pre_scale), M, K, int(bits), int(bool(symmetric)), int(group_mode),
        _ptr(q), _ptr(scales), _ptr(zeros), _ptr(channel), _ptr(flags), _ptr(ws), ws_bytes,
        _stream(dev),
    )
    _check(status)
    _check(int(lib.wq_rtn_flags_status(int(flags.item()))))
    out = {"codes": q, "scales": scales, "zeros": zeros}
    if channel is not None:
        out["channel_scale"] = channel
    return out


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """codes [M, K] in [0, 15] -> packed uint8 [M, ceil(K/2)] (pack.py:17-33)."""
    if codes.ndim != 2:
        raise ValueError("codes must have shape [M, K]")
    dev = _cuda_device([codes])
    c = codes.to(dtype=torch.int32).contiguous()
    M, K = int(c.shape[0]), int(c.shape[1])
    packed = torch.empty((M, (K + 1) // 2), dtype=torch.uint8, device=dev)
    mm = torch.empty(2, dtype=torch.int32, device=dev)
    _check(library().wq_pack_int4(_ptr(c), M, K, _ptr(packed), _ptr(mm), _stream(dev)))
    if M * K > 0:
        lo, hi = (int(v) for v in mm.tolist())
        if lo < 0 or hi > 15:
            raise ValueError(f"int4 codes must lie in [0, 15], got [{lo}, {hi}]")
    return packed


def unpack_int4(packed: torch.Tensor, in_features: int) -> torch.Tensor:
    """Invert pack_int4 and drop the pad nibble (pack.py:36-55)."""
    if packed.ndim != 2 or packed.dtype != torch.uint8:
        raise ValueError("packed int4 storage must be a uint8 matrix")
    if in_features < 0:
        raise ValueError("in_features must be non-negative")
    need = (in_features + 1) // 2
    if packed.shape[1] < need:
        raise ValueError("packed row is shorter than in_features")
    dev = _cuda_device([packed])
    p = packed.contiguous()
    M = int(p.shape[0])
    out = torch.empty((M, in_features), dtype=torch.uint8, device=dev)
    _check(library().wq_unpack_int4(_ptr(p), M, int(p.shape[1]), int(in_features), _ptr(out), _stream(dev)))
    return out


def dequantize(
    q: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    channel_scale: torch.Tensor | None,
    in_features: int,
    group_size: int,
    bits: int,
) -> torch.Tensor:
    """W_hat fp32 [M, K] exactly as quant.py:292-308 computes it."""
    dev = _cuda_device([q, scales, zeros] + ([] if channel_scale is None else [channel_scale]))
    q = q.contiguous()
    scales = scales.to(dtype=torch.float32).contiguous()
    zeros = zeros.to(dtype=torch.float32).contiguous()
    if channel_scale is not None:
        channel_scale = channel_scale.to(dtype=torch.float32).contiguous()
    M, K = int(q.shape[0]), int(in_features)
    out = torch.empty((M, K), dtype=torch.float32, device=dev)
    _check(
        library().wq_dequantize_f32(
            _ptr(q), M, K, int(q.shape[1]), _ptr(scales), int(scales.shape[0]), int(scales.shape[1]),
            _ptr(zeros), _ptr(channel_scale), int(group_size), int(bits), _ptr(out), _stream(dev),
        )
    )
    return out


def gather_permute(src: torch.Tensor, parts: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """[P, B, Mp] (row-sharded outputs stacked by rank) -> [B, P*Mp]."""
    dev = _cuda_device([src])
    P, B, Mp = int(src.shape[0]), int(src.shape[1]), int(src.shape[2])
    if P != parts:
        raise ValueError("leading dimension must equal the number of parts")
    s = src.contiguous()
    dst = out if out is not None else torch.empty((B, P * Mp), dtype=torch.float32, device=dev)
    _check(library().wq_gather_permute_f32(_ptr(s), P, B, Mp, _ptr(dst), _stream(dev)))
    return dst


def dequant_gemm_multi(
    x: torch.Tensor,
    q: torch.Tensor,
    scales: torch.Tensor,
    zeros: torch.Tensor,
    channel_scale: torch.Tensor | None,
    group_size: int,
    bits: int,
    outputs: list[int],
    ldy: int,
    y_all: int = 0,
    bias: torch.Tensor | None = None,
) -> None:
    """dequant_gemm writing the same [B, M] result (row stride ``ldy``) into
    every device pointer of ``outputs`` (this GPU's buffers or peer buffers
    mapped with :func:`ipc_open`). The first output must be on the inputs'
    device; the tensor-core path stores into all of them from its epilogue.
    ``y_all`` (nonzero) is an NVLink-switch address that reaches every rank's
    buffer at once; the tensor-core epilogue then stores through it alone.
    ``bias`` (fp32 [M]) is added to every output row in the kernels' epilogue."""
    if x.ndim != 2:
        raise ValueError("x must have shape [B, K]")
    if q.ndim != 2 or scales.ndim != 2 or zeros.ndim != 2:
        raise ValueError("q, scales, and zeros must be rank 2")
    if not 1 <= len(outputs) <= MAX_OUTPUTS:
        raise ValueError(f"between 1 and {MAX_OUTPUTS} outputs")
    tensors = [x, q, scales, zeros] + ([] if channel_scale is None else [channel_scale])
    dev = _cuda_device(tensors)
    x = x.to(dtype=torch.float32).contiguous()
    q = q.to(dtype=torch.uint8).contiguous()
    scales = scales.to(dtype=torch.float32).contiguous()
    zeros = zeros.to(dtype=torch.float32).contiguous()
    ch_len = -1
    if channel_scale is not None:
        channel_scale = channel_scale.to(dtype=torch.float32).contiguous()
        ch_len = int(channel_scale.shape[0])
    B, K = int(x.shape[0]), int(x.shape[1])
    M = int(q.shape[0])
    lib = library()
    ws_bytes = int(lib.wq_dequant_gemm_workspace_bytes(B, M, K, int(group_size), int(bits)))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
    arr = (ctypes.c_void_p * len(outputs))(*[ctypes.c_void_p(int(o)) for o in outputs])
    status = lib.wq_dequant_gemm_f32_multi(
        _ptr(x), B, K,
        _ptr(q), M, int(q.shape[1]),
        _ptr(scales), int(scales.shape[0]), int(scales.shape[1]),
        _ptr(zeros), int(zeros.shape[0]), int(zeros.shape[1]),
        _ptr(channel_scale), ch_len,
        int(group_size), int(bits),
        ctypes.cast(arr, ctypes.c_void_p), len(outputs), int(ldy), ctypes.c_void_p(int(y_all)) if y_all else None,
        _ptr(_bias_arg(bias, int(q.shape[0]), dev)),
        _ptr(ws), ws_bytes,
        _stream(dev),
    )
    _check(status)
    if _fault_check:
        _raise_on_fault()


def _bias_arg(bias: torch.Tensor | None, M: int, dev: torch.device) -> torch.Tensor | None:
    if bias is None:
        return None
    if bias.device != dev:
        raise ValueError("bias must be on the inputs' device")
    bias = bias.to(dtype=torch.float32).contiguous().reshape(-1)
    if int(bias.numel()) != M:
        raise ValueError("bias does not match out_features")
    return bias


def ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """IPC handle of the device allocation holding ``t`` and t's byte offset in it."""
    lib = library()
    n = int(lib.wq_ipc_handle_bytes())
    buf = ctypes.create_string_buffer(n)
    off = ctypes.c_int64(0)
    _check(lib.wq_ipc_get_handle(ctypes.c_void_p(t.data_ptr()), buf, ctypes.byref(off)))
    return bytes(buf.raw), int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Maps another process's allocation; returns the device pointer at ``offset``."""
    lib = library()
    ptr = ctypes.c_void_p(0)
    _check(lib.wq_ipc_open_handle(ctypes.c_char_p(handle), int(offset), ctypes.byref(ptr)))
    return int(ptr.value or 0)


def ipc_close(ptr: int, offset: int) -> None:
    _check(library().wq_ipc_close_handle(ctypes.c_void_p(int(ptr)), int(offset)))


def widen_f16_f32(src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 -> fp32 (exact) on the device; ``out`` (fp32, same element count) is
    written in place when given. Used by the compressed-format loader."""
    dev = _cuda_device([src] if out is None else [src, out])
    if src.dtype != torch.float16:
        raise ValueError("widen_f16_f32 expects a float16 tensor")
    s = src.contiguous()
    dst = out if out is not None else torch.empty(s.shape, dtype=torch.float32, device=dev)
    if dst.dtype != torch.float32 or not dst.is_contiguous() or dst.numel() != s.numel():
        raise ValueError("out must be a contiguous float32 tensor with the input's element count")
    _check(library().wq_widen_f16_f32(_ptr(s), _ptr(dst), int(s.numel()), _stream(dev)))
    return dst


def narrow_f32_f16(src: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 -> fp16 (round to nearest even) on the device, as compressed_state
    stores scales, zeros and channel scales (convert.py:318-323)."""
    dev = _cuda_device([src] if out is None else [src, out])
    if src.dtype != torch.float32:
        raise ValueError("narrow_f32_f16 expects a float32 tensor")
    s = src.contiguous()
    dst = out if out is not None else torch.empty(s.shape, dtype=torch.float16, device=dev)
    if dst.dtype != torch.float16 or not dst.is_contiguous() or dst.numel() != s.numel():
        raise ValueError("out must be a contiguous float16 tensor with the input's element count")
    _check(library().wq_narrow_f32_f16(_ptr(s), _ptr(dst), int(s.numel()), _stream(dev)))
    return dst


# ---- AWQ search reductions (src/ptqkit/awq.py:39-81, convert.py:35-63) -------


def channel_abs_sum(x: torch.Tensor, acc: torch.Tensor | None = None) -> torch.Tensor:
    """acc[k] += sum_i |x[i, k]| in fp64 (rows in order); returns acc (fp64 [K]).

    ActivationStats.update's ``x64.abs().sum(dim=0)`` (convert.py:47-48); a new
    zeroed accumulator is made when ``acc`` is None.
    """
    if x.ndim != 2:
        raise ValueError("activations must have shape [n, in]")
    dev = _cuda_device([x])
    x = x.to(dtype=torch.float32)
    if x.stride(1) != 1:
        x = x.contiguous()
    n, k = int(x.shape[0]), int(x.shape[1])
    if acc is None:
        acc = torch.zeros(k, dtype=torch.float64, device=dev)
    elif acc.dtype != torch.float64 or acc.device != dev or int(acc.numel()) != k or not acc.is_contiguous():
        raise ValueError("acc must be a contiguous fp64 [in] tensor on the activations' device")
    ld = int(x.stride(0)) if n > 1 else k
    _check(library().wq_channel_abs_sum_f64(_ptr(x), n, k, ld, _ptr(acc), _stream(dev)))
    return acc


def awq_pre_scale(mag: torch.Tensor, alpha: float) -> torch.Tensor:
    """s = mag^alpha / max(mean(mag^alpha), 1e-8) in fp32 (awq.py:68-74); 1 for alpha = 0."""
    dev = _cuda_device([mag])
    m = mag.to(dtype=torch.float32).contiguous().reshape(-1)
    pre = torch.empty_like(m)
    _check(library().wq_awq_pre_scale_f32(_ptr(m), int(m.numel()), float(alpha), _ptr(pre), _stream(dev)))
    return pre


def sq_err_sum(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """sum (a - b)^2 over all elements, in fp64, as a device scalar (awq.py:76-77)."""
    if a.shape != b.shape:
        raise ValueError("operands must have the same shape")
    dev = _cuda_device([a, b])
    a = a.to(dtype=torch.float32).contiguous()
    b = b.to(dtype=torch.float32).contiguous()
    lib = library()
    ws_bytes = int(lib.wq_sq_err_workspace_bytes())
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty((), dtype=torch.float64, device=dev)
    _check(lib.wq_sq_err_sum_f64(_ptr(a), _ptr(b), int(a.numel()), _ptr(out), _ptr(ws), ws_bytes, _stream(dev)))
    return out


# ---- GPTQ column sweep (src/ptqkit/gptq.py:86-191) ---------------------------


def gptq_qparams(w: torch.Tensor, c0: int, c1: int, bits: int, symmetric: bool, per_tensor: bool,
                 scale_out: torch.Tensor, zero_out: torch.Tensor, out_stride: int) -> None:
    """quant.py:146-172 in fp64 over columns [c0, c1) of w, per row (into
    scale_out[r * out_stride]) or over the whole range (into [0])."""
    dev = _cuda_device([w, scale_out, zero_out])
    if w.dtype != torch.float64 or w.stride(1) != 1:
        raise ValueError("w must be an fp64 matrix with unit column stride")
    lib = library()
    rows = int(w.shape[0])
    ws_bytes = int(lib.wq_gptq_qparams_workspace_bytes(rows)) if per_tensor else 0
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
    _check(lib.wq_gptq_qparams_f64(_ptr(w), rows, int(w.stride(0)), int(c0), int(c1), int(bits), int(symmetric),
                                   int(per_tensor), _ptr(scale_out), _ptr(zero_out), int(out_stride), _ptr(ws),
                                   ws_bytes, _stream(dev)))


def gptq_block(w: torch.Tensor, hinv: torch.Tensor, s0: int, count: int, scale: torch.Tensor,
               zero: torch.Tensor, qp_stride: int, bits: int, codes: torch.Tensor, err_block: torch.Tensor,
               zero_err: torch.Tensor | None = None, bad_col: torch.Tensor | None = None) -> None:
    """_obs_block's column sweep over [s0, s0 + count) (gptq.py:86-121): writes
    codes[:, s0:s0 + count] and the OBS errors into err_block [rows, count].
    ``zero_err`` (uint8 [count]) marks columns whose error counts as 0;
    ``bad_col`` (int32 [1], preset to 2^31 - 1) receives the first other
    column whose error is not finite in some row."""
    dev = _cuda_device([w, hinv, scale, zero, codes, err_block])
    for t in (w, hinv, scale, zero, err_block):
        if t.dtype != torch.float64:
            raise ValueError("GPTQ operands are fp64")
    if codes.dtype != torch.int32 or not err_block.is_contiguous() or w.stride(1) != 1 or hinv.stride(1) != 1:
        raise ValueError("codes must be int32; w, hinv row-major; err_block contiguous")
    _check(library().wq_gptq_block_f64(_ptr(w), int(w.shape[0]), int(w.stride(0)), _ptr(hinv), int(hinv.stride(0)),
                                       int(s0), int(count), _ptr(scale), _ptr(zero), int(qp_stride), int(bits),
                                       _ptr(codes), int(codes.stride(0)), _ptr(err_block), _ptr(zero_err),
                                       _ptr(bad_col), _stream(dev)))


def gptq_tail(w: torch.Tensor, c0: int, err_block: torch.Tensor, hinv: torch.Tensor, s0: int) -> None:
    """w[:, c0:] -= err_block @ hinv[s0:s0 + count, c0:] in fp64 (gptq.py:124-125),
    this library's kernel, the sum over the block's columns in order."""
    dev = _cuda_device([w, err_block, hinv])
    rows, count = int(err_block.shape[0]), int(err_block.shape[1])
    ncols = int(w.shape[1]) - int(c0)
    if not err_block.is_contiguous() or w.stride(1) != 1 or hinv.stride(1) != 1:
        raise ValueError("err_block contiguous; w, hinv row-major")
    _check(library().wq_gptq_tail_f64(_ptr(w), rows, int(w.stride(0)), int(c0), ncols, _ptr(err_block), count,
                                      _ptr(hinv), int(hinv.stride(0)), int(s0), _stream(dev)))


def chol_inverse_upper(a: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """U with U^T U = a^-1 (a symmetric positive definite, fp64, on the GPU;
    its upper triangle is read): the factor of gptq.py:59-66, on this
    library's kernels. Returns (U, info): info is a one-element int32 device
    tensor, 0, or 1 + a column whose pivot was not positive and finite (U is
    then not valid); nothing here waits for the GPU."""
    dev = _cuda_device([a])
    if a.dtype != torch.float64 or a.ndim != 2 or a.shape[0] != a.shape[1] or a.stride(1) != 1:
        raise ValueError("a must be a square row-major fp64 matrix")
    n = int(a.shape[0])
    u = torch.empty((n, n), dtype=torch.float64, device=dev)
    info = torch.empty(1, dtype=torch.int32, device=dev)
    ws_bytes = int(library().wq_chol_inverse_upper_workspace_bytes(n))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    _check(library().wq_chol_inverse_upper_f64(_ptr(a), n, int(a.stride(0)), _ptr(u), n, _ptr(ws), ws_bytes,
                                               _ptr(info), _stream(dev)))
    return u, info
