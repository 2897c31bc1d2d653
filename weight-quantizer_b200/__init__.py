"""wq_b200: the dequant-GEMM hot path of ptqkit (cvs0/weight-quantizer) on B200 (sm_100a).

y[b, m] = sum_k scale[m, g] * (q[m, k] - zero[m, g]) * channel_scale[k] * x[b, k]

in ptqkit's storage layout (uint8 int8 codes, low-nibble-even int4 packing
with an odd-K zero pad, fp32 [out, ceil(K/G)] scales/zeros, optional AWQ
channel scale), plus the RTN quantize + pack step that produces it. The
public names mirror ptqkit's (src/ptqkit/__init__.py:3-47) for this path; the
compute runs in hand-written CUDA kernels behind the C ABI declared in
include/wq_b200.h (``libwq_b200.so``, loaded by ``_kernels``).

The directory name is not a Python identifier; import it with
``importlib.import_module("weight-quantizer_b200")``.
"""

from .compressed import (
    compressed_state,
    load_compressed,
    load_compressed_layers,
    matrix_nbytes,
    payload_nbytes,
    read_compressed,
    save_compressed,
    state_dict_nbytes,
)
from .convert import iter_targets, quantize_model, weight_out_in
from .gemm import dequant_gemm, kernel_info
from .linear import QuantizedLinear
from .pack import pack_int4, unpack_int4
from .quant import (
    Method,
    QuantConfig,
    QuantizedWeight,
    absolute_error_bound,
    assemble_quantized,
    dequantize_weight,
    element_scales,
    quantize_weight,
)

__version__ = "0.1.0"

__all__ = [
    "Method",
    "QuantConfig",
    "QuantizedLinear",
    "QuantizedWeight",
    "absolute_error_bound",
    "assemble_quantized",
    "compressed_state",
    "dequant_gemm",
    "dequantize_weight",
    "element_scales",
    "iter_targets",
    "kernel_info",
    "load_compressed",
    "load_compressed_layers",
    "matrix_nbytes",
    "pack_int4",
    "payload_nbytes",
    "quantize_model",
    "quantize_weight",
    "read_compressed",
    "save_compressed",
    "state_dict_nbytes",
    "unpack_int4",
    "weight_out_in",
]
