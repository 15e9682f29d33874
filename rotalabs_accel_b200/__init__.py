"""rotalabs_accel_b200 -- a B200-native (sm_100a) W8A16 GEMM behind
rotalabs-accel's GEMM and quantization API.

Drop-in names (rotalabs-accel ``src/rotalabs_accel/__init__.py:31-104``):
``int8_gemm``, ``int8_gemm_torch``, ``Int8Linear``, ``quantize_symmetric``,
``dequantize``, ``quantize_weight_per_channel``,
``calculate_quantization_error``, ``QuantizedLinear``, ``rmsnorm``,
``rmsnorm_torch``, ``TritonRMSNorm``, ``swiglu_torch`` and the device
helpers; for the MLP block, ``int8_gemm_swiglu`` and ``Int8SwiGLU``
(``rotalabs_accel_b200.mlp``).
CUDA tensors run hand-written sm_100a kernels through the C ABI of
``include/rla_w8a16.h``; the column-parallel multi-GPU layer is in
``rotalabs_accel_b200.sharded``.
"""

from ._version import __version__, __b200_version__
from .gemm import Int8Linear, int8_gemm, int8_gemm_torch
from .mlp import Int8SwiGLU, TritonRMSNorm, int8_gemm_swiglu, rmsnorm, rmsnorm_torch, swiglu_torch
from .quantization import (QuantizedLinear, calculate_quantization_error, dequantize, quantize_symmetric,
                           quantize_weight_per_channel)
from .utils import get_device, get_device_properties, is_cuda_available, is_triton_available

__all__ = [
    "__version__",
    "int8_gemm", "int8_gemm_torch", "Int8Linear",
    "rmsnorm", "rmsnorm_torch", "TritonRMSNorm", "swiglu_torch", "int8_gemm_swiglu", "Int8SwiGLU",
    "quantize_symmetric", "dequantize", "quantize_weight_per_channel", "calculate_quantization_error",
    "QuantizedLinear",
    "get_device", "is_cuda_available", "is_triton_available", "get_device_properties",
]
