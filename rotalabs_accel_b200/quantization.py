"""Symmetric int8 quantization: the reference's quantization API, host side.

Same names, arguments, dtypes and results as rotalabs-accel's
``src/rotalabs_accel/quantization/symmetric.py``:

* ``quantize_symmetric``           (symmetric.py:24-82)
* ``dequantize``                   (symmetric.py:85-123)
* ``quantize_weight_per_channel``  (symmetric.py:126-151)
* ``calculate_quantization_error`` (symmetric.py:154-207)
* ``QuantizedLinear``              (symmetric.py:210-317); its forward is
  rerouted to the sm_100a W8A16 kernel for CUDA tensors.

Quantization is a once-per-layer, off-path step.  On CUDA tensors with int8
per-channel output it runs the library's own quantize kernel
(``rla_quantize_per_channel``), bit-identical to the CPU arithmetic: scale =
absmax/127 in the input's dtype, a zero scale becomes 1, ``round`` half to
even, clamp to [-128, 127].
"""

from __future__ import annotations

from typing import Optional

import torch

QMAX = 127


def quantize_symmetric(tensor: torch.Tensor, bits: int = 8, dim: Optional[int] = None):
    """Symmetric absmax quantization to int8.

    ``scale = max|t| / 127`` (over everything, or over ``dim`` for
    per-channel); a zero scale is replaced by 1; ``q = round(t / scale)``
    (half to even) clamped to [-128, 127].  Returns ``(int8 tensor, float32
    scale)``; a per-channel scale has ``dim`` squeezed away.
    """
    assert bits == 8, f"Only 8-bit quantization supported, got {bits}"
    if dim is None:
        scale = tensor.abs().max() / QMAX
    else:
        scale = tensor.abs().amax(dim=dim, keepdim=True) / QMAX
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = torch.round(tensor / scale).clamp(-128, 127).to(torch.int8)
    scale = scale.float()
    if dim is not None:
        scale = scale.squeeze(dim)
    return q, scale


def dequantize(quantized: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.float16,
               dim: Optional[int] = None) -> torch.Tensor:
    """``quantized.float() * scale`` (per-channel scales broadcast along
    ``dim``: rows for ``dim`` None/0, columns otherwise), cast to ``dtype``."""
    qf = quantized.float()
    if scale.dim() == 1 and quantized.dim() == 2:
        scale = scale.unsqueeze(1) if (dim is None or dim == 0) else scale.unsqueeze(0)
    return (qf * scale).to(dtype)


def quantize_weight_per_channel(weight: torch.Tensor):
    """Per-output-channel int8 quantization of an ``[out, in]`` weight:
    ``(int8 [out, in], float32 [out])``.

    CUDA fp32/fp16/bf16 weights go through the library's quantize kernel;
    CPU weights through the same arithmetic in torch ops."""
    assert weight.dim() == 2, f"Expected 2D weight matrix, got {weight.dim()}D"
    if weight.is_cuda:
        from . import _capi
        return _capi.quantize_per_channel(weight)
    return quantize_symmetric(weight, bits=8, dim=1)


def calculate_quantization_error(original: torch.Tensor, quantized: torch.Tensor, scale: torch.Tensor,
                                 dim: Optional[int] = None) -> dict:
    """Error metrics of a quantization: max / mean absolute error, max
    relative error (%) over values above 10 % of the max, and SNR in dB."""
    restored = dequantize(quantized, scale, dtype=original.dtype, dim=dim)
    diff = (original - restored).float()
    of = original.float()
    max_abs = diff.abs().max().item()
    mean_abs = diff.abs().mean().item()
    significant = of.abs() > of.abs().max() * 0.1
    if significant.any():
        rel = (diff[significant].abs() / of[significant].abs()).max().item() * 100
    else:
        rel = 0.0
    snr = 10 * torch.log10((of ** 2).mean() / ((diff ** 2).mean() + 1e-10)).item()
    return {"max_abs_error": max_abs, "mean_abs_error": mean_abs,
            "relative_error_pct": rel, "snr_db": snr}


class QuantizedLinear(torch.nn.Module):
    """Linear layer with per-output-channel int8 weights.

    State dict: ``weight_int8`` int8 ``[out, in]``, ``weight_scale`` fp32
    ``[out]``, optional ``bias`` (an fp32 Parameter), as in the reference.
    ``_quantized`` is a plain attribute (not saved), so a module restored with
    ``load_state_dict`` must be re-marked (``quantize_weights`` or
    ``mark_quantized()``) before ``forward``, exactly like the reference.

    Forward: on CUDA the sm_100a W8A16 kernel (no full-weight dequantization);
    the result has ``x.dtype`` as the reference's ``F.linear`` would give.  On
    the CPU: the reference arithmetic (dequantize to ``x.dtype``, then
    ``F.linear``).
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight_int8", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("weight_scale", torch.ones(out_features, dtype=torch.float32))
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(out_features))
        else:
            self.register_parameter("bias", None)
        self._quantized = False

    def quantize_weights(self, weight: torch.Tensor) -> None:
        assert weight.shape == (self.out_features, self.in_features)
        q, s = quantize_weight_per_channel(weight)
        self.weight_int8.copy_(q)
        self.weight_scale.copy_(s)
        self._quantized = True

    def mark_quantized(self) -> None:
        """Declare the buffers (e.g. from ``load_state_dict``) quantized."""
        self._quantized = True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self._quantized:
            raise RuntimeError("Weights not quantized. Call quantize_weights() first.")
        if x.is_cuda and self.weight_int8.is_cuda:
            from .gemm import int8_gemm
            y = int8_gemm(x, self.weight_int8, self.weight_scale, self.bias)
            return y if y.dtype == x.dtype else y.to(x.dtype)
        w = dequantize(self.weight_int8, self.weight_scale, dtype=x.dtype, dim=0)
        return torch.nn.functional.linear(x, w, self.bias)

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear) -> "QuantizedLinear":
        has_bias = linear.bias is not None
        # Buffers stay where the constructor put them (the CPU), as in the
        # reference (symmetric.py:306-311); move the module with .cuda().
        m = cls(linear.in_features, linear.out_features, bias=has_bias)
        m.quantize_weights(linear.weight.data)
        if has_bias:
            m.bias.data.copy_(linear.bias.data)
        return m

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, quantized={self._quantized}")
