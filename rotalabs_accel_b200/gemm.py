"""W8A16 GEMM: the reference's GEMM API, routed to sm_100a CUDA kernels.

Same names, signatures, shape rules and error conventions as rotalabs-accel's
``src/rotalabs_accel/kernels/gemm.py``:

* ``int8_gemm(x, weight_int8, scale, bias=None, weight_transposed=None,
  scale_fp16=None, use_cublas=None)``   (gemm.py:189-238)
* ``int8_gemm_torch(x, weight_int8, scale, bias=None)``   (gemm.py:31-48)
* ``Int8Linear``                                          (gemm.py:241-336)

Routing.  CUDA tensors always go to the C-ABI library (``rla_w8a16_gemm``:
a per-shape selector picking the decode kernel or the tcgen05 prefill
kernel); if that library cannot be loaded the call raises.  There is no
Triton path and no silent CPU fallback for CUDA tensors.  CPU tensors keep
the reference's documented CPU behaviour: ``int8_gemm_torch`` (dequantize to
``x.dtype``, then ``F.linear``), exactly as the reference dispatcher does for
non-CUDA inputs (gemm.py:234-238).

Numerics on the GPU: fp32 accumulation of ``x * q`` over k, then
``fp16(acc * scale[n] + bias[n])`` in one rounding (the reference Triton
kernel rounds ``acc * scale`` to fp16 and adds the bias in a second fp16
op, gemm.py:133-138 and :180-182).  The output is fp16 whatever ``x.dtype``
is, as on the reference's GPU path (gemm.py:162); fp32 / bf16 activations
are cast to fp16 first.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _capi
from .quantization import dequantize, quantize_weight_per_channel


def int8_gemm_torch(x: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
                    bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The reference's PyTorch W8A16 GEMM: dequantize the full weight to
    ``x.dtype``, then ``F.linear``.  Any device; used by ``int8_gemm`` for
    CPU tensors only."""
    w = dequantize(weight_int8, scale, dtype=x.dtype, dim=0)
    return torch.nn.functional.linear(x, w, bias)


def _as_2d_fp16(x: torch.Tensor, K: int) -> torch.Tensor:
    rows = 1
    for d in x.shape[:-1]:
        rows *= d
    x2 = x.reshape(rows, K)
    if x2.dtype != torch.float16:
        x2 = x2.to(torch.float16)
    if x2.shape[0] > 0 and x2.stride(1) != 1:
        x2 = x2.contiguous()
    return x2


def int8_gemm(x: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
              bias: Optional[torch.Tensor] = None, weight_transposed: Optional[torch.Tensor] = None,
              scale_fp16: Optional[torch.Tensor] = None, use_cublas: Optional[bool] = None) -> torch.Tensor:
    """W8A16 GEMM ``y = x @ (weight_int8 * scale).T + bias``.

    Args (as in the reference):
        x: activations ``(..., K)`` (fp16 on the GPU path).
        weight_int8: int8 ``(N, K)``.
        scale: ``(N,)`` fp32 or fp16 per-output-channel scale.
        bias: optional ``(N,)`` (fp16 or fp32).
        weight_transposed: accepted for compatibility; the sm_100a kernels
            read ``weight_int8`` ``[N, K]`` directly and never need it.
        scale_fp16, use_cublas: accepted and ignored, as in the reference.

    Returns ``(..., N)``: fp16 for CUDA inputs, ``x.dtype`` for CPU inputs.
    """
    assert weight_int8.dtype == torch.int8, "Weight must be INT8"
    K = x.shape[-1]
    N = weight_int8.shape[0]
    assert weight_int8.shape == (N, K), f"Weight shape mismatch: {weight_int8.shape} vs ({N}, {K})"
    assert scale.shape == (N,), f"Scale shape mismatch: {scale.shape} vs ({N},)"

    if x.is_cuda and weight_int8.is_cuda and scale.is_cuda:
        # (a 2-D fp16 x with unit inner stride, the per-token case, is used as is)
        plain = x.dim() == 2 and x.dtype == torch.float16 and (x.shape[0] == 0 or x.stride(1) == 1)
        op = _capi._torch_op_direct
        if (plain and op is not None and weight_int8.stride(1) == 1 and scale.is_contiguous()
                and (bias is None or (bias.dtype in (torch.float16, torch.float32) and bias.is_contiguous()))):
            return op(x, weight_int8, scale, bias)
        x2 = x if plain else _as_2d_fp16(x, K)
        w = weight_int8 if (N == 0 or weight_int8.stride(1) == 1) else weight_int8.contiguous()
        s = scale if scale.is_contiguous() else scale.contiguous()
        b = None
        if bias is not None:
            b = bias if bias.dtype in (torch.float16, torch.float32) else bias.to(torch.float16)
            b = b.contiguous()
        y = _capi.w8a16_gemm(x2, w, s, b)
        return y if plain else y.view(*x.shape[:-1], N)

    return int8_gemm_torch(x, weight_int8, scale, bias)


class Int8Linear(torch.nn.Module):
    """Linear layer with int8 weights and per-output-channel scales.

    State dict (the reference's layout, byte-compatible,
    src/rotalabs_accel/kernels/gemm.py:266-286): ``weight_int8`` int8
    ``[out, in]``, ``scale`` fp32 ``[out]``, ``weight_transposed`` int8
    ``[in, out]`` and an optional fp16 ``bias`` Parameter, in that order
    after the bias.

    Only ``weight_int8`` and ``scale`` (and ``bias``) live on the device.  The
    reference keeps a second, transposed copy of every weight for its Triton
    path (gemm.py:276-281, :302); the sm_100a kernels read ``weight_int8``
    directly, so here ``weight_transposed`` is a transposed *view* of
    ``weight_int8`` (no extra memory), materialized as a contiguous ``[in,
    out]`` tensor only when the state dict is saved, and checked against
    ``weight_int8`` (not stored) when one is loaded.

    ``_quantized`` is a plain attribute, not saved: a module restored with
    ``load_state_dict`` must be re-marked (``quantize_weights`` or
    ``mark_quantized()``) before ``forward``, as in the reference.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight_int8", torch.zeros(out_features, in_features, dtype=torch.int8))
        self.register_buffer("scale", torch.ones(out_features, dtype=torch.float32))
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(out_features, dtype=torch.float16))
        else:
            self.register_parameter("bias", None)
        self._quantized = False

    @property
    def weight_transposed(self) -> torch.Tensor:
        """``weight_int8`` as ``[in, out]``: a view, not a copy."""
        return self.weight_int8.t()

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        wt = self.weight_int8.t().contiguous()
        destination[prefix + "weight_transposed"] = wt if keep_vars else wt.detach()

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        key = prefix + "weight_transposed"
        wt = state_dict.get(key)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)
        if key in unexpected_keys:
            unexpected_keys.remove(key)
        if wt is None:
            if strict:
                missing_keys.append(key)
        elif tuple(wt.shape) != (self.in_features, self.out_features) or wt.dtype != torch.int8:
            error_msgs.append(f"size mismatch for {key}: copying a param with shape {tuple(wt.shape)} "
                              f"({wt.dtype}), expected ({self.in_features}, {self.out_features}) int8")
        elif prefix + "weight_int8" in state_dict and not torch.equal(
                wt.to(state_dict[prefix + "weight_int8"].device).t(), state_dict[prefix + "weight_int8"]):
            error_msgs.append(f"{key} is not the transpose of {prefix}weight_int8")

    def quantize_weights(self, weight: torch.Tensor) -> None:
        """Quantize an ``[out, in]`` float weight into the int8 buffers.

        Bit-identical to the reference, which quantizes on the CPU
        (gemm.py:295-296); a CUDA weight is quantized on its device by the
        library's quantize kernel with the same arithmetic."""
        assert weight.shape == (self.out_features, self.in_features)
        q, s = quantize_weight_per_channel(weight)
        device = self.weight_int8.device
        self.weight_int8.copy_(q.to(device))
        self.scale.copy_(s.to(device))
        self._quantized = True

    def mark_quantized(self) -> None:
        """Declare the buffers (e.g. from ``load_state_dict``) quantized."""
        self._quantized = True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self._quantized:
            raise RuntimeError("Weights not quantized. Call quantize_weights() first.")
        # (the buffer and parameter dicts directly: nn.Module attribute lookup
        # costs host time on every decode call)
        b = self._buffers
        w, s, bias = b["weight_int8"], b["scale"], self._parameters["bias"]
        op = _capi._torch_op_direct
        # Per-token fast path straight to the library's op (its CUDA kernel
        # function, without the dispatcher): a 2-D fp16 CUDA x of this
        # layer's width with unit inner stride, contiguous buffers.  Anything
        # else takes int8_gemm's checks and conversions.
        if (op is not None and x.is_cuda and x.dim() == 2 and x.dtype == torch.float16
                and x.shape[1] == self.in_features and x.stride(1) == 1 and w.is_cuda and w.is_contiguous()
                and s.is_contiguous() and (bias is None or (bias.dtype == torch.float16 and bias.is_contiguous()))):
            return op(x, w, s, bias)
        return int8_gemm(x, w, s, bias)

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear) -> "Int8Linear":
        has_bias = linear.bias is not None
        m = cls(linear.in_features, linear.out_features, bias=has_bias)
        m = m.to(linear.weight.device)
        m.quantize_weights(linear.weight.data)
        if has_bias:
            m.bias.data.copy_(linear.bias.data.half())
        return m

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, quantized={self._quantized}")
