"""The W8A16 MLP block: RMSNorm -> gate/up GEMM with SwiGLU -> down GEMM.

rotalabs-accel builds a Llama MLP from separate pieces: ``rmsnorm``
(src/rotalabs_accel/kernels/normalization.py:186-213), two ``Int8Linear``
calls for gate and up (kernels/gemm.py:241-336), ``swiglu_fused``
(kernels/activations.py:109-137) and ``Int8Linear`` down.  On CUDA tensors
this module runs the block in three launches of the sm_100a library:

* ``rmsnorm`` -> ``rla_rmsnorm`` (the arithmetic of the reference's CUDA
  kernel: fp32 mean of squares, ``fp16(x * rsqrt(mean + eps) * w)``);
* ``int8_gemm_swiglu`` -> ``rla_w8a16_gemm_swiglu``: gate and up in one GEMM,
  ``fp16(silu(g) * u)`` in the epilogue from the fp16-rounded gate and up
  values (what ``int8_gemm`` twice plus the reference's CUDA SwiGLU compute,
  without the two ``[M, intermediate]`` tensors);
* down -> ``int8_gemm``.

CPU tensors follow the reference's CPU composition (``rmsnorm_torch``,
``int8_gemm_torch``, ``swiglu_torch``).  Names that exist in the reference
(``rmsnorm``, ``rmsnorm_torch``, ``TritonRMSNorm``, ``swiglu_torch``) keep
its signatures.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _capi
from .gemm import Int8Linear, _as_2d_fp16, int8_gemm


def rmsnorm_torch(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """The reference's PyTorch RMSNorm (normalization.py:32-45):
    ``(x.float() * rsqrt(mean(x^2) + eps)).to(x.dtype) * weight``."""
    x_fp32 = x.float()
    rms = torch.rsqrt(x_fp32.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (x_fp32 * rms).to(x.dtype) * weight


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """RMSNorm over the last dimension (normalization.py:186-213).  CUDA:
    ``rla_rmsnorm`` (fp16 output, the reference's CUDA arithmetic); CPU:
    ``rmsnorm_torch``."""
    assert x.shape[-1] == weight.shape[0], f"Hidden dim mismatch: {x.shape[-1]} vs {weight.shape[0]}"
    if x.is_cuda and weight.is_cuda:
        K = x.shape[-1]
        x2 = _as_2d_fp16(x, K)
        return _capi.rmsnorm(x2, weight, eps).view(*x.shape[:-1], K)
    return rmsnorm_torch(x, weight, eps)


class TritonRMSNorm(torch.nn.Module):
    """RMSNorm layer with the reference's interface (normalization.py:268-297):
    ``weight`` Parameter of ones ``[hidden_size]``, ``eps``."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.hidden_size = hidden_size
        self.eps = eps
        self.weight = torch.nn.Parameter(torch.ones(hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rmsnorm(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{self.hidden_size}, eps={self.eps}"


def swiglu_torch(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """The reference's PyTorch SwiGLU (activations.py:36-46): ``silu(gate) * up``."""
    return torch.nn.functional.silu(gate) * up


def int8_gemm_swiglu(x: torch.Tensor, weight_gate: torch.Tensor, scale_gate: torch.Tensor,
                     weight_up: torch.Tensor, scale_up: torch.Tensor, bias_gate: Optional[torch.Tensor] = None,
                     bias_up: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(int8_gemm(x, gate)) * int8_gemm(x, up)``: one launch on CUDA
    (fp16 output; gate and up rounded to fp16 before the activation, which is
    computed in fp32), the reference's composition on the CPU."""
    assert weight_gate.dtype == torch.int8 and weight_up.dtype == torch.int8, "Weight must be INT8"
    K = x.shape[-1]
    N = weight_gate.shape[0]
    assert weight_gate.shape == (N, K) and weight_up.shape == (N, K), \
        f"Weight shape mismatch: {weight_gate.shape} / {weight_up.shape} vs ({N}, {K})"
    assert scale_gate.shape == (N,) and scale_up.shape == (N,), f"Scale shape mismatch: expected ({N},)"
    if x.is_cuda and weight_gate.is_cuda and weight_up.is_cuda:
        lead = x.shape[:-1]
        x2 = _as_2d_fp16(x, K)
        wg = weight_gate if (N == 0 or weight_gate.stride(1) == 1) else weight_gate.contiguous()
        wu = weight_up if (N == 0 or weight_up.stride(1) == 1) else weight_up.contiguous()
        if wg.stride() != wu.stride():
            wg, wu = wg.contiguous(), wu.contiguous()
        sg = scale_gate.contiguous()
        su = scale_up.to(sg.dtype).contiguous()
        bg = bu = None
        if bias_gate is not None or bias_up is not None:
            bdt = torch.float32 if (bias_gate is not None and bias_gate.dtype == torch.float32) else torch.float16
            bg = (bias_gate if bias_gate is not None else torch.zeros(N, device=x.device)).to(bdt).contiguous()
            bu = (bias_up if bias_up is not None else torch.zeros(N, device=x.device)).to(bdt).contiguous()
        y = _capi.w8a16_gemm_swiglu(x2, wg, sg, wu, su, bg, bu)
        return y.view(*lead, N)
    gate = int8_gemm(x, weight_gate, scale_gate, bias_gate)
    up = int8_gemm(x, weight_up, scale_up, bias_up)
    return swiglu_torch(gate, up)


class Int8SwiGLU(torch.nn.Module):
    """The reference's ``SwiGLU`` FFN (activations.py:140-181) with W8A16
    projections: ``w_gate``, ``w_up`` (hidden -> intermediate) and ``w_down``
    (intermediate -> hidden) are ``Int8Linear`` layers with the reference's
    buffers.  ``forward(x) = w_down(silu(w_gate(x)) * w_up(x))``; on CUDA the
    gate/up pair is one fused launch (``int8_gemm_swiglu``)."""

    def __init__(self, hidden_size: int, intermediate_size: int, bias: bool = False):
        super().__init__()
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.w_gate = Int8Linear(hidden_size, intermediate_size, bias=bias)
        self.w_up = Int8Linear(hidden_size, intermediate_size, bias=bias)
        self.w_down = Int8Linear(intermediate_size, hidden_size, bias=bias)

    def quantize_weights(self, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> None:
        """Quantize float ``[out, in]`` weights of the three projections."""
        self.w_gate.quantize_weights(w_gate)
        self.w_up.quantize_weights(w_up)
        self.w_down.quantize_weights(w_down)

    @classmethod
    def from_swiglu(cls, module: torch.nn.Module) -> "Int8SwiGLU":
        """Quantize a module with ``torch.nn.Linear`` attributes ``w_gate``,
        ``w_up``, ``w_down`` (the reference's ``SwiGLU``)."""
        has_bias = module.w_gate.bias is not None
        m = cls(module.w_gate.in_features, module.w_gate.out_features, bias=has_bias)
        m = m.to(module.w_gate.weight.device)
        m.quantize_weights(module.w_gate.weight.data, module.w_up.weight.data, module.w_down.weight.data)
        if has_bias:
            for name in ("w_gate", "w_up", "w_down"):
                getattr(m, name).bias.data.copy_(getattr(module, name).bias.data.half())
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for lin in (self.w_gate, self.w_up, self.w_down):
            if not lin._quantized:
                raise RuntimeError("Weights not quantized. Call quantize_weights() first.")
        h = int8_gemm_swiglu(x, self.w_gate.weight_int8, self.w_gate.scale, self.w_up.weight_int8, self.w_up.scale,
                             self.w_gate.bias, self.w_up.bias)
        return self.w_down(h)

    def extra_repr(self) -> str:
        return f"hidden_size={self.hidden_size}, intermediate_size={self.intermediate_size}"
