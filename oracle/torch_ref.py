"""rotalabs-accel's CPU route for the W8A16 GEMM, restated with torch ops
(TEST INFRASTRUCTURE, never shipped).

This is the path the reference's ``int8_gemm`` takes for every non-CUDA
tensor (src/rotalabs_accel/kernels/gemm.py:234-238): dequantize the whole
int8 weight to the activation dtype, then ``F.linear``.  It exists here for
one job: the CPU baseline of ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm), which times the reference's own CPU algorithm on
the host's cores with torch's own threading.  ``oracle/w8a16_oracle.py``
(numpy) remains the checker of the tests; ``tests/test_oracle_golden.py``
pins both against the vectors the reference itself produced.

* ``dequantize``       <- src/rotalabs_accel/quantization/symmetric.py:85-123
  (``q.float() * scale[:, None]`` for per-output-channel scales, then one
  rounding to the requested dtype)
* ``int8_gemm_torch``  <- src/rotalabs_accel/kernels/gemm.py:31-48
  (``F.linear(x, dequantize(w, s, x.dtype, dim=0), bias)``)

The arithmetic is torch's (``torch>=2.0.0``, unpinned in the reference's
pyproject.toml:42; the golden vectors were made with 2.11.0).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F


def dequantize(quantized: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.float16,
               dim: Optional[int] = None) -> torch.Tensor:
    """int8 -> float32, times the scale broadcast along ``dim`` (per output
    channel for dim 0 or None, per input channel for dim 1 of a 2-D weight),
    rounded once to ``dtype`` (symmetric.py:85-123)."""
    s = scale
    if s.dim() == 1 and quantized.dim() == 2:
        s = s.unsqueeze(0) if dim not in (None, 0) else s.unsqueeze(1)
    return (quantized.to(torch.float32) * s).to(dtype)


def int8_gemm_torch(x: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
                    bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The reference's CPU W8A16 GEMM (gemm.py:31-48): the weight is
    dequantized to ``x.dtype`` (so fp16 activations meet an fp16 weight),
    then ``F.linear``."""
    return F.linear(x, dequantize(weight_int8, scale, dtype=x.dtype, dim=0), bias)
