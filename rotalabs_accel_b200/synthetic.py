"""Seeded synthetic W8A16 workloads (the shapes and value distributions of the
benchmark configurations; no dataset is involved).

Every workload is drawn from a ``torch.Generator`` seeded explicitly, so the
same seed gives the same bytes on any machine with the same torch build:

* ``x  ~ N(0, 1)`` cast to fp16, shape ``[M, K]``;
* ``W ~ N(0, 0.02)`` fp32, shape ``[N, K]``, quantized per output channel
  (absmax/127, round half to even, clamp) into int8 ``[N, K]`` plus a scale
  ``[N]`` (fp32, or cast to fp16 as in the decode/prefill configurations).

The CPU generator is used for anything a CPU oracle must reproduce; the
device generator (``device="cuda"``) is used for large benchmark layers where
only size-independent properties are checked.
"""

from __future__ import annotations

import torch

from .quantization import quantize_weight_per_channel

# Shapes of the reference configurations.
CONFIG0 = dict(M=32, K=4096, N=4096)
DECODE_MS = (1, 4, 8, 16)
DECODE_KN = ((4096, 4096), (4096, 11008), (11008, 4096), (4096, 14336))
PREFILL_M = 2048
PREFILL_KN = ((4096, 12288), (4096, 11008), (11008, 4096))
LLAMA70B_KN = ((8192, 28672), (28672, 8192))
LLAMA70B_MS = (1, 16, 4096)


def make_x(M: int, K: int, seed: int = 0, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(M, K, generator=g, device=device).half()


def make_weight(N: int, K: int, seed: int = 0, device="cpu", scale_dtype=torch.float16):
    """int8 ``[N, K]`` weight and ``[N]`` scale from ``N(0, 0.02)`` fp32."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = torch.randn(N, K, generator=g, device=device) * 0.02
    q, s = quantize_weight_per_channel(w)
    return q, s.to(scale_dtype)


def make_problem(M: int, N: int, K: int, seed: int = 0, device="cpu", scale_dtype=torch.float16):
    """``(x fp16 [M,K], w int8 [N,K], scale [N])`` drawn from one generator:
    x first, then the fp32 weight (the order the golden vectors use)."""
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=device).half()
    w = torch.randn(N, K, generator=g, device=device) * 0.02
    q, s = quantize_weight_per_channel(w)
    return x, q, s.to(scale_dtype)
