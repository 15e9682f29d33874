"""CPU oracle for the W8A16 GEMM path (TEST INFRASTRUCTURE, never shipped).

This module is the checker, not the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm
may import it.  The product path (``rotalabs_accel_b200``) never imports it
and never computes a CUDA tensor on the CPU.

It restates, in numpy, the arithmetic of rotalabs-accel's CPU path for the
W8A16 GEMM, step by step:

* ``quantize_symmetric``          <- src/rotalabs_accel/quantization/symmetric.py:24-82
* ``dequantize``                  <- src/rotalabs_accel/quantization/symmetric.py:85-123
* ``quantize_weight_per_channel`` <- src/rotalabs_accel/quantization/symmetric.py:126-151
* ``calculate_quantization_error``<- src/rotalabs_accel/quantization/symmetric.py:154-207
* ``int8_gemm_torch``             <- src/rotalabs_accel/kernels/gemm.py:31-48
  (the reference's ``int8_gemm`` routes every non-CUDA call here,
  src/rotalabs_accel/kernels/gemm.py:234-238)
* ``rmsnorm_torch``               <- src/rotalabs_accel/kernels/normalization.py:32-45
* ``swiglu_torch``                <- src/rotalabs_accel/kernels/activations.py:36-46
* ``swiglu_mlp``                  <- the MLP block of the benchmark's config 3 as
  the reference composes it on the CPU: rmsnorm -> int8_gemm gate, up ->
  swiglu -> int8_gemm down (kernels/activations.py:175-178 with Int8Linear)

The reference's arithmetic lives in its third-party dependency torch
(``torch>=2.0.0``, pyproject.toml:42, unpinned; 2.11.0 was used to make the
golden vectors): ``amax``, true division, ``torch.round`` (round half to
even), ``clamp``, and ``F.linear`` (fp32 accumulation with one rounding to the
output dtype on the CPU).  numpy gives the same IEEE results for the
element-wise steps, so quantization is bit-exact; the matmul is fp32
accumulation followed by one rounding, so the GEMM output agrees with
the reference's to within an fp16 ulp (summation order differs).

Parity pin: ``tests/golden/*.npz`` were produced by running the reference
itself (``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py``
checks this module against every one of them.
"""

from __future__ import annotations

import numpy as np

QMAX = 127


def quantize_symmetric(tensor: np.ndarray, bits: int = 8, dim: int | None = None):
    """Symmetric absmax/127 quantization (symmetric.py:24-82).

    The scale is computed in the input's own dtype (an fp16 weight gets an
    fp16 scale before the final ``.float()``, symmetric.py:62-76), a zero
    scale becomes 1 (symmetric.py:70), values are ``round(t / scale)`` with
    round-half-even, clamped to [-128, 127] and cast to int8 (symmetric.py:73).
    Returns ``(int8 array, float32 scale)``; per-channel scales are squeezed.
    """
    assert bits == 8, f"Only 8-bit quantization supported, got {bits}"
    t = np.asarray(tensor)
    qmax = np.asarray(QMAX, dtype=t.dtype)
    if dim is None:
        max_val = np.abs(t).max()
        scale = np.asarray(max_val / qmax, dtype=t.dtype)
    else:
        max_val = np.abs(t).max(axis=dim, keepdims=True)
        scale = (max_val / qmax).astype(t.dtype)
    scale = np.where(scale == 0, np.ones_like(scale), scale).astype(t.dtype)
    q = np.clip(np.round(t / scale), -128, 127).astype(np.int8)
    scale = scale.astype(np.float32)
    if dim is not None:
        scale = np.squeeze(scale, axis=dim)
    return q, scale


def dequantize(quantized: np.ndarray, scale: np.ndarray, dtype=np.float16, dim: int | None = None):
    """``quantized.float() * scale`` broadcast per channel, cast to ``dtype``
    (symmetric.py:85-123).  numpy's float32*float16 promotes to float32 just
    as torch's does, so an fp16 scale multiplies in fp32."""
    qf = np.asarray(quantized).astype(np.float32)
    s = np.asarray(scale)
    if s.ndim == 1 and qf.ndim == 2:
        s = s[:, None] if (dim is None or dim == 0) else s[None, :]
    out = qf * s
    return out.astype(dtype)


def quantize_weight_per_channel(weight: np.ndarray):
    """Per-output-channel (row) quantization (symmetric.py:126-151)."""
    w = np.asarray(weight)
    assert w.ndim == 2, f"Expected 2D weight matrix, got {w.ndim}D"
    return quantize_symmetric(w, bits=8, dim=1)


def calculate_quantization_error(original, quantized, scale, dim=None):
    """Error metrics dict (symmetric.py:154-207)."""
    orig = np.asarray(original)
    restored = dequantize(quantized, scale, dtype=orig.dtype, dim=dim)
    diff = (orig - restored).astype(np.float32)
    of = orig.astype(np.float32)
    max_abs = float(np.abs(diff).max())
    mean_abs = float(np.abs(diff).mean())
    thr = np.abs(of).max() * np.float32(0.1)
    mask = np.abs(of) > thr
    rel = float((np.abs(diff[mask]) / np.abs(of[mask])).max() * 100) if mask.any() else 0.0
    sig = np.float32((of ** 2).mean())
    noise = np.float32((diff ** 2).mean())
    snr = float(10 * np.log10(sig / (noise + np.float32(1e-10))))
    return {"max_abs_error": max_abs, "mean_abs_error": mean_abs,
            "relative_error_pct": rel, "snr_db": snr}


def int8_gemm_torch(x: np.ndarray, weight_int8: np.ndarray, scale: np.ndarray, bias=None):
    """The reference's CPU W8A16 GEMM (gemm.py:31-48): dequantize the whole
    weight to ``x.dtype`` first (gemm.py:43), then ``linear`` (gemm.py:46),
    which on the CPU accumulates in fp32 and rounds once to ``x.dtype``.
    ``x`` is ``(..., K)``; the result is ``(..., N)`` in ``x.dtype``."""
    x = np.asarray(x)
    w_deq = dequantize(weight_int8, scale, dtype=x.dtype, dim=0)
    K = x.shape[-1]
    x2 = x.reshape(-1, K).astype(np.float32)
    acc = x2 @ w_deq.astype(np.float32).T
    if bias is not None:
        acc = acc + np.asarray(bias).astype(np.float32)
    return acc.astype(x.dtype).reshape(x.shape[:-1] + (weight_int8.shape[0],))


def int8_gemm(x, weight_int8, scale, bias=None, weight_transposed=None, scale_fp16=None, use_cublas=None):
    """Shape/dtype validation of the reference dispatcher (gemm.py:223-231),
    then its CPU route (gemm.py:238)."""
    assert weight_int8.dtype == np.int8, "Weight must be INT8"
    K = x.shape[-1]
    N = weight_int8.shape[0]
    assert weight_int8.shape == (N, K), f"Weight shape mismatch: {weight_int8.shape} vs ({N}, {K})"
    assert scale.shape == (N,), f"Scale shape mismatch: {scale.shape} vs ({N},)"
    return int8_gemm_torch(x, weight_int8, scale, bias)


def dequant_matmul_fp32(x, weight_int8, scale, bias=None):
    """The tolerance reference of the north star: fp32-accumulated
    dequant-matmul, ``x.float() @ (w.float() * s.float()[:, None]).T (+ bias)``,
    returned in float32 (no output rounding)."""
    x = np.asarray(x).astype(np.float32)
    w = np.asarray(weight_int8).astype(np.float32) * np.asarray(scale).astype(np.float32)[:, None]
    K = x.shape[-1]
    y = x.reshape(-1, K) @ w.T
    if bias is not None:
        y = y + np.asarray(bias).astype(np.float32)
    return y.reshape(x.shape[:-1] + (w.shape[0],))


def rmsnorm_torch(x, weight, eps: float = 1e-6):
    """The reference's CPU RMSNorm (normalization.py:32-45): in fp32,
    ``rms = 1 / sqrt(mean(x^2) + eps)``; ``(x * rms)`` rounded to ``x.dtype``,
    then times ``weight`` with the usual dtype promotion."""
    x = np.asarray(x)
    x32 = x.astype(np.float32)
    rms = (np.float32(1.0) / np.sqrt((x32 * x32).mean(axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps)))
    return (x32 * rms).astype(x.dtype) * np.asarray(weight)


def swiglu_torch(gate, up):
    """The reference's CPU SwiGLU (activations.py:36-46): ``silu(gate) * up``;
    for fp16 tensors ``silu`` is computed in fp32 and rounded to fp16, then
    the product is rounded to fp16."""
    gate = np.asarray(gate)
    g32 = gate.astype(np.float32)
    silu = (g32 / (np.float32(1.0) + np.exp(-g32))).astype(gate.dtype)
    return silu * np.asarray(up)


def swiglu_mlp(x, norm_weight, eps, wg, sg, wu, su, wd, sd):
    """RMSNorm -> gate / up W8A16 GEMMs -> SwiGLU -> down W8A16 GEMM, each
    step with the reference's CPU arithmetic."""
    xn = rmsnorm_torch(x, norm_weight, eps)
    gate = int8_gemm_torch(xn, wg, sg)
    up = int8_gemm_torch(xn, wu, su)
    return int8_gemm_torch(swiglu_torch(gate, up), wd, sd)
