"""The MLP block on the GPU: rla_w8a16_gemm_swiglu, rla_rmsnorm and the
benchmark's config 3 block (RMSNorm(4096) -> gate/up 4096 -> 11008 with
SwiGLU -> down 11008 -> 4096, M = 8 and 2048).

References are fp32 computations with the reference's rounding points
(gate and up rounded to fp16, SwiGLU in fp32 rounded to fp16); the bar is
the north star's: max |y - ref| <= 1e-2 * max(1, |ref|).  The block is also
checked against the CPU oracle (the reference's CPU composition) at M = 8.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _q(N, K, g):
    from rotalabs_accel_b200 import quantize_weight_per_channel
    return quantize_weight_per_channel(torch.randn(N, K, generator=g, device="cuda") * 0.02)


def _ref_gated(x, wg, sg, wu, su, bg=None, bu=None):
    xf = x.float()
    g = xf @ (wg.float() * sg.float()[:, None]).T
    u = xf @ (wu.float() * su.float()[:, None]).T
    if bg is not None:
        g = g + bg.float()
        u = u + bu.float()
    g16 = g.half().float()
    u16 = u.half().float()
    return torch.nn.functional.silu(g16) * u16


def _check(y, ref, what):
    err = (y.float() - ref).abs()
    bound = 1e-2 * torch.clamp(ref.abs(), min=1.0)
    assert torch.isfinite(y.float()).all(), what
    assert bool((err <= bound).all()), f"{what}: max err {err.max().item():.4g}"


@pytest.mark.parametrize("M,N,K,bias,sdt", [
    (1, 11008, 4096, False, torch.float16),    # skinny, decode
    (8, 11008, 4096, True, torch.float32),
    (16, 352, 4096, False, torch.float16),     # narrow N: split-K partials of gate and up
    (32, 256, 2048, True, torch.float16),
    (3, 100, 128, False, torch.float32),       # ragged N
    (64, 11008, 4096, False, torch.float16),   # tcgen05, 64-token tiles
    (200, 1000, 1024, True, torch.float16),    # tcgen05, ragged M and N
    (2048, 11008, 4096, False, torch.float16), # config 3 prefill shape
    (5, 70, 72, True, torch.float16),          # K % 16 != 0: generic kernel
    (40, 33, 24, False, torch.float32),        # generic, prefill-sized M
])
def test_gated_gemm_parity(cuda_lib, M, N, K, bias, sdt):
    from rotalabs_accel_b200 import _capi, int8_gemm_swiglu
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    wg, sg = _q(N, K, g)
    wu, su = _q(N, K, g)
    sg, su = sg.to(sdt), su.to(sdt)
    bg = bu = None
    if bias:
        bg = (torch.randn(N, generator=g, device="cuda") * 0.1).half()
        bu = (torch.randn(N, generator=g, device="cuda") * 0.1).half()
    n0 = _capi.launch_count()
    y = int8_gemm_swiglu(x, wg, sg, wu, su, bg, bu)
    torch.cuda.synchronize()
    # decode and ragged shapes: one fused launch; prefill: gate and up tcgen05
    # GEMMs into the workspace, then the SwiGLU pass
    prefill = M > 32 and K % 16 == 0
    assert _capi.launch_count() == n0 + (3 if prefill else 1)
    assert y.shape == (M, N) and y.dtype == torch.float16
    _check(y, _ref_gated(x, wg, sg, wu, su, bg, bu), f"M={M} N={N} K={K}")
    # the same arithmetic as two of the library's GEMMs plus an fp32 SwiGLU
    gate = _capi.w8a16_gemm(x, wg, sg, bg)
    up = _capi.w8a16_gemm(x, wu, su, bu)
    # (the split-K partition may differ from the plain GEMM's, so gate / up can
    # differ in the last fp16 bit: the same bar as above, not bit equality)
    two_step = (torch.nn.functional.silu(gate.float()) * up.float()).half()
    _check(y, two_step.float(), f"gated GEMM vs two GEMMs, M={M} N={N} K={K}")
    assert _capi.device_error() == 0


def test_gated_gemm_repeated_calls_share_workspace(cuda_lib):
    """Split-K counters return to zero after every call: shapes of different
    splits run back to back on one workspace."""
    from rotalabs_accel_b200 import _capi
    g = torch.Generator(device="cuda").manual_seed(5)
    # (a prefill call in between: its gate / up buffers share the workspace)
    for (M, N, K) in [(16, 352, 4096), (8, 11008, 4096), (64, 352, 1024), (16, 256, 8192), (1, 352, 4096)] * 2:
        x = torch.randn(M, K, generator=g, device="cuda").half()
        wg, sg = _q(N, K, g)
        wu, su = _q(N, K, g)
        y = _capi.w8a16_gemm_swiglu(x, wg, sg.half(), wu, su.half())
        _check(y, _ref_gated(x, wg, sg.half(), wu, su.half()), f"M={M} N={N} K={K}")
    assert _capi.device_error() == 0


@pytest.mark.parametrize("M,K", [(1, 4096), (8, 4096), (2048, 4096), (3, 96), (5, 4100)])
@pytest.mark.parametrize("wdt", [torch.float32, torch.float16, torch.bfloat16])
def test_rmsnorm_parity(cuda_lib, M, K, wdt):
    from rotalabs_accel_b200 import rmsnorm
    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = (torch.randn(M, K, generator=g, device="cuda") * 2).half()
    x[0, :] = 0                                          # rms of a zero row
    w = (torch.rand(K, generator=g, device="cuda") + 0.5).to(wdt)
    y = rmsnorm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert y.dtype == torch.float16 and y.shape == x.shape
    err = (y.float() - ref).abs()
    assert bool((err <= 2e-3 * ref.abs() + 1e-3).all()), f"max err {err.max().item():.3g}"


def _block(hidden=4096, inter=11008, seed=0):
    import rotalabs_accel_b200 as ra
    g = torch.Generator(device="cuda").manual_seed(seed)
    norm = ra.TritonRMSNorm(hidden).cuda()
    mlp = ra.Int8SwiGLU(hidden, inter).cuda()
    mlp.quantize_weights(torch.randn(inter, hidden, generator=g, device="cuda") * 0.02,
                         torch.randn(inter, hidden, generator=g, device="cuda") * 0.02,
                         torch.randn(hidden, inter, generator=g, device="cuda") * 0.02)
    return norm, mlp


def _ref_block(x, norm, mlp):
    xf = x.float()
    xn = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm.eps) * norm.weight.float()).half()
    h = _ref_gated(xn, mlp.w_gate.weight_int8, mlp.w_gate.scale, mlp.w_up.weight_int8, mlp.w_up.scale).half()
    return h.float() @ (mlp.w_down.weight_int8.float() * mlp.w_down.scale[:, None]).T


@pytest.mark.parametrize("M", [8, 2048])
def test_config3_block(cuda_lib, M):
    from rotalabs_accel_b200 import _capi
    norm, mlp = _block()
    g = torch.Generator(device="cuda").manual_seed(100 + M)
    x = torch.randn(M, 4096, generator=g, device="cuda").half()
    n0 = _capi.launch_count()
    y = mlp(norm(x))
    torch.cuda.synchronize()
    # rmsnorm, gate/up + SwiGLU (one launch in decode, three in prefill), down
    assert _capi.launch_count() == n0 + (3 if M <= 32 else 5)
    assert y.shape == (M, 4096) and y.dtype == torch.float16
    _check(y, _ref_block(x, norm, mlp), f"config 3 block M={M}")


def test_config3_block_matches_cpu_oracle(cuda_lib):
    """Against the reference's CPU composition (the oracle) at M = 8."""
    from oracle import w8a16_oracle as orc
    norm, mlp = _block(seed=1)
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(8, 4096, generator=g, device="cuda").half()
    y = mlp(norm(x)).float().cpu().numpy()
    c = lambda t: t.detach().cpu().numpy()
    ref = orc.swiglu_mlp(c(x), c(norm.weight.half()), norm.eps, c(mlp.w_gate.weight_int8), c(mlp.w_gate.scale),
                         c(mlp.w_up.weight_int8), c(mlp.w_up.scale), c(mlp.w_down.weight_int8),
                         c(mlp.w_down.scale)).astype(np.float32)
    err = np.abs(y - ref)
    assert np.all(err <= 1e-2 * np.maximum(1.0, np.abs(ref))), err.max()
