"""The allocation-free decode entry point, ``rla_w8a16_gemm_noalloc``.

It serves callers that cannot allocate GPU memory where the GEMM runs (a
serving loop that must not let cudaMalloc synchronise the device, a process
whose memory is reserved up front, a plugin callback that gets no
workspace): its split-K scratch is a static 1 MiB device array instead of a
caller workspace.  This test calls it through the C ABI and checks its output
against ``rla_w8a16_gemm`` (the workspace entry point) on two calls in a row,
within the tolerance the other GPU tests use, and checks a short-K shape whose
slices add up inside a thread-block cluster (no scratch at all).

The file is named so that pytest collects it last; it also passes alone in a
fresh process.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2
F16, F32, NONE = 1, 2, 0


def _lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from rotalabs_accel_b200 import _capi, build
    build.build()
    lib = _capi.load_library()
    i64, p = ctypes.c_int64, ctypes.c_void_p
    f = lib.rla_w8a16_gemm_noalloc
    f.argtypes = [p, i64, p, i64, p, ctypes.c_int, p, ctypes.c_int, p, i64, i64, i64, i64, p]
    f.restype = ctypes.c_int
    return lib


def _problem(M, N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev).half()
    from rotalabs_accel_b200 import quantize_weight_per_channel
    q, s = quantize_weight_per_channel(torch.randn(N, K, generator=g, device=dev) * 0.02)
    b = (torch.randn(N, generator=g, device=dev) * 0.1).half()
    return x, q, s.half(), b


def _with_workspace(lib, x, q, s, b, stream):
    M, K = x.shape
    N = q.shape[0]
    y = torch.empty(M, N, dtype=torch.float16, device=x.device)
    need = lib.rla_w8a16_workspace_size(M, N, K)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=x.device)
    st = lib.rla_w8a16_gemm(x.data_ptr(), K, q.data_ptr(), K, s.data_ptr(), F16, b.data_ptr(), F16,
                            y.data_ptr(), N, M, N, K, ws.data_ptr(), ws.numel(), stream)
    assert st == 0, lib.rla_last_error()
    return y


def _no_alloc(lib, x, q, s, b, stream):
    M, K = x.shape
    N = q.shape[0]
    y = torch.full((M, N), float("nan"), dtype=torch.float16, device=x.device)
    st = lib.rla_w8a16_gemm_noalloc(x.data_ptr(), K, q.data_ptr(), K, s.data_ptr(), F16, b.data_ptr(), F16,
                                    y.data_ptr(), N, M, N, K, stream)
    assert st == 0, lib.rla_last_error()
    return y


def test_no_alloc_matches_workspace_entry_point():
    lib = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    # split-K plans of several shapes and one without split-K; the first
    # needs more than 8 K slices, so its partial sums really go through the
    # static scratch (not through a thread-block cluster)
    from rotalabs_accel_b200 import _capi
    assert lib.rla_w8a16_workspace_size(8, 1024, 28672) > 0
    assert _capi.plan(8, 1024, 28672)["splits"] > 8
    for i, (M, N, K) in enumerate([(8, 1024, 28672), (16, 1024, 4096), (1, 512, 8192), (4, 14336, 4096)]):
        x, q, s, b = _problem(M, N, K, 100 + i, dev)
        y_ws = _with_workspace(lib, x, q, s, b, stream)
        ref = x.float() @ (q.float() * s.float()[:, None]).t() + b.float()
        for _ in range(2):                              # two calls in a row share the array
            y = _no_alloc(lib, x, q, s, b, stream)
            torch.cuda.synchronize()
            assert torch.isfinite(y).all()
            assert (y.float() - y_ws.float()).abs().max().item() <= TOL
            assert (y.float() - ref).abs().max().item() <= TOL + 2.0 ** -10 * ref.abs().max().item()


def test_no_alloc_short_k_cluster_split():
    """A short-K layer whose split-K plan would need 1.5 MiB + 4 KiB of
    workspace partial sums (3 slices of 32 x 4096 fp32) adds its slices
    inside a thread-block cluster instead: it needs no scratch and runs."""
    lib = _lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    M, N, K = 32, 4096, 960
    assert lib.rla_w8a16_workspace_size(M, N, K) == 0
    x, q, s, b = _problem(M, N, K, 7, dev)
    n0 = lib.rla_launch_count()
    y = _no_alloc(lib, x, q, s, b, stream)
    torch.cuda.synchronize()
    assert lib.rla_launch_count() == n0 + 1
    ref = x.float() @ (q.float() * s.float()[:, None]).t() + b.float()
    assert (y.float() - ref).abs().max().item() <= TOL + 2.0 ** -10 * ref.abs().max().item()
