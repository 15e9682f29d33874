"""The C-ABI library on a CPU-only host: it loads, exports every symbol
``include/*.h`` declares, and its host-side logic (argument validation, the
per-shape selector, workspace sizing) behaves.  No compute call is made.
"""

import ctypes
import glob
import os
import re

import pytest

from rotalabs_accel_b200 import _capi, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _capi.load_library()


def _declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        syms |= set(re.findall(r"RLA_API\s+[\w\s\*]+?\b(rla_\w+)\s*\(", text))
    return syms


def test_header_declares_the_abi():
    syms = _declared_symbols()
    assert {"rla_w8a16_gemm", "rla_w8a16_workspace_size", "rla_w8a16_plan", "rla_quantize_per_channel",
            "rla_gather_columns", "rla_launch_count", "rla_get_device_error", "rla_last_error",
            "rla_version"} <= syms
    assert set(_capi.EXPORTED_SYMBOLS) <= syms


def test_library_exports_every_declared_symbol(lib):
    for sym in _declared_symbols():
        assert hasattr(lib, sym), f"{sym} declared in include/ but not exported"
    assert lib.rla_version() == 10000


def test_library_is_sm100a_only():
    # the fatbin holds sm_100a code only (no PTX / other archs): check the build flags
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.NVCC_FLAGS)


def test_invalid_arguments_are_rejected_without_launch(lib):
    n0 = lib.rla_launch_count()
    p = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    # negative size
    assert lib.rla_w8a16_gemm(p, 64, p, 64, p, 1, None, 0, p, 64, -1, 64, 64, None, 0, None) == 1
    # bad scale dtype
    assert lib.rla_w8a16_gemm(p, 64, p, 64, p, 7, None, 0, p, 64, 4, 64, 64, None, 0, None) == 1
    # bias dtype set but NULL bias
    assert lib.rla_w8a16_gemm(p, 64, p, 64, p, 1, None, 1, p, 64, 4, 64, 64, None, 0, None) == 1
    # leading dimension too small
    assert lib.rla_w8a16_gemm(p, 32, p, 64, p, 1, None, 0, p, 64, 4, 64, 64, None, 0, None) == 1
    # misaligned workspace
    assert lib.rla_w8a16_gemm(p, 64, p, 64, p, 1, None, 0, p, 64, 4, 64, 64, ctypes.c_void_p(8), 64, None) == 4
    assert b"workspace" in lib.rla_last_error()
    # empty problems are a no-op success
    assert lib.rla_w8a16_gemm(None, 0, None, 0, p, 1, None, 0, p, 0, 0, 64, 64, None, 0, None) == 0
    assert lib.rla_w8a16_gemm(None, 0, None, 0, p, 1, None, 0, p, 0, 4, 0, 64, None, 0, None) == 0
    assert lib.rla_quantize_per_channel(p, 9, 8, 4, 8, p, 8, p, None) == 1
    assert lib.rla_gather_columns(p, 0, 1, 1, p, 1, None) == 1
    assert lib.rla_launch_count() == n0


def test_selector_rules(lib):
    # decode regime: from M = 9 on, the persistent stream-K kernel on large
    # weights (>= 120 MB, or >= 40 MB when the skinny grid is more than one
    # wave); the skinny kernel otherwise (M <= 8 always).  Without a device the
    # occupancy query falls back to 2 resident CTAs per SM on 148 SMs.
    for M in (1, 4, 8, 16, 32):
        for K, N in ((4096, 4096), (4096, 11008), (11008, 4096), (4096, 14336), (8192, 28672), (28672, 1024)):
            _capi.set_decode_kernel("skinny")
            try:
                sk = _capi.plan(M, N, K)
            finally:
                _capi.set_decode_kernel("auto")
            multi_wave = sk["grid_x"] > 2 * 148
            p = _capi.plan(M, N, K)
            big = 8 < M <= 16 and ((N * K >= 40e6 and multi_wave) or N * K >= 120e6)
            assert (M, K, N, p["kernel_name"]) != (16, 11008, 4096, "stream")
            assert p["kernel_name"] == ("stream" if big else "skinny"), (M, N, K)
            assert p["x_rows"] >= M and p["x_rows"] <= 32
            if p["kernel_name"] == "skinny":
                assert p["grid_x"] * p["w_rows"] >= N
    # narrow column shards with long K get split-K across CTAs; without a
    # workspace the slices add up inside a thread-block cluster (at most 8)
    p = _capi.plan(1, 1024, 28672)
    assert p["kernel_name"] == "skinny" and p["splits"] > 1
    p = _capi.plan(1, 1024, 28672, have_workspace=False)
    assert p["kernel_name"] == "skinny" and 1 < p["splits"] <= 8
    # split-K plans of up to 8 slices need no workspace (cluster exchange)
    lib = _capi.load_library()
    assert _capi.plan(1, 4096, 4096)["splits"] <= 8
    assert lib.rla_w8a16_workspace_size(32, 4096, 960) == 0
    # prefill regime -> tcgen05
    for K, N in ((4096, 12288), (4096, 11008), (11008, 4096)):
        p = _capi.plan(2048, N, K)
        assert p["kernel_name"] == "tcgen05" and p["w_rows"] == 128
        assert p["grid_x"] * 128 >= N and p["grid_y"] * p["x_rows"] >= 2048 and p["threads"] == 320
        assert p["smem"] <= 227 * 1024
    p = _capi.plan(257, 384, 1040)
    assert p["kernel_name"] == "tcgen05" and p["threads"] == 320 and p["grid_y"] * p["x_rows"] >= 257
    # the persistent stream-K decode kernel, when chosen: at most one CTA per SM
    _capi.set_decode_kernel("stream")
    try:
        for M in (1, 8, 16, 32):
            p = _capi.plan(M, 14336, 4096)
            assert p["kernel_name"] == "stream" and p["grid_x"] <= 148 and p["grid_y"] == 1
            assert p["x_rows"] >= M and p["smem"] <= 227 * 1024
            assert lib.rla_w8a16_workspace_size(M, 14336, 4096) == 4096 + p["grid_x"] * 2 * 128 * M * 4
        assert _capi.plan(1, 16, 64)["grid_x"] == 1          # one 128x128 unit -> one CTA
        assert _capi.plan(1, 1024, 28672, have_workspace=False)["kernel_name"] == "skinny"
    finally:
        _capi.set_decode_kernel("auto")
    assert lib.rla_set_decode_kernel(2) == 1                 # only NONE / SKINNY / STREAM
    # unaligned / ragged -> generic; K == 0 -> fill; empty -> none
    assert _capi.plan(4, 64, 64, aligned=False)["kernel_name"] == "generic"
    assert _capi.plan(4, 64, 40)["kernel_name"] == "generic"        # K % 16 != 0 on the skinny path
    assert _capi.plan(4, 64, 0)["kernel_name"] == "fill"
    assert _capi.plan(0, 64, 64)["kernel_name"] == "none"


def test_workspace_size(lib):
    assert lib.rla_w8a16_workspace_size(2048, 4096, 4096) == 0
    # more than 8 slices: fp32 partial sums in the workspace
    p = _capi.plan(1, 256, 28672)
    assert p["splits"] > 8
    need = lib.rla_w8a16_workspace_size(1, 256, 28672)
    assert need >= p["splits"] * 1 * 256 * 4
    assert need % 4 == 0
    # up to 8 slices: a thread-block cluster, no workspace
    assert 1 < _capi.plan(1, 1024, 28672)["splits"] <= 8
    assert lib.rla_w8a16_workspace_size(1, 1024, 28672) == 0


def test_cuda_path_never_falls_back(monkeypatch):
    """If the library cannot be loaded, the CUDA path raises; it never
    computes CUDA tensors another way."""
    monkeypatch.setattr(_capi, "_lib", None)
    with pytest.raises(RuntimeError, match="missing"):
        _capi.load_library("/nonexistent/librla_w8a16.so")


def test_fast_call_bindings_share_the_library():
    """The CPython fast-call module is linked to the same library instance as
    the ctypes bindings: a status and error message set through one are seen
    through the other, and the process maps one copy of the library."""
    lib = _capi.load_library()
    fast = _capi._fast
    assert fast is not None, "rotalabs_accel_b200/_rla_fast is not built"
    assert fast.workspace_size(1, 256, 28672) == lib.rla_w8a16_workspace_size(1, 256, 28672)
    assert fast.workspace_size(2048, 4096, 4096) == 0
    n0 = lib.rla_launch_count()
    # M < 0: invalid argument, reported through the shared error string
    assert fast.gemm(0, 0, 0, 0, 0, 1, 0, 0, 0, 0, -1, 64, 64, 0, 0, 0) == 1
    assert b"M, N, K" in lib.rla_last_error()
    assert fast.gemm_swiglu(0, 0, 0, 0, 0, 0, 0, 7, 0, 0, 0, 0, 0, 4, 64, 64, 0, 0, 0) == 1
    assert b"scale_dtype" in lib.rla_last_error()
    assert lib.rla_launch_count() == n0
    with pytest.raises(TypeError):
        fast.gemm(1, 2, 3)
    maps = open("/proc/self/maps").read()
    paths = {line.split()[-1] for line in maps.splitlines() if line.endswith("librla_w8a16.so")}
    assert len(paths) == 1, paths


def test_allgather_workspace_size():
    """The fused-exchange launch is planned for its own kernel form: for a
    70B shard at M = 16 it takes the stream kernel, whose workspace the
    exchange query reports; sizes are multiples of 4 and 0 for empty shapes."""
    lib = _capi.load_library()
    need = lib.rla_w8a16_allgather_workspace_size(16, 14336, 8192)
    assert need > 4096 and need % 4 == 0
    assert lib.rla_w8a16_allgather_workspace_size(0, 14336, 8192) == 0
    assert lib.rla_w8a16_allgather_workspace_size(-1, 14336, 8192) == 0


def test_torch_library_op_registered():
    """rla::w8a16_gemm is registered with torch (CUDA and Meta kernels over
    the C ABI); its Meta kernel gives shapes and the reference's checks
    without a device."""
    import torch
    from rotalabs_accel_b200 import _capi
    assert _capi.torch_op_loaded()
    meta = dict(device="meta")
    x = torch.empty(5, 96, dtype=torch.float16, **meta)
    w = torch.empty(40, 96, dtype=torch.int8, **meta)
    s = torch.empty(40, dtype=torch.float32, **meta)
    y = torch.ops.rla.w8a16_gemm(x, w, s)
    assert y.shape == (5, 40) and y.dtype == torch.float16 and y.device.type == "meta"
    y = torch.ops.rla.w8a16_gemm(x, w, s.half(), torch.empty(40, dtype=torch.float16, **meta))
    assert y.shape == (5, 40)
    # the same CUDA kernel function, exported for calls without the dispatcher
    # (the per-token path); its checks run before any device work
    assert _capi._torch_op_direct is not None
    import pytest
    with pytest.raises(RuntimeError, match="Weight must be INT8"):
        _capi._torch_op_direct(torch.empty(5, 96, dtype=torch.float16), torch.empty(40, 96), torch.empty(40))
    with pytest.raises(RuntimeError, match="Weight must be INT8"):
        torch.ops.rla.w8a16_gemm(x, w.to(torch.float16), s)
    with pytest.raises(RuntimeError, match="Scale shape mismatch"):
        torch.ops.rla.w8a16_gemm(x, w, torch.empty(39, **meta))
    with pytest.raises(RuntimeError, match="Weight shape mismatch"):
        torch.ops.rla.w8a16_gemm(x, torch.empty(40, 95, dtype=torch.int8, **meta), s)
