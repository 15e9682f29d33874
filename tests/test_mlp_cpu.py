"""The MLP block's pieces on CPU only: oracle and package against the golden
vectors made by rotalabs-accel itself (``tests/golden/ref_mlp.npz``:
``rmsnorm_torch``, ``swiglu_torch`` and the RMSNorm -> gate/up -> SwiGLU ->
down block through the reference's CPU path), and the C ABI's argument
checks for the gated GEMM and RMSNorm (nothing is launched).
"""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import w8a16_oracle as orc


@pytest.fixture(scope="module")
def mlp(golden_dir):
    return np.load(os.path.join(golden_dir, "ref_mlp.npz"))


def test_oracle_rmsnorm_bit_exact(mlp):
    xn = orc.rmsnorm_torch(mlp["x"], mlp["norm_weight"], float(mlp["eps"]))
    assert xn.dtype == np.float16 and np.array_equal(xn, mlp["xn"])
    yr = orc.rmsnorm_torch(mlp["rms_x"], mlp["rms_w"], 1e-5)
    assert yr.dtype == np.float32 and np.array_equal(yr, mlp["rms_y"])   # fp32 weight promotes


def test_oracle_swiglu_bit_exact(mlp):
    assert np.array_equal(orc.swiglu_torch(mlp["swiglu_gate"], mlp["swiglu_up"]), mlp["swiglu_out"])
    assert np.array_equal(orc.swiglu_torch(mlp["gate"], mlp["up"]), mlp["h"])


def test_oracle_block_matches_reference(mlp):
    y = orc.swiglu_mlp(mlp["x"], mlp["norm_weight"], float(mlp["eps"]), mlp["wg"], mlp["sg"], mlp["wu"],
                       mlp["su"], mlp["wd"], mlp["sd"])
    ref = mlp["y"].astype(np.float32)
    # fp32 accumulation in both, different summation order: within an fp16 ulp
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(y.astype(np.float32) - ref) <= ulp + 1e-6)


def test_oracle_catches_a_planted_error(mlp):
    bad = mlp["gate"].copy()
    bad[2, 5] = np.float16(float(bad[2, 5]) + 0.5)
    assert not np.array_equal(orc.swiglu_torch(bad, mlp["up"]), mlp["h"])


def test_package_cpu_path_matches_reference(mlp):
    import rotalabs_accel_b200 as ra
    x = torch.from_numpy(mlp["x"])
    nw = torch.from_numpy(mlp["norm_weight"])
    xn = ra.rmsnorm(x, nw, float(mlp["eps"]))
    assert torch.equal(xn, torch.from_numpy(mlp["xn"]))
    h = ra.int8_gemm_swiglu(xn, torch.from_numpy(mlp["wg"]), torch.from_numpy(mlp["sg"]),
                            torch.from_numpy(mlp["wu"]), torch.from_numpy(mlp["su"]))
    assert torch.equal(h, torch.from_numpy(mlp["h"]))
    H, I = mlp["wg"].shape[1], mlp["wg"].shape[0]
    m = ra.Int8SwiGLU(H, I)
    for name, w, s in (("w_gate", "wg", "sg"), ("w_up", "wu", "su"), ("w_down", "wd", "sd")):
        lin = getattr(m, name)
        lin.weight_int8.copy_(torch.from_numpy(mlp[w]))
        lin.scale.copy_(torch.from_numpy(mlp[s]).float())
        lin.mark_quantized()
    y = m(xn)
    assert torch.allclose(y.float(), torch.from_numpy(mlp["y"]).float(), atol=2e-3, rtol=0)


def test_module_surface():
    import rotalabs_accel_b200 as ra
    norm = ra.TritonRMSNorm(64, eps=1e-5)
    assert norm.weight.shape == (64,) and norm.weight.dtype == torch.float32 and norm.eps == 1e-5
    assert "64, eps=1e-05" in repr(norm)
    m = ra.Int8SwiGLU(64, 96)
    with pytest.raises(RuntimeError, match="Weights not quantized"):
        m(torch.randn(2, 64))
    lin = torch.nn.Module()
    # (no biases: Int8Linear keeps an fp16 bias, which fp32 activations on the
    # CPU reject in F.linear, as in the reference)
    lin.w_gate, lin.w_up, lin.w_down = (torch.nn.Linear(64, 96, bias=False), torch.nn.Linear(64, 96, bias=False),
                                        torch.nn.Linear(96, 64, bias=False))
    q = ra.Int8SwiGLU.from_swiglu(lin)
    x = torch.randn(3, 64)
    ref = lin.w_down(torch.nn.functional.silu(lin.w_gate(x)) * lin.w_up(x))
    assert q(x).shape == (3, 64)
    assert (q(x) - ref).abs().max() < 0.05 * ref.abs().max() + 1e-3
    with pytest.raises(AssertionError):
        ra.int8_gemm_swiglu(torch.randn(2, 64), q.w_gate.weight_int8, q.w_gate.scale, q.w_down.weight_int8,
                            q.w_down.scale)


@pytest.fixture(scope="module")
def lib():
    from rotalabs_accel_b200 import build, _capi
    build.build()
    return _capi.load_library()


def test_capi_rejects_bad_arguments(lib):
    n0 = lib.rla_launch_count()
    p = ctypes.c_void_p(16)   # never dereferenced: validation fails first
    gemm = lib.rla_w8a16_gemm_swiglu
    ok = dict(x=p, ldx=64, wg=p, wu=p, ldw=64, sg=p, su=p, sdt=1, bg=None, bu=None, bdt=0, y=p, ldy=64,
              M=4, N=64, K=64, ws=None, wsb=0)

    def st(**kw):
        a = dict(ok, **kw)
        return gemm(a["x"], a["ldx"], a["wg"], a["wu"], a["ldw"], a["sg"], a["su"], a["sdt"], a["bg"], a["bu"],
                    a["bdt"], a["y"], a["ldy"], a["M"], a["N"], a["K"], a["ws"], a["wsb"], None)

    assert st(M=-1) == 1
    assert st(sdt=3) == 1                 # bf16 scales are not a W8A16 scale type
    assert st(bdt=1, bg=p) == 1           # one bias missing
    assert st(wu=None) == 1
    assert st(su=None) == 1
    assert st(ldx=32) == 1
    assert st(ws=ctypes.c_void_p(8), wsb=64) == 4
    assert st(M=0) == 0 and st(N=0) == 0  # empty problems: nothing to do
    rms = lib.rla_rmsnorm
    assert rms(p, 64, p, 9, 1e-6, p, 64, 4, 64, None) == 1       # weight dtype
    assert rms(p, 32, p, 2, 1e-6, p, 64, 4, 64, None) == 1       # ldx < K
    assert rms(None, 64, p, 2, 1e-6, p, 64, 4, 64, None) == 1
    assert rms(p, 64, p, 2, -1.0, p, 64, 4, 64, None) == 1       # eps < 0
    assert rms(p, 64, p, 2, 1e-6, p, 64, 0, 64, None) == 0       # no rows
    assert lib.rla_launch_count() == n0


def test_gated_workspace_sizes(lib):
    # decode: the skinny plan for 2N rows (split-K partials of gate and up)
    assert lib.rla_w8a16_swiglu_workspace_size(8, 11008, 4096) % 4 == 0
    assert lib.rla_w8a16_swiglu_workspace_size(8, 256, 4096) == 0             # narrow: split-K in a cluster
    assert lib.rla_w8a16_swiglu_workspace_size(8, 128, 28672) > 4096          # > 8 slices: workspace partials
    # prefill: the counter region, then fp16 gate and up outputs, each padded to 256 bytes
    assert lib.rla_w8a16_swiglu_workspace_size(2048, 11008, 4096) == 4096 + 2 * 2048 * 11008 * 2
    assert lib.rla_w8a16_swiglu_workspace_size(33, 3, 64) == 4096 + 2 * 256
