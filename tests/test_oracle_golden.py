"""Pin the CPU oracle against golden vectors made by rotalabs-accel itself.

``tests/golden/*.npz`` were produced by ``tests/golden/make_golden.py``
running the reference (its CPU path: ``int8_gemm`` -> ``int8_gemm_torch``,
src/rotalabs_accel/kernels/gemm.py:31-48, :234-238, and its quantization,
src/rotalabs_accel/quantization/symmetric.py:24-207).  Quantization must be
bit-exact; the GEMM agrees within an fp16 ulp (fp32 accumulation in both,
different summation order).
"""

import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import w8a16_oracle as orc


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def _ulp_close(a, b, ulps=1, atol=1e-5):
    """|a - b| <= ulps * ulp(max(|a|, |b|)) + atol elementwise (fp16 ulps).

    ``atol`` absorbs fp32 summation-order noise where the result is near 0
    (there an fp16 ulp is far below the fp32 rounding of a 4096-term sum)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    mag = np.maximum(np.abs(a), np.abs(b))
    ulp = np.spacing(mag.astype(np.float16)).astype(np.float32)
    return np.all(np.abs(a - b) <= ulps * ulp + atol)


def test_reference_test_shapes_gemm(golden_dir):
    d = _load(golden_dir, "ref_test_imports_gemm.npz")
    y = orc.int8_gemm_torch(d["x"], d["w"], d["scale"])
    assert y.shape == (2, 8, 128) and y.dtype == np.float32
    np.testing.assert_allclose(y, d["y"], rtol=1e-5, atol=1e-4)


def test_quantization_bit_exact(golden_dir):
    d = _load(golden_dir, "ref_quantization.npz")
    q, s = orc.quantize_symmetric(d["t"])
    assert q.dtype == np.int8 and np.array_equal(q, d["q_tensor"])
    assert s.dtype == np.float32 and np.array_equal(s, d["s_tensor"])
    np.testing.assert_array_equal(orc.dequantize(q, s), d["r_tensor"])
    q, s = orc.quantize_weight_per_channel(d["t"])
    assert np.array_equal(q, d["q_channel"]) and np.array_equal(s, d["s_channel"])
    np.testing.assert_array_equal(orc.dequantize(q, s, dtype=np.float32, dim=0), d["r_channel"])
    # fp16 weights: the scale and quotient are rounded to fp16 (symmetric.py:62-76)
    q, s = orc.quantize_weight_per_channel(d["t_half"])
    assert np.array_equal(q, d["q_half"]) and np.array_equal(s, d["s_half"])


def test_quantization_error_metrics(golden_dir):
    d = _load(golden_dir, "ref_quantization.npz")
    e = orc.calculate_quantization_error(d["t"], d["q_tensor"], d["s_tensor"])
    got = np.array([e["max_abs_error"], e["mean_abs_error"], e["relative_error_pct"], e["snr_db"]])
    np.testing.assert_allclose(got, d["err_tensor"], rtol=1e-5)
    e = orc.calculate_quantization_error(d["t"], d["q_channel"], d["s_channel"], dim=0)
    got = np.array([e["max_abs_error"], e["mean_abs_error"], e["relative_error_pct"], e["snr_db"]])
    np.testing.assert_allclose(got, d["err_channel"], rtol=1e-5)


def test_quantization_edges_bit_exact(golden_dir):
    d = _load(golden_dir, "ref_quant_edges.npz")
    q, s = orc.quantize_weight_per_channel(d["w"])
    assert np.array_equal(q, d["q"]) and np.array_equal(s, d["s"])
    assert s[0] == 1.0                         # all-zero row -> scale 1 (symmetric.py:70)
    assert q[2, 0] == 127 and s[2] == 1.0      # row max 127 -> scale exactly 1
    assert list(q[2, 1:9]) == [2, 2, 0, -2, -2, 4, -4, 0]   # x.5 ties: round half to even
    assert q.min() >= -128 and q.max() <= 127


def test_gemm_cases(golden_dir):
    d = _load(golden_dir, "ref_gemm_cases.npz")
    n = int(d["n_cases"])
    assert n >= 8
    for i in range(n):
        x, w, s = d[f"c{i}_x"], d[f"c{i}_w"], d[f"c{i}_scale"]
        b = d[f"c{i}_bias"] if bool(d[f"c{i}_has_bias"]) else None
        y = orc.int8_gemm(x, w, s, b)
        assert y.dtype == np.float16 and y.shape == d[f"c{i}_y"].shape
        assert _ulp_close(y, d[f"c{i}_y"], ulps=1), f"case {i}"
        ref = orc.dequant_matmul_fp32(x, w, s, b)
        assert np.abs(y.astype(np.float32) - ref).max() <= 1e-2


def test_modules_golden(golden_dir):
    d = _load(golden_dir, "ref_modules.npz")
    q, s = orc.quantize_weight_per_channel(d["W"])
    assert np.array_equal(q, d["weight_int8"]) and np.array_equal(s, d["scale"])
    assert np.array_equal(q.T, d["weight_transposed"])
    y = orc.int8_gemm_torch(d["x"], q, s)
    np.testing.assert_allclose(y, d["y_int8linear"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(y, d["y_quantizedlinear"], rtol=1e-5, atol=1e-5)


def test_config0_regenerates_and_matches(golden_dir):
    """Config 0 (M=32, K=N=4096, seed 0): the seeded generator reproduces the
    reference's inputs bit for bit, and the oracle reproduces its output."""
    from rotalabs_accel_b200.synthetic import make_problem
    d = _load(golden_dir, "ref_config0.npz")
    x, q, s = make_problem(32, 4096, 4096, seed=0)
    assert hashlib.sha256(x.numpy().tobytes()).hexdigest() == str(d["sha_x"])
    assert hashlib.sha256(q.numpy().tobytes()).hexdigest() == str(d["sha_w"])
    assert np.array_equal(s.numpy(), d["scale"])
    y = orc.int8_gemm(x.numpy(), q.numpy(), s.numpy())
    assert _ulp_close(y, d["y"], ulps=1)
    ref = orc.dequant_matmul_fp32(x.numpy(), q.numpy(), s.numpy())
    err = np.abs(y.astype(np.float32) - ref).max()
    assert err <= 1e-2
    np.testing.assert_allclose(err, float(d["ref_err"]), rtol=0.25)


def test_oracle_catches_a_planted_error(golden_dir):
    """The checker is sensitive: a one-code change in one weight of a golden
    case (planted on the CPU, in the oracle's input) is detected."""
    d = _load(golden_dir, "ref_gemm_cases.npz")
    x, w, s = d["c3_x"], d["c3_w"].copy(), d["c3_scale"]
    w[5, 7] = np.int8(w[5, 7] + 1 if w[5, 7] < 127 else w[5, 7] - 1)
    b = d["c3_bias"] if bool(d["c3_has_bias"]) else None
    y = orc.int8_gemm(x, w, s, b)
    assert not _ulp_close(y, d["c3_y"], ulps=1)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_package_quantization_matches_oracle(dtype):
    """The package's host-side quantization (torch ops on the CPU) equals the
    oracle bit for bit."""
    from rotalabs_accel_b200 import quantize_weight_per_channel
    g = torch.Generator().manual_seed(99)
    w = (torch.randn(67, 300, generator=g) * 0.05).to({np.float32: torch.float32, np.float16: torch.float16}[dtype])
    w[3] = 0
    q, s = quantize_weight_per_channel(w)
    qo, so = orc.quantize_weight_per_channel(w.numpy())
    assert np.array_equal(q.numpy(), qo) and np.array_equal(s.numpy(), so)


def test_torch_restatement_matches_reference_vectors(golden_dir):
    """The torch restatement of the reference's CPU route (the CPU baseline of
    bench.py) reproduces the reference's own outputs bit for bit: it runs the
    same torch ops as the reference on the same inputs."""
    from oracle import torch_ref
    d = _load(golden_dir, "ref_gemm_cases.npz")
    for i in range(int(d["n_cases"])):
        x = torch.from_numpy(d[f"c{i}_x"])
        w = torch.from_numpy(d[f"c{i}_w"])
        s = torch.from_numpy(d[f"c{i}_scale"])
        b = torch.from_numpy(d[f"c{i}_bias"]) if bool(d[f"c{i}_has_bias"]) else None
        y = torch_ref.int8_gemm_torch(x, w, s, b)
        assert y.dtype == torch.float16
        assert np.array_equal(y.numpy(), d[f"c{i}_y"]), f"case {i}"
    d = _load(golden_dir, "ref_test_imports_gemm.npz")
    y = torch_ref.int8_gemm_torch(torch.from_numpy(d["x"]), torch.from_numpy(d["w"]), torch.from_numpy(d["scale"]))
    assert np.array_equal(y.numpy(), d["y"])
    q = torch.from_numpy(_load(golden_dir, "ref_quantization.npz")["q_channel"])
    s = torch.from_numpy(_load(golden_dir, "ref_quantization.npz")["s_channel"])
    r = torch_ref.dequantize(q, s, dtype=torch.float32, dim=0)
    assert np.array_equal(r.numpy(), _load(golden_dir, "ref_quantization.npz")["r_channel"])


def test_torch_restatement_config0(golden_dir):
    """Config 0 through the torch restatement: the reference's output, bit for bit."""
    from oracle import torch_ref
    from rotalabs_accel_b200.synthetic import make_problem
    d = _load(golden_dir, "ref_config0.npz")
    x, q, s = make_problem(32, 4096, 4096, seed=0)
    y = torch_ref.int8_gemm_torch(x, q, s)
    assert np.array_equal(y.numpy(), d["y"])
