"""API-contract tests on a CPU-only host.

They mirror rotalabs-accel's own GEMM / quantization / module tests
(tests/test_imports.py:42-62, :116-127, :133-169, :209-233) against this
package, and check the drop-in boundary: names, signatures, state-dict
layout, error types and messages (src/rotalabs_accel/kernels/gemm.py:223,
:230-231, :307-308; quantization/symmetric.py:284-285).
"""

import inspect
import os

import numpy as np
import pytest
import torch

import rotalabs_accel_b200 as ra


def test_public_names():
    for name in ("int8_gemm", "int8_gemm_torch", "Int8Linear", "quantize_symmetric", "dequantize",
                 "quantize_weight_per_channel", "calculate_quantization_error", "QuantizedLinear",
                 "get_device", "is_cuda_available", "is_triton_available", "get_device_properties",
                 "__version__"):
        assert hasattr(ra, name), name
    assert ra.__version__ == "0.2.0"


def test_signatures_match_reference():
    sig = inspect.signature(ra.int8_gemm)
    assert list(sig.parameters) == ["x", "weight_int8", "scale", "bias", "weight_transposed", "scale_fp16",
                                    "use_cublas"]
    assert list(inspect.signature(ra.int8_gemm_torch).parameters) == ["x", "weight_int8", "scale", "bias"]
    assert list(inspect.signature(ra.quantize_symmetric).parameters) == ["tensor", "bits", "dim"]
    assert list(inspect.signature(ra.dequantize).parameters) == ["quantized", "scale", "dtype", "dim"]
    assert list(inspect.signature(ra.Int8Linear.__init__).parameters) == ["self", "in_features", "out_features",
                                                                          "bias"]


def test_int8_gemm_torch_reference_test():
    # tests/test_imports.py:116-127
    x = torch.randn(2, 8, 64)
    weight = torch.randint(-128, 127, (128, 64), dtype=torch.int8)
    scale = torch.ones(128)
    out = ra.int8_gemm_torch(x, weight, scale)
    assert out.shape == (2, 8, 128)
    assert not torch.isnan(out).any()


def test_int8_gemm_cpu_matches_golden(golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_gemm_cases.npz"))
    for i in range(int(d["n_cases"])):
        x = torch.from_numpy(d[f"c{i}_x"])
        q = torch.from_numpy(d[f"c{i}_w"])
        s = torch.from_numpy(d[f"c{i}_scale"])
        b = torch.from_numpy(d[f"c{i}_bias"]) if bool(d[f"c{i}_has_bias"]) else None
        y = ra.int8_gemm(x, q, s, b)
        assert y.dtype == torch.float16
        # same torch ops as the reference on the same host: identical output
        assert torch.equal(y, torch.from_numpy(d[f"c{i}_y"])), i


def test_int8_gemm_asserts():
    x = torch.randn(4, 64).half()
    with pytest.raises(AssertionError, match="Weight must be INT8"):
        ra.int8_gemm(x, torch.zeros(8, 64), torch.ones(8))
    with pytest.raises(AssertionError, match=r"Weight shape mismatch"):
        ra.int8_gemm(x, torch.zeros(8, 32, dtype=torch.int8), torch.ones(8))
    with pytest.raises(AssertionError, match=r"Scale shape mismatch"):
        ra.int8_gemm(x, torch.zeros(8, 64, dtype=torch.int8), torch.ones(9))


def test_quantization_reference_tests():
    # tests/test_imports.py:133-169
    x = torch.randn(64, 128)
    xq, s = ra.quantize_symmetric(x)
    xr = ra.dequantize(xq, s)
    assert xq.dtype == torch.int8 and xr.shape == x.shape
    assert (x - xr).abs().mean() < 0.1
    wq, s = ra.quantize_weight_per_channel(torch.randn(64, 128))
    assert wq.dtype == torch.int8 and wq.shape == (64, 128) and s.shape == (64,)
    err = ra.calculate_quantization_error(x, xq, s := ra.quantize_symmetric(x)[1])
    assert {"max_abs_error", "mean_abs_error", "relative_error_pct", "snr_db"} <= set(err)
    assert err["max_abs_error"] >= 0
    with pytest.raises(AssertionError):
        ra.quantize_weight_per_channel(torch.randn(2, 3, 4))
    with pytest.raises(AssertionError):
        ra.quantize_symmetric(x, bits=4)


def test_quantization_golden_bit_exact(golden_dir):
    d = np.load(os.path.join(golden_dir, "ref_quantization.npz"))
    t = torch.from_numpy(d["t"])
    q, s = ra.quantize_symmetric(t)
    assert np.array_equal(q.numpy(), d["q_tensor"]) and np.array_equal(s.numpy(), d["s_tensor"])
    q, s = ra.quantize_weight_per_channel(t)
    assert np.array_equal(q.numpy(), d["q_channel"]) and np.array_equal(s.numpy(), d["s_channel"])
    q, s = ra.quantize_weight_per_channel(torch.from_numpy(d["t_half"]))
    assert np.array_equal(q.numpy(), d["q_half"]) and np.array_equal(s.numpy(), d["s_half"])
    e = np.load(os.path.join(golden_dir, "ref_quant_edges.npz"))
    q, s = ra.quantize_weight_per_channel(torch.from_numpy(e["w"]))
    assert np.array_equal(q.numpy(), e["q"]) and np.array_equal(s.numpy(), e["s"])


def test_modules_reference_tests(golden_dir):
    # tests/test_imports.py:209-233
    for cls in (ra.Int8Linear, ra.QuantizedLinear):
        lin = cls(in_features=64, out_features=128)
        with pytest.raises(RuntimeError, match="Weights not quantized. Call quantize_weights\\(\\) first."):
            lin(torch.randn(2, 8, 64))
        lin.quantize_weights(torch.randn(128, 64))
        out = lin(torch.randn(2, 8, 64))
        assert out.shape == (2, 8, 128) and not torch.isnan(out).any()
    d = np.load(os.path.join(golden_dir, "ref_modules.npz"))
    W, x = torch.from_numpy(d["W"]), torch.from_numpy(d["x"])
    il = ra.Int8Linear(64, 128)
    il.quantize_weights(W)
    assert torch.equal(il(x), torch.from_numpy(d["y_int8linear"]))
    ql = ra.QuantizedLinear(64, 128)
    ql.quantize_weights(W)
    assert torch.equal(ql(x), torch.from_numpy(d["y_quantizedlinear"]))


def test_state_dict_layout():
    il = ra.Int8Linear(64, 128, bias=True)
    sd = il.state_dict()
    assert list(sd) == ["bias", "weight_int8", "scale", "weight_transposed"]
    assert sd["weight_int8"].dtype == torch.int8 and sd["weight_int8"].shape == (128, 64)
    assert sd["scale"].dtype == torch.float32 and sd["weight_transposed"].shape == (64, 128)
    assert sd["bias"].dtype == torch.float16
    ql = ra.QuantizedLinear(64, 128, bias=True)
    sd = ql.state_dict()
    assert list(sd) == ["bias", "weight_int8", "weight_scale"]
    assert sd["bias"].dtype == torch.float32
    # weight_transposed is the reference's key, materialized on save from
    # weight_int8 (no second copy is held by the module)
    assert dict(il.named_buffers()).keys() == {"weight_int8", "scale"}
    il.quantize_weights(torch.randn(128, 64))
    assert torch.equal(il.state_dict()["weight_transposed"], il.weight_int8.t())
    assert il.state_dict()["weight_transposed"].is_contiguous()
    assert torch.equal(il.weight_transposed, il.weight_int8.t())
    # a state dict whose weight_transposed disagrees with weight_int8 is refused
    bad = il.state_dict()
    bad["weight_transposed"] = bad["weight_transposed"].clone()
    bad["weight_transposed"][0, 0] += 1
    with pytest.raises(RuntimeError, match="transpose"):
        ra.Int8Linear(64, 128, bias=True).load_state_dict(bad)
    with pytest.raises(RuntimeError, match="weight_transposed"):
        ra.Int8Linear(64, 128, bias=True).load_state_dict(
            {k: v for k, v in il.state_dict().items() if k != "weight_transposed"})
    # _quantized is not persisted: a restored module must be re-marked
    il2 = ra.Int8Linear(64, 128, bias=True)
    il.quantize_weights(torch.randn(128, 64))
    il2.load_state_dict(il.state_dict())
    with pytest.raises(RuntimeError, match="Weights not quantized"):
        il2(torch.randn(1, 64))
    il2.mark_quantized()
    x = torch.randn(1, 64).half()        # fp16 bias: fp16 activations (as in the reference)
    assert torch.equal(il2(x), il(x))


def test_from_linear_cpu():
    lin = torch.nn.Linear(64, 32, bias=True)
    m = ra.Int8Linear.from_linear(lin)
    assert m.bias.dtype == torch.float16 and m._quantized
    assert "quantized=True" in m.extra_repr()
    q = ra.QuantizedLinear.from_linear(lin)
    assert q.bias.dtype == torch.float32
    x = torch.randn(3, 64)
    assert (q(x) - lin(x)).abs().max() < 0.05


def test_device_utils_cpu():
    assert ra.get_device("cpu") == torch.device("cpu")
    assert isinstance(ra.is_cuda_available(), bool)
    props = ra.get_device_properties() if not torch.cuda.is_available() else {}
    if props:
        assert props["supports_sm100a"] is False
