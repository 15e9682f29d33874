"""GPU parity of the sm_100a W8A16 kernels (run with ``-m gpu``).

Every case goes through the C ABI (``rla_w8a16_gemm`` via the package API)
and is compared with:
  * the CPU oracle (``oracle/w8a16_oracle.py``, pinned to rotalabs-accel's
    own outputs) and the committed golden vectors, at small sizes;
  * an fp32-accumulated dequant-matmul (torch fp32 on the GPU, TF32 off) at
    the benchmark configurations' full sizes.
Tolerance (the north star's): max |y - y_fp32| <= 1e-2 with fp16 output;
where |y_fp32| is large the bound also allows one fp16 ulp of the value
(half an ulp of fp16 exceeds 1e-2 above 32).
"""

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _fp32_ref(x2d, q, s, b=None):
    torch.backends.cuda.matmul.allow_tf32 = False
    w = q.float() * s.float()[:, None]
    y = x2d.float() @ w.t()
    if b is not None:
        y = y + b.float()
    return y


def _check(y, ref, tol=TOL):
    y = y.float()
    err = (y - ref).abs()
    bound = tol + torch.abs(ref) * (2.0 ** -10)
    bad = err > bound
    assert not bool(bad.any()), (
        f"max err {err.max().item():.3e} at |ref|={ref.abs().flatten()[err.argmax()].item():.3f}; "
        f"{int(bad.sum())} of {bad.numel()} outside tolerance")
    return err.max().item()


def _problem(M, N, K, seed, scale_dtype=torch.float16, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=device).half()
    w = torch.randn(N, K, generator=g, device=device) * 0.02
    from rotalabs_accel_b200 import quantize_weight_per_channel
    q, s = quantize_weight_per_channel(w)
    return x, q, s.to(scale_dtype)


@pytest.fixture(scope="module")
def dev(cuda_lib):
    cap = torch.cuda.get_device_capability()
    assert cap[0] == 10, f"sm_100 device required, got {cap}"
    return torch.device("cuda", 0)


def test_library_is_native_and_loaded(dev):
    from rotalabs_accel_b200 import _capi
    x, q, s = _problem(4, 256, 512, 1)
    from rotalabs_accel_b200 import int8_gemm
    torch.cuda.synchronize()
    before = _capi.launch_count()
    int8_gemm(x, q, s)
    torch.cuda.synchronize()
    assert _capi.launch_count() == before + 1
    import ctypes
    maps = open("/proc/self/maps").read()
    assert "librla_w8a16.so" in maps


def test_golden_cases_vs_reference_outputs(dev, golden_dir):
    from rotalabs_accel_b200 import int8_gemm, _capi
    from oracle import w8a16_oracle as orc
    d = np.load(os.path.join(golden_dir, "ref_gemm_cases.npz"))
    for i in range(int(d["n_cases"])):
        x = torch.from_numpy(d[f"c{i}_x"]).to(dev)
        q = torch.from_numpy(d[f"c{i}_w"]).to(dev)
        s = torch.from_numpy(d[f"c{i}_scale"]).to(dev)
        b = torch.from_numpy(d[f"c{i}_bias"]).to(dev) if bool(d[f"c{i}_has_bias"]) else None
        y = int8_gemm(x, q, s, b)
        assert y.dtype == torch.float16 and tuple(y.shape) == d[f"c{i}_y"].shape
        ref = _fp32_ref(x, q, s, b)
        _check(y, ref)
        # against the reference's own output and the oracle
        gold = torch.from_numpy(d[f"c{i}_y"]).to(dev).float()
        assert (y.float() - gold).abs().max().item() <= 2 * TOL
        yo = torch.from_numpy(orc.int8_gemm(d[f"c{i}_x"], d[f"c{i}_w"], d[f"c{i}_scale"],
                                            d[f"c{i}_bias"] if bool(d[f"c{i}_has_bias"]) else None)).to(dev)
        assert (y.float() - yo.float()).abs().max().item() <= 2 * TOL


def test_config0_vs_golden(dev, golden_dir):
    """BASELINE config 0 (M=32, K=N=4096, seed 0, fp16 scale, no bias)."""
    from rotalabs_accel_b200 import int8_gemm
    from rotalabs_accel_b200.synthetic import make_problem
    d = np.load(os.path.join(golden_dir, "ref_config0.npz"))
    x, q, s = make_problem(32, 4096, 4096, seed=0)
    y = int8_gemm(x.to(dev), q.to(dev), s.to(dev))
    ref = _fp32_ref(x.to(dev), q.to(dev), s.to(dev))
    err = _check(y, ref)
    assert err <= TOL
    gold = torch.from_numpy(d["y"]).to(dev).float()
    assert (y.float() - gold).abs().max().item() <= 2 * TOL


@pytest.fixture(params=["stream", "skinny"])
def decode_kernel(request, dev):
    """Run a decode test once per decode kernel family."""
    from rotalabs_accel_b200 import _capi
    _capi.set_decode_kernel(request.param)
    yield request.param
    _capi.set_decode_kernel("auto")


@pytest.mark.parametrize("M", [1, 4, 8, 16])
@pytest.mark.parametrize("KN", [(4096, 4096), (4096, 11008), (11008, 4096), (4096, 14336)])
def test_decode_sweep(dev, decode_kernel, M, KN):
    """the decode GEMV sweep at full size."""
    from rotalabs_accel_b200 import int8_gemm, _capi
    K, N = KN
    x, q, s = _problem(M, N, K, seed=M * 7 + K + N)
    assert _capi.plan(M, N, K)["kernel_name"] == decode_kernel
    y = int8_gemm(x, q, s)
    _check(y, _fp32_ref(x, q, s))


@pytest.mark.parametrize("M,N,K", [(1, 1, 16), (3, 33, 64), (7, 129, 80), (17, 100, 272), (31, 257, 1024),
                                   (32, 4096, 4096), (8, 1024, 28672), (16, 64, 65536), (2, 5000, 48),
                                   (9, 192, 4160), (1, 7, 4096)])
@pytest.mark.parametrize("bias", [None, "f16"])
def test_decode_kernels_ragged(dev, decode_kernel, M, N, K, bias):
    """Ragged decode shapes on both decode kernels: partial row blocks, K not a
    multiple of the stage, row blocks split across many CTAs."""
    from rotalabs_accel_b200 import int8_gemm, _capi
    x, q, s = _problem(M, N, K, seed=M * 31 + N + K)
    b = (torch.randn(N, device=dev) * 0.1).half() if bias else None
    assert _capi.plan(M, N, K)["kernel_name"] == decode_kernel
    y1 = int8_gemm(x, q, s, b)
    y2 = int8_gemm(x, q, s, b)
    assert torch.equal(y1, y2)          # fixed-order reductions: bit-reproducible
    _check(y1, _fp32_ref(x, q, s, b))


@pytest.mark.parametrize("KN", [(4096, 12288), (4096, 11008), (11008, 4096)])
def test_prefill_llama7b(dev, KN):
    """M = 2048 prefill through the tcgen05 kernel."""
    from rotalabs_accel_b200 import int8_gemm, _capi
    K, N = KN
    x, q, s = _problem(2048, N, K, seed=K + N)
    assert _capi.plan(2048, N, K)["kernel_name"] == "tcgen05"
    y = int8_gemm(x, q, s)
    _check(y, _fp32_ref(x, q, s))


@pytest.mark.parametrize("M", [1, 16, 4096])
@pytest.mark.parametrize("KN", [(8192, 28672), (28672, 8192)])
def test_llama70b_single_gpu(dev, M, KN):
    """BASELINE config 4 shapes at world size 1."""
    from rotalabs_accel_b200 import int8_gemm
    K, N = KN
    x, q, s = _problem(M, N, K, seed=M + K)
    y = int8_gemm(x, q, s)
    ref = _fp32_ref(x, q, s)
    _check(y, ref)
    del q, ref


@pytest.mark.parametrize("M,N,K", [
    (1, 1, 16), (3, 33, 64), (7, 129, 80), (17, 100, 272), (31, 257, 1024),   # skinny, ragged
    (33, 130, 64), (64, 512, 4096), (100, 1000, 2048), (257, 384, 1040),     # tcgen05, ragged M/N/K
    (300, 129, 4100), (512, 256, 8),                                          # tcgen05, K % 16 != 0 / tiny K
    (1000, 5000, 1040), (2304, 8200, 4096), (256, 18944, 64),                 # tcgen05, many tiles, ragged
    (5, 7, 13), (40, 50, 30), (2, 3, 1),                                      # generic (K % 8 != 0)
])
@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("bias", [None, "f16", "f32"])
def test_ragged_shapes_vs_oracle(dev, M, N, K, scale_dtype, bias):
    from rotalabs_accel_b200 import int8_gemm
    from oracle import w8a16_oracle as orc
    x, q, s = _problem(M, N, K, seed=M * 1000 + N + K, scale_dtype=scale_dtype)
    b = None
    if bias is not None:
        b = (torch.randn(N, device=dev) * 0.1).to(torch.float16 if bias == "f16" else torch.float32)
    y = int8_gemm(x, q, s, b)
    _check(y, _fp32_ref(x, q, s, b))
    if M * N * K <= 2e7:
        yo = orc.int8_gemm(x.cpu().numpy(), q.cpu().numpy(), s.cpu().numpy(),
                           None if b is None else b.cpu().numpy())
        # the oracle rounds the dequantized weight to fp16 first (gemm.py:43)
        assert (y.float().cpu() - torch.from_numpy(yo.astype(np.float32))).abs().max().item() <= 2 * TOL


def test_extreme_weights_and_zero_rows(dev):
    """int8 extremes -128 / 127 and all-zero rows (scale 1)."""
    from rotalabs_accel_b200 import int8_gemm
    for M in (4, 64):
        N, K = 256, 512
        q = torch.full((N, K), 127, dtype=torch.int8, device=dev)
        q[1::2] = -128
        q[10] = 0
        s = torch.full((N,), 1e-3, dtype=torch.float16, device=dev)
        s[10] = 1.0
        x = torch.randn(M, K, device=dev).half() * 0.1
        y = int8_gemm(x, q, s)
        _check(y, _fp32_ref(x, q, s))
        assert (y[:, 10] == 0).all()


def test_strided_and_3d_inputs(dev):
    from rotalabs_accel_b200 import int8_gemm
    x, q, s = _problem(48, 320, 512, 5)
    wide = torch.zeros(48, 640, device=dev, dtype=torch.float16)
    wide[:, :512] = x
    xs = wide[:, :512]                        # ldx = 640 > K
    assert not xs.is_contiguous()
    _check(int8_gemm(xs, q, s), _fp32_ref(x, q, s))
    x3 = x.view(4, 12, 512)
    y3 = int8_gemm(x3, q, s)
    assert y3.shape == (4, 12, 320)
    _check(y3.view(48, 320), _fp32_ref(x, q, s))
    xt = torch.randn(512, 8, device=dev).half().t()   # inner stride != 1
    _check(int8_gemm(xt, q, s), _fp32_ref(xt.contiguous(), q, s))


def test_empty_and_k0(dev):
    from rotalabs_accel_b200 import int8_gemm
    q = torch.zeros(16, 0, dtype=torch.int8, device=dev)
    s = torch.ones(16, device=dev)
    b = torch.arange(16, device=dev).half()
    y = int8_gemm(torch.zeros(3, 0, device=dev).half(), q, s, b)
    assert torch.equal(y, b.expand(3, 16))
    y = int8_gemm(torch.zeros(0, 64, device=dev).half(), torch.zeros(16, 64, dtype=torch.int8, device=dev), s)
    assert y.shape == (0, 16)


def test_deterministic_split_k(dev):
    """Split-K partial sums are added in a fixed order: bit-identical reruns."""
    from rotalabs_accel_b200 import int8_gemm, _capi
    x, q, s = _problem(8, 1024, 28672, 3)          # one rank's column shard of 70B gate/up
    assert _capi.plan(8, 1024, 28672)["splits"] > 1
    y1 = int8_gemm(x, q, s)
    y2 = int8_gemm(x, q, s)
    assert torch.equal(y1, y2)
    _check(y1, _fp32_ref(x, q, s))


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (8, 512, 8192), (16, 1024, 4096), (32, 4096, 960),
                                   (3, 1000, 4096), (1, 128, 28672), (8, 256, 28672)])
@pytest.mark.parametrize("bias", [None, "f32"])
def test_split_k_cluster_and_workspace_paths(dev, M, N, K, bias):
    """Split-K of up to 8 slices adds the slices inside a thread-block
    cluster (no workspace); more slices add fp32 partial sums in the
    workspace.  Both are bit-identical from run to run and within the bar."""
    from rotalabs_accel_b200 import int8_gemm, _capi
    x, q, s = _problem(M, N, K, seed=M + N + K, scale_dtype=torch.float32)
    b = (torch.randn(N, device=dev) * 0.1) if bias == "f32" else None
    p = _capi.plan(M, N, K)
    ws = _capi.load_library().rla_w8a16_workspace_size(M, N, K)
    if p["kernel_name"] == "skinny" and p["splits"] > 1:
        assert (ws == 0) == (p["splits"] <= 8), (p, ws)
    y1 = int8_gemm(x, q, s, b)
    y2 = int8_gemm(x, q, s, b)
    assert torch.equal(y1, y2)
    _check(y1, _fp32_ref(x, q, s, b))
    assert _capi.device_error() == 0


def test_workspace_shared_across_shapes(dev):
    """Split-K calls of different shapes share one workspace: the fixed
    counter region must not overlap an earlier call's partial sums."""
    from rotalabs_accel_b200 import int8_gemm, _capi
    # (narrow layers: the selector splits K only while the grid stays one wave)
    # (up to 8 slices add up in a thread-block cluster and leave the workspace
    # alone; (1, 128, 28672) and (8, 256, 28672) split further, through it)
    shapes = [(4, 256, 1024), (16, 1024, 4096), (1, 1024, 28672), (16, 256, 4096), (8, 512, 8192),
              (1, 2048, 4096), (32, 512, 4096), (1, 128, 28672), (8, 256, 28672)]
    probs = [_problem(M, N, K, seed=i) for i, (M, N, K) in enumerate(shapes)]
    # the two decode kernels use the same workspace with the same fixed layout
    for kern in ("skinny", "stream", "skinny", "stream"):
        _capi.set_decode_kernel(kern)
        try:
            for (M, N, K), (x, q, s) in zip(shapes, probs):
                if kern == "skinny":
                    assert _capi.plan(M, N, K)["splits"] > 1
                _check(int8_gemm(x, q, s), _fp32_ref(x, q, s))
        finally:
            _capi.set_decode_kernel("auto")


def test_fp32_and_bf16_activations(dev):
    """Non-fp16 activations are cast to fp16; output is fp16 (reference GPU path)."""
    from rotalabs_accel_b200 import int8_gemm
    x, q, s = _problem(8, 256, 1024, 9)
    for dt in (torch.float32, torch.bfloat16):
        y = int8_gemm(x.to(dt), q, s)
        assert y.dtype == torch.float16
        _check(y, _fp32_ref(x.to(dt).half(), q, s))


def test_modules_on_gpu(dev, golden_dir):
    from rotalabs_accel_b200 import Int8Linear, QuantizedLinear
    d = np.load(os.path.join(golden_dir, "ref_modules.npz"))
    W = torch.from_numpy(d["W"]).to(dev)
    m = Int8Linear(64, 128).to(dev)
    m.quantize_weights(W)
    assert torch.equal(m.weight_int8.cpu(), torch.from_numpy(d["weight_int8"]))
    assert torch.equal(m.scale.cpu(), torch.from_numpy(d["scale"]))
    assert torch.equal(m.weight_transposed.cpu(), torch.from_numpy(d["weight_transposed"]))
    # the module holds N*K + 4N bytes of weight state on the device (no second,
    # transposed copy); its saved state dict is the reference's byte for byte
    assert sum(b.numel() * b.element_size() for b in m.buffers()) == 128 * 64 + 4 * 128
    sd = m.state_dict()
    assert list(sd) == ["weight_int8", "scale", "weight_transposed"]
    for k in ("weight_int8", "scale", "weight_transposed"):
        assert sd[k].cpu().numpy().tobytes() == np.ascontiguousarray(d[k]).tobytes(), k
    m3 = Int8Linear(64, 128).to(dev)
    m3.load_state_dict(sd)
    m3.mark_quantized()
    assert torch.equal(m3(torch.from_numpy(d["x"]).to(dev)), m(torch.from_numpy(d["x"]).to(dev)))
    x = torch.from_numpy(d["x"]).to(dev)
    y = m(x)
    assert y.shape == (2, 8, 128) and y.dtype == torch.float16
    ref = torch.from_numpy(d["y_int8linear"]).to(dev)
    assert (y.float() - ref).abs().max().item() <= 2e-2
    lin = torch.nn.Linear(64, 128, bias=True).to(dev)
    m2 = Int8Linear.from_linear(lin)
    assert m2.bias.dtype == torch.float16
    y2 = m2(x.half())
    _check(y2.view(-1, 128), _fp32_ref(x.half().view(-1, 64), m2.weight_int8, m2.scale, m2.bias))
    ql = QuantizedLinear(64, 128).to(dev)
    ql.quantize_weights(W)
    yq = ql(x)
    assert yq.dtype == torch.float32
    assert (yq - torch.from_numpy(d["y_quantizedlinear"]).to(dev)).abs().max().item() <= 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_kernel_bit_exact(dev, dtype, golden_dir):
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.quantization import quantize_symmetric
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(300, 1000, generator=g) * 0.02).to(dtype)
    w[7] = 0
    w[8, 3] = 1.0
    q, s = _capi.quantize_per_channel(w.to(dev))
    qc, sc = quantize_symmetric(w, dim=1)
    assert torch.equal(q.cpu(), qc) and torch.equal(s.cpu(), sc)
    d = np.load(os.path.join(golden_dir, "ref_quantization.npz"))
    if dtype == torch.float32:
        q, s = _capi.quantize_per_channel(torch.from_numpy(d["t"]).to(dev))
        assert np.array_equal(q.cpu().numpy(), d["q_channel"]) and np.array_equal(s.cpu().numpy(), d["s_channel"])
    elif dtype == torch.float16:
        q, s = _capi.quantize_per_channel(torch.from_numpy(d["t_half"]).to(dev))
        assert np.array_equal(q.cpu().numpy(), d["q_half"]) and np.array_equal(s.cpu().numpy(), d["s_half"])
    e = np.load(os.path.join(golden_dir, "ref_quant_edges.npz"))
    q, s = _capi.quantize_per_channel(torch.from_numpy(e["w"]).to(dev))
    assert np.array_equal(q.cpu().numpy(), e["q"]) and np.array_equal(s.cpu().numpy(), e["s"])


def test_gather_columns(dev):
    from rotalabs_accel_b200 import _capi
    for world, M, nl in [(2, 1, 512), (4, 16, 256), (8, 3, 100), (8, 33, 1024)]:
        st = torch.randn(world, M, nl, device=dev).half()
        out = torch.empty(M, world * nl, device=dev, dtype=torch.float16)
        _capi.gather_columns(st, world, M, nl, out)
        assert torch.equal(out, st.permute(1, 0, 2).reshape(M, world * nl))


def test_no_device_error_recorded(dev):
    from rotalabs_accel_b200 import _capi
    assert _capi.device_error() == 0
