"""Generate the golden vectors for the W8A16 path by running rotalabs-accel.

Run in a container where the reference is importable (its ``src/`` on
``PYTHONPATH``); the GPU box has no reference, so the outputs are committed
as ``tests/golden/*.npz`` and only ever read there.

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py          # everything
    PYTHONPATH=<reference>/src python tests/golden/make_golden.py mlp      # ref_mlp.npz only

Everything runs on the CPU, i.e. through the reference's own fallback:
``int8_gemm`` -> ``int8_gemm_torch`` (src/rotalabs_accel/kernels/gemm.py:234-238)
-> ``dequantize`` + ``F.linear``; quantization through
``quantize_symmetric`` / ``quantize_weight_per_channel``
(src/rotalabs_accel/quantization/symmetric.py:24-151).
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def mlp_vectors() -> None:
    """Config 3 pieces through the reference's CPU path: rmsnorm_torch,
    swiglu_torch and the composed block (RMSNorm -> Int8Linear gate and up
    -> SwiGLU -> Int8Linear down), fp16 activations, fp16 RMSNorm weight."""
    import rotalabs_accel as ra
    from rotalabs_accel import int8_gemm, quantize_weight_per_channel, rmsnorm_torch, swiglu_torch
    assert ra.__version__ == "0.2.0"
    g = torch.Generator().manual_seed(33)
    M, H, I = 8, 128, 352
    x = torch.randn(M, H, generator=g).half()
    x[3] = 0                                            # a zero row: rms = 1/sqrt(eps)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).half()
    xn = rmsnorm_torch(x, nw, 1e-6)
    qs = {}
    for name, (n_out, n_in) in (("gate", (I, H)), ("up", (I, H)), ("down", (H, I))):
        q, s = quantize_weight_per_channel(torch.randn(n_out, n_in, generator=g) * 0.02)
        qs[name] = (q, s.half())
    gate = int8_gemm(xn, *qs["gate"])
    up = int8_gemm(xn, *qs["up"])
    h = swiglu_torch(gate, up)
    y = int8_gemm(h, *qs["down"])
    # SwiGLU alone on a spread of magnitudes (large negative, zero, large positive)
    ga = (torch.linspace(-30, 30, 241) * torch.rand(241, generator=g)).half()
    ua = torch.randn(241, generator=g).half()
    sa = swiglu_torch(ga, ua)
    # RMSNorm alone with an fp32 weight (dtype promotion: fp32 result)
    xr = (torch.randn(4, 96, generator=g) * 3).half()
    wr = torch.rand(96, generator=g) + 0.5
    yr = rmsnorm_torch(xr, wr, 1e-5)
    np.savez_compressed(os.path.join(HERE, "ref_mlp.npz"), x=x.numpy(), norm_weight=nw.numpy(), eps=np.array(1e-6),
                        xn=xn.numpy(), wg=qs["gate"][0].numpy(), sg=qs["gate"][1].numpy(),
                        wu=qs["up"][0].numpy(), su=qs["up"][1].numpy(), wd=qs["down"][0].numpy(),
                        sd=qs["down"][1].numpy(), gate=gate.numpy(), up=up.numpy(), h=h.numpy(), y=y.numpy(),
                        swiglu_gate=ga.numpy(), swiglu_up=ua.numpy(), swiglu_out=sa.numpy(),
                        rms_x=xr.numpy(), rms_w=wr.numpy(), rms_y=yr.numpy())
    print("ref_mlp.npz written to", HERE)


def main() -> None:
    if len(sys.argv) > 1 and sys.argv[1] == "mlp":
        return mlp_vectors()
    import rotalabs_accel as ra  # the reference package
    from rotalabs_accel import (int8_gemm, int8_gemm_torch, quantize_symmetric, dequantize,
                                quantize_weight_per_channel, calculate_quantization_error,
                                Int8Linear, QuantizedLinear)
    assert ra.__version__ == "0.2.0"
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    # 1. The reference's own test shapes (tests/test_imports.py:116-127, :133-169, :209-233),
    #    with fixed seeds so the outputs can be pinned.
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(2, 8, 64, generator=g)
    w = torch.randint(-128, 127, (128, 64), dtype=torch.int8, generator=g)
    s = torch.ones(128)
    y = int8_gemm_torch(x, w, s)
    np.savez_compressed(os.path.join(HERE, "ref_test_imports_gemm.npz"),
                        x=x.numpy(), w=w.numpy(), scale=s.numpy(), y=y.numpy())

    g = torch.Generator().manual_seed(4321)
    t = torch.randn(64, 128, generator=g)
    q_t, s_t = quantize_symmetric(t)
    r_t = dequantize(q_t, s_t)
    q_c, s_c = quantize_weight_per_channel(t)
    r_c = dequantize(q_c, s_c, dtype=torch.float32, dim=0)
    err = calculate_quantization_error(t, q_t, s_t)
    err_c = calculate_quantization_error(t, q_c, s_c, dim=0)
    th = t.half()
    q_h, s_h = quantize_weight_per_channel(th)   # fp16 weight: fp16 scale arithmetic
    np.savez_compressed(os.path.join(HERE, "ref_quantization.npz"),
                        t=t.numpy(), q_tensor=q_t.numpy(), s_tensor=s_t.numpy(), r_tensor=r_t.numpy(),
                        q_channel=q_c.numpy(), s_channel=s_c.numpy(), r_channel=r_c.numpy(),
                        err_tensor=np.array([err["max_abs_error"], err["mean_abs_error"],
                                             err["relative_error_pct"], err["snr_db"]]),
                        err_channel=np.array([err_c["max_abs_error"], err_c["mean_abs_error"],
                                              err_c["relative_error_pct"], err_c["snr_db"]]),
                        t_half=th.numpy(), q_half=q_h.numpy(), s_half=s_h.numpy())

    # 2. Quantization edge cases: zero rows (scale -> 1, symmetric.py:70), exact
    #    half-way values (round half to even), and the clamp.
    e = torch.zeros(6, 32)
    e[1, :] = torch.linspace(-1.0, 1.0, 32)
    e[2, :] = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5] * 4)
    e[2, 0] = 127.0                                   # row scale exactly 1.0 -> x.5 values tie
    e[3, :] = -1e-30
    e[4, 5] = 3.0e4
    e[5, :] = torch.arange(32, dtype=torch.float32) - 16.0
    q_e, s_e = quantize_weight_per_channel(e)
    np.savez_compressed(os.path.join(HERE, "ref_quant_edges.npz"), w=e.numpy(), q=q_e.numpy(), s=s_e.numpy())

    # 3. fp16 GEMM cases through the reference dispatcher, ragged sizes, with and
    #    without bias, fp32 and fp16 scales, 2-D and 3-D x.
    cases = []
    for (M, N, K, bias, sdt, seed) in [
            (1, 33, 64, False, "f32", 11), (3, 128, 96, True, "f16", 12), (17, 40, 208, False, "f16", 13),
            (16, 256, 512, True, "f32", 14), (5, 7, 16, False, "f16", 15), (33, 129, 272, True, "f16", 16),
            (64, 96, 1024, False, "f16", 17), (2, 300, 4096, False, "f16", 18)]:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(M, K, generator=g).half()
        W = torch.randn(N, K, generator=g) * 0.02
        q, s = quantize_weight_per_channel(W)
        s = s.half() if sdt == "f16" else s
        b = (torch.randn(N, generator=g) * 0.1).half() if bias else None
        y = int8_gemm(x, q, s, b)
        cases.append(dict(M=M, N=N, K=K, x=x.numpy(), w=q.numpy(), scale=s.numpy(),
                          bias=(b.numpy() if b is not None else np.zeros(0, np.float16)),
                          has_bias=bias, y=y.numpy()))
    arrs = {}
    for i, c in enumerate(cases):
        for k, v in c.items():
            arrs[f"c{i}_{k}"] = np.asarray(v)
    arrs["n_cases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "ref_gemm_cases.npz"), **arrs)

    # 3-D x through Int8Linear and QuantizedLinear (fp32 activations, as in
    # tests/test_imports.py:209-233), with the modules' own quantization.
    g = torch.Generator().manual_seed(77)
    Wm = torch.randn(128, 64, generator=g)
    xm = torch.randn(2, 8, 64, generator=g)
    il = Int8Linear(64, 128)
    il.quantize_weights(Wm)
    ql = QuantizedLinear(64, 128)
    ql.quantize_weights(Wm)
    np.savez_compressed(os.path.join(HERE, "ref_modules.npz"), W=Wm.numpy(), x=xm.numpy(),
                        y_int8linear=il(xm).detach().numpy(), y_quantizedlinear=ql(xm).detach().numpy(),
                        weight_int8=il.weight_int8.numpy(), scale=il.scale.numpy(),
                        weight_transposed=il.weight_transposed.numpy())

    # 4. Config 0 of the benchmark: M=32, K=N=4096, seed 0, x ~ N(0,1) fp16,
    #    W ~ N(0, 0.02) per-channel int8, fp16 scale, no bias.  The inputs are
    #    regenerated from the seed by rotalabs_accel_b200.synthetic.make_problem;
    #    their hashes pin that regeneration.
    g = torch.Generator().manual_seed(0)
    x = torch.randn(32, 4096, generator=g).half()
    W = torch.randn(4096, 4096, generator=g) * 0.02
    q, s = quantize_weight_per_channel(W)
    s16 = s.half()
    y = int8_gemm(x, q, s16)
    ref32 = x.float() @ (q.float() * s16.float()[:, None]).T
    np.savez_compressed(os.path.join(HERE, "ref_config0.npz"),
                        scale=s16.numpy(), y=y.numpy(),
                        sha_x=np.array(_sha(x)), sha_w=np.array(_sha(q)),
                        ref_err=np.array(float((y.float() - ref32).abs().max())))
    mlp_vectors()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    sys.exit(main())
