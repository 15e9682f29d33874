"""Benchmark of the W8A16 GEMM path on B200 (one JSON line on rank 0).

Workload (a "step"): the decode GEMV sweep of the benchmark configuration --
M in {1, 4, 8, 16} x (K, N) in {(4096, 4096), (4096, 11008), (11008, 4096),
(4096, 14336)}: 16 W8A16 GEMMs, each with its own int8 weight (663 MB of
weights in all, > the 126 MB L2, so every GEMM streams its weight from HBM).
x ~ N(0, 1) fp16, W ~ N(0, 0.02) quantized per output channel, fp16 scales,
seeded synthetic data.  With N GPUs every rank runs the whole sweep on its
own batch (data-parallel decode, weak scaling): these 7B layers fit one GPU
many times over, and splitting them only adds latency to launches that are
already latency-bound.

Column-parallel sharding is measured where the benchmark configuration asks
for it, on the Llama-3-70B MLP GEMMs of config 4 (the ``sharded`` object, at
every N, N = 1 included): each rank holds N_layer / world output channels
and runs its slice.  For decode (M = 1, 16), by default (``--exchange p2p``)
the decode kernel sends its slice to every peer over NVLink as flagged words
and unpacks theirs in the same launch (``rla_w8a16_gemm_allgather``);
``--exchange nccl`` all-gathers the slices with NCCL instead.  The M = 4096
prefill slice runs the tcgen05 kernel, then an NCCL all-gather (strong
scaling).

Reported (rank 0, one line):
  value      algorithmic bytes of the whole sweep (sum of N*K + 2MK + 2N + 2MN
             over the 16 GEMMs), times the number of GPUs, / device time per
             step, TB/s; steps replay a CUDA graph of the step; device time is
             CUDA events on the replay stream, max over ranks.
  e2e        the same metric through the public API (``Int8Linear``), eager,
             with every step's x copied host->device from pinned memory and
             every y copied back.
  roofline   the decode kernel: bytes per launch / its average launch time,
             against the measured HBM copy bandwidth.
  prefill    (N=1) the M=2048 prefill GEMMs of the benchmark configuration,
             TFLOP/s, against the measured dense bf16/fp16 tensor peak.
  mlp_block  (N=1) config 3, the Llama-2-7B MLP block (RMSNorm -> gated
             gate/up GEMM -> down) at M=8 (TB/s; 3 launches, SwiGLU in the
             decode kernel's epilogue) and M=2048 (TFLOP/s; 5 launches), next
             to the same block unfused (6 launches).
  sharded    config 4: the 70B MLP GEMMs column-parallel over the N GPUs,
             per shape and M, whole-job TB/s (decode) or TFLOP/s (M = 4096).
  cpu_baseline  rotalabs-accel's CPU route (int8_gemm -> int8_gemm_torch,
             restated with the same torch ops and pinned bit for bit to the
             reference's outputs) on one pass of the sweep, on every host core.

``--impl reference`` times the same CPU route (rotalabs-accel is Python and
Triton: nothing of it compiles, and its source is not on the GPU host) on
the same workload and metric: one pass of the 16-GEMM sweep per step.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DECODE_MS = (1, 4, 8, 16)
DECODE_KN = ((4096, 4096), (4096, 11008), (11008, 4096), (4096, 14336))
PREFILL_M = 2048
PREFILL_KN = ((4096, 12288), (4096, 11008), (11008, 4096))
SHARDED_KN = ((8192, 28672), (28672, 8192))
SHARDED_DECODE_M = (1, 16)
SHARDED_PREFILL_M = 4096
L2_BYTES = 126e6
METRIC = "W8A16 GEMM achieved TB/s (decode M<=16) and TFLOPS (prefill M=2048) vs B200 roofline"


def sweep():
    return [(M, K, N) for M in DECODE_MS for (K, N) in DECODE_KN]


def gemm_bytes(M, K, N):
    return N * K + 2 * M * K + 2 * N + 2 * M * N


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def load_traffic(name="decode_sweep_traffic.json"):
    """Per-launch DRAM bytes (read + write) from one ncu capture: the decode
    kernel's mean over the sweep's 16 launches, or one config 2 prefill
    launch (the JSON files under profiles/ hold the figure and the command
    that measured it)."""
    p = os.path.join(ROOT, "profiles", name)
    try:
        return float(json.load(open(p))["traffic_bytes_per_launch"])
    except (OSError, ValueError, KeyError, TypeError):
        return None


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(prefix=f"rla_clocks_gpu{self.gpu}_", suffix=".csv")
            self.fh = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], None, set()
        keep = os.environ.get("RLA_BENCH_CLOCKS_DIR")   # optional: keep the raw samples there
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if keep:
            import shutil
            os.makedirs(keep, exist_ok=True)
            shutil.copy(self.path, os.path.join(keep, f"clocks_gpu{self.gpu}.csv"))
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU arms: rotalabs-accel's own CPU route (int8_gemm -> int8_gemm_torch:
# dequantize the whole weight to fp16, then F.linear), restated with the same
# torch ops in oracle/torch_ref.py and pinned bit for bit to the reference's
# outputs; torch's own intra-op threads on every host core.
# ---------------------------------------------------------------------------
REF_SAMPLE_DESC = ("rotalabs-accel's CPU route for CPU tensors (int8_gemm -> int8_gemm_torch: whole-weight "
                   "dequantize to fp16, then F.linear), restated with the same torch ops (oracle/torch_ref.py, "
                   "bit-identical to the reference's outputs), torch intra-op threads = cores")


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_problems(jobs, seed0):
    """Host copies of the sweep's GEMMs: x ~ N(0, 1) fp16, W ~ N(0, 0.02)
    quantized per output channel (the package's host quantization, the
    reference's arithmetic), fp16 scales."""
    import torch
    from rotalabs_accel_b200.quantization import quantize_weight_per_channel
    probs = []
    for i, (M, K, N) in enumerate(jobs):
        g = torch.Generator().manual_seed(seed0 + i)
        x = torch.randn(M, K, generator=g).half()
        q, sc = quantize_weight_per_channel(torch.randn(N, K, generator=g) * 0.02)
        probs.append((x, q, sc.half()))
    return probs


def time_cpu_gemms(probs, threads):
    """Wall time of one int8_gemm_torch per problem, in order (seconds)."""
    import torch
    from oracle import torch_ref
    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    for (x, q, sc) in probs:
        torch_ref.int8_gemm_torch(x, q, sc)
    return time.perf_counter() - t0


def run_reference(args):
    """--impl reference: the reference's CPU route, on this host's cores.  A
    step is one pass of the 16-GEMM sweep, the same workload as the GPU arm's
    step; if --steps such passes would not end within a few minutes, each
    step is a fixed sample of whole GEMMs of the sweep (stated in the line)."""
    threads = cpu_threads()
    jobs = sweep()
    probs = cpu_problems(jobs, 1000)
    t_pass = time_cpu_gemms(probs, threads)          # first pass: warm-up, also sizes the run
    for _ in range(max(0, min(args.warmup, 3) - 1)):
        t_pass = min(t_pass, time_cpu_gemms(probs, threads))
    budget_s = 240.0
    per_step = len(jobs)
    if args.steps * t_pass > budget_s:
        per_step = max(1, int(len(jobs) * budget_s / (args.steps * t_pass)))
    tot_b, tot_t, k = 0, 0.0, 0
    for i in range(args.steps):
        sel = [(k + j) % len(jobs) for j in range(per_step)]
        k += per_step
        tot_t += time_cpu_gemms([probs[j] for j in sel], threads)
        tot_b += sum(gemm_bytes(*jobs[j]) for j in sel)
    value = tot_b / tot_t / 1e12
    sample = (f"one pass of the 16-GEMM decode sweep per step" if per_step == len(jobs) else
              f"{per_step} of the sweep's 16 GEMMs per step, in sweep order, cycling")
    line = {"metric": METRIC, "value": round(value, 6), "unit": "TB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(tot_t / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (int8 weights)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": "decode GEMV sweep, BASELINE config 1: M in {1,4,8,16} x (K,N) in "
                                   "{(4096,4096),(4096,11008),(11008,4096),(4096,14336)}, 16 GEMMs per step",
                       "parallelism": "host CPU"},
            "cpu_baseline": {"value": round(value, 6), "unit": "TB/s", "cores": threads, "kind": "port",
                             "sample": f"{sample}; {REF_SAMPLE_DESC}"},
            "e2e": {"value": round(value, 6), "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def measure_mlp_block(ra, _capi, dev, capture, timed, peaks, args):
    """Config 3: RMSNorm(4096) -> gate/up 4096 -> 11008 -> SwiGLU -> down
    11008 -> 4096 at M = 8 (decode, HBM-bound: bytes / time) and M = 2048
    (prefill, tensor-bound: GEMM FLOPs / time).  One CUDA graph per step of
    the block as the package runs it (3 launches at M = 8, 5 at M = 2048), and of the unfused
    composition through the same library (RMSNorm, gate GEMM, up GEMM, torch
    SiLU and product, down GEMM: 6 launches) for comparison.  Each step uses one of 3 copies of
    the weights (405 MB), more than L2."""
    import torch
    H, I, reps = 4096, 11008, 3
    blocks = []
    for r in range(reps):
        g = torch.Generator(device=dev).manual_seed(3000 + r)
        norm = ra.TritonRMSNorm(H).to(dev)
        mlp = ra.Int8SwiGLU(H, I).to(dev)
        mlp.quantize_weights(torch.randn(I, H, generator=g, device=dev) * 0.02,
                             torch.randn(I, H, generator=g, device=dev) * 0.02,
                             torch.randn(H, I, generator=g, device=dev) * 0.02)
        for lin in (mlp.w_gate, mlp.w_up, mlp.w_down):
            lin.scale = lin.scale.half()
        blocks.append((norm, mlp))
    out = {}
    for M in (8, 2048):
        xs = [torch.randn(M, H, device=dev).half() for _ in range(reps)]

        def fused():
            for (norm, mlp), x in zip(blocks, xs):
                mlp(norm(x))

        def unfused():
            for (norm, mlp), x in zip(blocks, xs):
                h = norm(x)
                gate = ra.int8_gemm(h, mlp.w_gate.weight_int8, mlp.w_gate.scale)
                up = ra.int8_gemm(h, mlp.w_up.weight_int8, mlp.w_up.scale)
                ra.int8_gemm(torch.nn.functional.silu(gate) * up, mlp.w_down.weight_int8, mlp.w_down.scale)

        # (scaled with --steps, so that a short run stays short under a profiler)
        steps = max(20, min(2000, args.steps // 10)) if M == 8 else max(10, min(100, args.steps // 200))
        res = {}
        for name, fn in (("fused", fused), ("unfused", unfused)):
            gph = capture(fn)
            ms, clk = timed(gph, steps, max(3, args.warmup // 4), sample_clocks=(name == "fused"))
            res[name] = (ms / reps, clk)
            del gph
        us = res["fused"][0] * 1e3
        wbytes = 3 * H * I
        io = 2 * M * H * 2 + 2 * (2 * I + H)            # x in, y out, fp16 scales
        entry = {"us_per_block": round(us, 2), "unfused_us_per_block": round(res["unfused"][0] * 1e3, 2),
                 "launches_per_block": 3 if M <= 32 else 5, "unfused_launches_per_block": 6,
                 "clocks": res["fused"][1]}
        if M == 8:
            tbs = (wbytes + io) / (us * 1e-6) / 1e12
            entry.update({"value": round(tbs, 3), "unit": "TB/s",
                          "roofline": {"bound": "hbm", "achieved": round(tbs * 1e3, 1), "peak": peaks["hbm_gbs"],
                                       "unit": "GB/s", "frac": round(tbs * 1e3 / peaks["hbm_gbs"], 4),
                                       "peak_kind": f"HBM copy ({peaks['source']})"}})
        else:
            tf = 3 * 2 * M * H * I / (us * 1e-6) / 1e12
            entry.update({"value": round(tf, 1), "unit": "TFLOP/s",
                          "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peaks["bf16_tflops"],
                                       "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_tflops"], 4),
                                       "peak_kind": f"dense bf16/fp16 burst ({peaks['source']})"}})
        out[f"M={M}"] = entry
    out["workload"] = ("BASELINE config 3: RMSNorm(4096) -> Int8Linear gate, up 4096->11008 -> SwiGLU -> "
                       "Int8Linear down 11008->4096, random-init weights N(0, 0.02), x ~ N(0, 1) fp16")
    return out


def _sharded_parity(dist, world, x, q, sc, y, prefill):
    """Every rank's assembled output ``y [M, world * n_local]`` against the
    fp32-accumulated dequant-matmul of the full layer (the north star's
    tolerance reference, what rotalabs-accel's CPU route approximates):
    each rank computes its own shard's slice, the slices are all-gathered in
    rank order, and each rank compares its whole assembled row block.
    Decode: every row; M = 4096: the first and last 64 rows.  Returns
    (max abs error, max error / max(1, |ref|)) over all ranks."""
    import torch
    M = x.shape[0]
    rows = torch.cat([torch.arange(0, 64), torch.arange(M - 64, M)]).to(x.device) if prefill else None
    xs = (x if rows is None else x.index_select(0, rows)).float()
    ref_local = xs @ (q.float() * sc.float()[:, None]).t()                      # [m, n_local]
    if world > 1:
        parts = torch.empty((world,) + tuple(ref_local.shape), device=x.device, dtype=torch.float32)
        dist.all_gather_into_tensor(parts, ref_local.contiguous())
        ref = parts.permute(1, 0, 2).reshape(ref_local.shape[0], -1)          # rank-major columns
    else:
        ref = ref_local
    ys = (y if rows is None else y.index_select(0, rows)).float()
    err = (ys - ref).abs()
    out = torch.stack([err.max(), (err / ref.abs().clamp(min=1.0)).max()]).double()
    if world > 1:
        dist.all_reduce(out, op=dist.ReduceOp.MAX)
    return float(out[0]), float(out[1]), int(ref.shape[0])


def measure_sharded(ra, _capi, dist, dev, world, rank, capture, timed, peaks, args, exchange, pexchange=None):
    """Config 4: the Llama-3-70B MLP GEMMs (K=8192 -> N=28672, K=28672 ->
    N=8192) column-parallel over the world's GPUs.  Each rank holds its
    N / world output channels.  Decode (M = 1, 16): the fused peer-exchange
    launch (``--exchange p2p``) or the local GEMM + NCCL all-gather + column
    assembly (``--exchange nccl``); one GPU: the plain GEMM.  A decode step
    runs the GEMM on several copies of the weight shard, together larger than
    3 x L2, so nothing is re-read from L2.  Prefill (M = 4096, one weight
    copy: the GEMM is compute-bound): row blocks of the local tcgen05 GEMM,
    each block pulled from every rank over NVLink by ``PrefillExchange``
    (``--exchange p2p``) or all-gathered with NCCL and reordered
    (``--exchange nccl``) behind the next block's GEMM.  Times are device-side, max over ranks; values are
    whole-job (the full layer's algorithmic bytes or FLOPs / time).

    Every shape's assembled output is checked after its timed replays
    (``parity``), and with N > 1 every rank also times the whole layer on its
    own GPU (``single_gpu_us``, same run, max over ranks), so that the line
    carries the strong-scaling efficiency t1 / (N * tN)."""
    import torch
    from rotalabs_accel_b200.sharded import assemble_columns, prefill_overlapped, shard_range
    out = {"workload": "BASELINE config 4: Llama-3-70B MLP GEMMs (8192->28672, 28672->8192), M in {1, 16, 4096}, "
                       f"column-parallel over {world} GPU(s); weights N(0, 0.02) per-channel int8, fp16 scales",
           "exchange": ("none (one GPU)" if world == 1 else
                        ("decode: peer-to-peer all-gather fused into the decode kernel; "
                         if exchange is not None else "decode: NCCL all-gather + column assembly; ")
                        + ("prefill: blocks of rows; each block's slices pulled from every rank's exchange "
                           "buffer over NVLink into the output's columns on a communication stream, "
                           "overlapping the next block's GEMM" if pexchange is not None else
                           "prefill: blocks of rows, each block's NCCL all-gather and column assembly on a "
                           "communication stream overlapping the next block's GEMM")),
           "scaling": "strong",
           "parity_reference": "fp32-accumulated dequant-matmul of the full layer; tolerance |err| <= "
                               "1e-2 * max(1, |ref|) per element, every rank's assembled output"}
    all_ok = True
    for (K, N) in SHARDED_KN:
        start, stop, n_local = shard_range(N, world, rank)
        assert n_local * world == N, "config 4 shapes split evenly"
        copies = max(1, min(16, math.ceil(3 * L2_BYTES / (n_local * K))))
        shards = []
        for c in range(copies):
            g = torch.Generator(device=dev).manual_seed(7000 + 31 * c + 1009 * rank + K)
            q, sc = ra.quantize_weight_per_channel(torch.randn(n_local, K, generator=g, device=dev) * 0.02)
            shards.append((q, sc.half()))
        torch.cuda.synchronize()
        for M in SHARDED_DECODE_M + (SHARDED_PREFILL_M,):
            prefill = M == SHARDED_PREFILL_M
            use = shards[:1] if prefill else shards
            g = torch.Generator(device=dev).manual_seed(8000 + M + K)
            x = torch.randn(M, K, generator=g, device=dev).half()
            y = torch.empty(M, world * n_local, device=dev, dtype=torch.float16)
            y_local = torch.empty(M, n_local, device=dev, dtype=torch.float16) if world > 1 else y
            staging = torch.empty(world, M, n_local, device=dev, dtype=torch.float16) if world > 1 else None

            def fn():
                for (q, sc) in use:
                    if world == 1:
                        _capi.w8a16_gemm(x, q, sc, None, out=y)
                    elif exchange is not None and not prefill:
                        exchange.gemm(x, q, sc, None, out=y)
                    elif prefill and pexchange is not None:
                        pexchange.gemm(x, q, sc, None, out=y)
                    elif prefill:
                        prefill_overlapped(x, q, sc, None, world * n_local, world, out=y)
                    else:
                        _capi.w8a16_gemm(x, q, sc, None, out=y_local)
                        dist.all_gather_into_tensor(staging, y_local)
                        assemble_columns(staging, N, out=y)

            steps = max(5, args.steps // 2000) if prefill else max(20, args.steps // 100)
            gph = capture(fn)
            ms, _ = timed(gph, steps, args.warmup)
            del gph
            torch.cuda.synchronize()
            # y now holds the output of the last weight copy of the last replay
            abs_err, rel_err, rows_checked = _sharded_parity(dist, world, x, use[-1][0], use[-1][1], y, prefill)
            ok = rel_err <= 1e-2
            all_ok = all_ok and ok
            ms_gemm = ms / len(use)
            key = f"M={M} {K}->{N}"
            entry = {"us": round(ms_gemm * 1e3, 2), "steps": steps,
                     "parity": {"max_abs_err": round(abs_err, 6), "max_err_over_max1_ref": round(rel_err, 6),
                                "rows_checked": rows_checked, "ok": ok}}
            if world > 1:
                # this rank's shard GEMM alone (no exchange), same weights and
                # steps: the exchange's cost is us - local_gemm_us
                def fn_local():
                    for (q, sc) in use:
                        _capi.w8a16_gemm(x, q, sc, None, out=y_local)

                gph = capture(fn_local)
                ms_l, _ = timed(gph, steps, args.warmup)
                del gph
                entry["local_gemm_us"] = round(ms_l / len(use) * 1e3, 2)
            if prefill:
                tf = 2.0 * M * N * K / (ms_gemm * 1e-3) / 1e12
                entry.update({"value": round(tf, 1), "unit": "TFLOP/s",
                              "frac": round(tf / (world * peaks["bf16_tflops"]), 4),
                              "peak": f"{world} x dense bf16/fp16 burst ({peaks['source']})"})
            else:
                tbs = gemm_bytes(M, K, N) / (ms_gemm * 1e-3) / 1e12
                entry.update({"value": round(tbs, 3), "unit": "TB/s",
                              "frac": round(tbs * 1e3 / (world * peaks["hbm_gbs"]), 4),
                              "peak": f"{world} x HBM copy ({peaks['source']})", "weight_copies": len(use)})
            out[key] = entry
            del x, y, y_local, staging
        del shards
        torch.cuda.synchronize()
        if world > 1:
            # The whole layer on each rank's own GPU, for the efficiency t1 / (N * tN).
            copies1 = max(1, min(16, math.ceil(3 * L2_BYTES / (N * K))))
            full = []
            for c in range(copies1):
                g = torch.Generator(device=dev).manual_seed(9000 + 31 * c + K)
                q, sc = ra.quantize_weight_per_channel(torch.randn(N, K, generator=g, device=dev) * 0.02)
                full.append((q, sc.half()))
            for M in SHARDED_DECODE_M + (SHARDED_PREFILL_M,):
                prefill = M == SHARDED_PREFILL_M
                use = full[:1] if prefill else full
                x = torch.randn(M, K, device=dev).half()
                y = torch.empty(M, N, device=dev, dtype=torch.float16)

                def fn1():
                    for (q, sc) in use:
                        _capi.w8a16_gemm(x, q, sc, None, out=y)

                steps = max(5, args.steps // 2000) if prefill else max(20, args.steps // 100)
                gph = capture(fn1)
                ms1, _ = timed(gph, steps, args.warmup)
                del gph
                e = out[f"M={M} {K}->{N}"]
                e["single_gpu_us"] = round(ms1 / len(use) * 1e3, 2)
                e["strong_scaling_eff"] = round((ms1 / len(use)) / (world * e["us"] * 1e-3), 3)
                del x, y
            del full
            torch.cuda.synchronize()
    out["parity_ok"] = all_ok
    return out


def run_case(case: str) -> int:
    """Small fixed workloads for profiler captures (no timing):
    ``sweep`` the 16 decode GEMMs once each; ``decode`` 4 launches of
    M=1, K=4096, N=14336; ``decode-large`` 3 launches of M=1, K=8192,
    N=28672; ``decode-large16`` 2 of M=16 on that shape; ``skinny16`` 3
    launches of the skinny kernel at M=16, K=4096, N=14336; ``prefill`` 2
    launches of M=2048, K=4096, N=11008; ``mlp8`` / ``mlp2048`` 2 gated
    gate/up GEMMs of config 3; ``exchange1`` the 8192 -> 14336 shard at M=1,
    2 plain launches then 2 world-1 fused-exchange launches."""
    import torch
    import rotalabs_accel_b200 as ra
    from rotalabs_accel_b200 import _capi
    dev = torch.device("cuda", 0)

    def prob(M, N, K, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        x = torch.randn(M, K, generator=g, device=dev).half()
        q, s = ra.quantize_weight_per_channel(torch.randn(N, K, generator=g, device=dev) * 0.02)
        return x, q, s.half()

    if case == "sweep":
        ps = [prob(M, N, K, i) for i, (M, K, N) in enumerate(sweep())]
        torch.cuda.synchronize()
        for (x, q, s) in ps:
            _capi.w8a16_gemm(x, q, s, None)
    elif case == "decode":
        x, q, s = prob(1, 14336, 4096, 0)
        for _ in range(4):
            _capi.w8a16_gemm(x, q, s, None)
    elif case == "decode-large":
        x, q, s = prob(1, 28672, 8192, 0)
        for _ in range(3):
            _capi.w8a16_gemm(x, q, s, None)
    elif case == "prefill":
        x, q, s = prob(2048, 11008, 4096, 0)
        for _ in range(2):
            _capi.w8a16_gemm(x, q, s, None)
    elif case == "decode-large16":
        x, q, s = prob(16, 28672, 8192, 0)
        for _ in range(2):
            _capi.w8a16_gemm(x, q, s, None)
    elif case == "skinny16":
        _capi.set_decode_kernel("skinny")
        x, q, s = prob(16, 14336, 4096, 0)
        for _ in range(3):
            _capi.w8a16_gemm(x, q, s, None)
        _capi.set_decode_kernel("auto")
    elif case in ("mlp8", "mlp2048"):
        M = 8 if case == "mlp8" else 2048
        x, qg, sg = prob(M, 11008, 4096, 0)
        _, qu, su = prob(1, 11008, 4096, 1)
        for _ in range(2):
            _capi.w8a16_gemm_swiglu(x, qg, sg, qu, su)
    elif case == "exchange1":
        # the same shard through the plain decode GEMM (2 launches) and the
        # world-1 fused exchange form (2 launches), for a side-by-side capture
        import datetime
        import torch.distributed as dist
        from rotalabs_accel_b200.peer import PeerExchange
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29561")
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
        ex = PeerExchange(max_rows=16, max_n_local=14336)
        x, q, s = prob(1, 14336, 8192, 0)
        y = torch.empty(1, 14336, device=dev, dtype=torch.float16)
        for _ in range(2):
            _capi.w8a16_gemm(x, q, s, None, out=y)
        torch.cuda.synchronize()
        for _ in range(2):
            ex.gemm(x, q, s, None, out=y)
        torch.cuda.synchronize()
        ex.close()
        dist.destroy_process_group()
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()
    err = _capi.device_error()
    print("case", case, "device_error", err)
    return 0 if err == 0 else 1


def run_prefill_timeline() -> int:
    """``--case prefill-timeline`` (under torchrun, one rank per GPU): the
    column-parallel prefill of config 4 (M = 4096, both 70B MLP shapes) with
    the pull exchange, per candidate split of the rows into blocks (the
    block model's pick and fixed ones), eager calls with CUDA events around
    every GEMM block (compute stream) and every pull (communication stream);
    medians of 8 calls, the call total as max over ranks.  Rank 0 prints one
    JSON object."""
    import datetime
    import statistics
    import torch
    import torch.distributed as dist
    import rotalabs_accel_b200 as ra
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PrefillExchange, comm_stream
    from rotalabs_accel_b200.sharded import prefill_row_blocks
    rank, world = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    else:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29563")
        dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    M = SHARDED_PREFILL_M
    pex = PrefillExchange(max_rows=M, max_n_local=max(N for (_, N) in SHARDED_KN) // world)
    out = {"world": world, "M": M}

    def mk(sizes):
        blocks, r = [], 0
        for z in sizes:
            blocks.append((r, z))
            r += z
        return blocks

    for (K, N) in SHARDED_KN:
        nl = N // world
        g = torch.Generator(device=dev).manual_seed(1 + rank)
        q, sc = ra.quantize_weight_per_channel(torch.randn(nl, K, generator=g, device=dev) * 0.02)
        sc = sc.half()
        x = torch.randn(M, K, generator=g, device=dev).half()
        y = torch.empty(M, N, device=dev, dtype=torch.float16)
        xb = pex._xb_flat[:M * nl].view(M, nl)
        cur, comm = torch.cuda.current_stream(dev), comm_stream(dev)
        model = prefill_row_blocks(M, nl, K, world, _capi.device_sm_count(dev.index), "p2p")
        cands = [model, mk([M]), mk([2048, 2048]), mk([3328, 768]), mk([2304, 1280, 512]), mk([1024] * 4),
                 mk([2560, 1536])]
        seen = set()
        for blocks in cands:
            key = tuple(r for _, r in blocks)
            if key in seen:
                continue
            seen.add(key)
            rec = {"total": [], "gemm": [[] for _ in blocks], "pull": [[] for _ in blocks]}
            for it in range(10):
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 + 3 * len(blocks))]
                dist.barrier()
                torch.cuda.synchronize()
                ev[0].record(cur)
                _capi.prefill_exchange_begin(pex._sync.ptrs, rank, cur.cuda_stream)
                for b, (r0, rows) in enumerate(blocks):
                    _capi.w8a16_gemm(x[r0:r0 + rows], q, sc, None, out=xb[r0:r0 + rows])
                    ev[2 + 3 * b].record(cur)
                    comm.wait_event(ev[2 + 3 * b])
                    ev[3 + 3 * b].record(comm)
                    _capi.prefill_exchange_block(pex._xb.ptrs, nl, pex._sync.ptrs, rank, b, b == len(blocks) - 1,
                                                 r0, rows, nl, y, comm.cuda_stream)
                    ev[4 + 3 * b].record(comm)
                cur.wait_stream(comm)
                ev[1].record(cur)
                torch.cuda.synchronize()
                if it < 2:
                    continue
                rec["total"].append(ev[0].elapsed_time(ev[1]) * 1e3)
                prev = ev[0]
                for b in range(len(blocks)):
                    rec["gemm"][b].append(prev.elapsed_time(ev[2 + 3 * b]) * 1e3)
                    prev = ev[2 + 3 * b]
                    rec["pull"][b].append(ev[3 + 3 * b].elapsed_time(ev[4 + 3 * b]) * 1e3)
            t = torch.tensor([statistics.median(rec["total"])], device=dev, dtype=torch.float64)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            out[f"{K}->{N} {list(key)}{' (model)' if blocks == model else ''}"] = {
                "total_us": round(t.item(), 1),
                "gemm_us": [round(statistics.median(v), 1) for v in rec["gemm"]],
                "pull_us": [round(statistics.median(v), 1) for v in rec["pull"]]}
        del q, sc, x, y
        torch.cuda.empty_cache()
    pex.check()
    pex.close()
    if rank == 0:
        print(json.dumps(out))
    dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--exchange", choices=("p2p", "nccl"), default="p2p",
                    help="N > 1: output exchange of the column-parallel config 4 decode GEMMs")
    ap.add_argument("--no-sharded", action="store_true", help="skip the config 4 column-parallel measurement")
    ap.add_argument("--no-mlp", action="store_true", help="skip the config 3 MLP block measurement")
    ap.add_argument("--case", choices=("sweep", "decode", "decode-large", "decode-large16", "skinny16", "prefill",
                                       "mlp8", "mlp2048", "exchange1", "prefill-timeline"),
                    help="run one small fixed workload for a profiler capture and exit (prefill-timeline: the "
                         "per-block event timeline of the column-parallel prefill, under torchrun)")
    args = ap.parse_args()
    if args.case == "prefill-timeline":
        return run_prefill_timeline()
    if args.case:
        return run_case(args.case)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            run_reference(args)
        return 0

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    import rotalabs_accel_b200 as ra
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PeerExchange, PrefillExchange

    peaks = load_peaks()

    # ---- workload: every rank runs the whole sweep on its own batch ----
    # (the same weights on every rank, as replicas of one model; x differs)
    jobs = sweep()
    layers = []
    for i, (M, K, N) in enumerate(jobs):
        g = torch.Generator(device=dev).manual_seed(1000 + i)
        w_full = torch.randn(N, K, generator=g, device=dev) * 0.02
        q, s = ra.quantize_weight_per_channel(w_full)
        del w_full
        gx = torch.Generator(device=dev).manual_seed(1000 + i + 100000 * rank)
        x = torch.randn(M, K, generator=gx, device=dev).half()
        y = torch.empty(M, N, device=dev, dtype=torch.float16)
        layers.append(dict(M=M, K=K, N=N, x=x, q=q, s=s.half(), y=y))
    torch.cuda.synchronize()
    bytes_step = sum(gemm_bytes(M, K, N) for (M, K, N) in jobs)
    p2p = world > 1 and args.exchange == "p2p"
    exchange = pexchange = None

    stream = torch.cuda.Stream(device=dev)

    def step():
        for L in layers:
            _capi.w8a16_gemm(L["x"], L["q"], L["s"], None, out=L["y"])

    def capture(fn):
        with torch.cuda.stream(stream):
            fn()   # warm (allocates the split-K workspace for this stream)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        return g

    def timed(graph, steps, warmup, sample_clocks=False):
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        # The clock sampler starts before the barrier: every rank must begin
        # its timed replays together (a rank that starts late makes the
        # others wait inside their first exchange, inside the timed region).
        sampler = ClockSampler(local_rank) if sample_clocks else None
        if sampler:
            sampler.start()
            time.sleep(0.3)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        clocks = sampler.stop() if sampler else None
        if world > 1:
            dist.barrier()
        ms = e0.elapsed_time(e1) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms, clocks

    launches_per_step = len(layers) * world   # one GEMM kernel per layer on every GPU

    g_step = capture(step)
    ms_step, clocks = timed(g_step, args.steps, args.warmup, sample_clocks=(rank == 0))
    value = world * bytes_step / (ms_step * 1e-3) / 1e12

    # ---- the decode kernel (roofline): every launch of the step is one ----
    avg_launch_us = ms_step * 1e3 / len(layers)
    achieved = bytes_step / len(layers) / (avg_launch_us * 1e-6) / 1e9
    traffic = load_traffic()

    # ---- end to end through the public API, host buffers ----
    torch.cuda.synchronize()
    xs_host = [L["x"].cpu().pin_memory() for L in layers]
    ys_host = [torch.empty(L["M"], L["N"], dtype=torch.float16).pin_memory() for L in layers]
    mods = []
    for L in layers:
        m = ra.Int8Linear(L["K"], L["N"])
        m.weight_int8 = L["q"]
        m.scale = L["s"]
        m._quantized = True
        mods.append(m)
    h2d = sum(t.numel() * 2 for t in xs_host)
    d2h = sum(t.numel() * 2 for t in ys_host)
    # A step's inputs travel in one host -> device copy (one pinned buffer
    # holding every layer's x) and its 16 results come back in one device ->
    # host copy after one gather on the device (each small copy is a separate
    # DMA whose latency would otherwise sit between two GEMMs).  The copies
    # run on a copy stream with two device buffer sets, so that step i+1's
    # input copy and step i's result copy overlap the GEMMs; every step still
    # copies its own inputs in and its own results out inside the timed
    # region.  (Measured per step with the copies serialised on the compute
    # stream: 0.29 ms, against 0.19 ms of device time for the GEMMs.)
    x_host_all = torch.cat([t.flatten() for t in xs_host]).pin_memory()
    n_out = sum(t.numel() for t in ys_host)
    y_host_all = [torch.empty(n_out, dtype=torch.float16).pin_memory() for _ in range(2)]
    bufs = []
    for _ in range(2):
        xd = torch.empty_like(x_host_all, device=dev)
        views, o = [], 0
        for t in xs_host:
            views.append(xd[o:o + t.numel()].view(t.shape))
            o += t.numel()
        bufs.append(dict(x=xd, views=views, y=torch.empty(n_out, dtype=torch.float16, device=dev),
                         x_ready=torch.cuda.Event(), y_ready=torch.cuda.Event(), y_read=torch.cuda.Event()))
    copy_stream = torch.cuda.Stream(device=dev)

    # The step's two copies are issued as plain cudaMemcpyAsync calls on the
    # copy stream (torch's copy_ from pinned memory also records an event in
    # its host allocator per call, tens of microseconds of host time per step
    # on this loop).
    import ctypes
    cudart = None
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            cudart = ctypes.CDLL(name)
            break
        except OSError:
            continue
    cudart.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_void_p]
    cudart.cudaMemcpyAsync.restype = ctypes.c_int
    H2D, D2H = 1, 2
    x_bytes = x_host_all.numel() * 2
    y_bytes = y_host_all[0].numel() * 2
    cs = copy_stream.cuda_stream

    def memcpy(dst, src, n, kind):
        st = cudart.cudaMemcpyAsync(dst, src, n, kind, cs)
        if st != 0:
            raise RuntimeError(f"cudaMemcpyAsync failed with status {st}")

    def e2e_run(steps, timed_events=None):
        """`steps` steps through the public API.  The compute stream stays
        current; each step has its read-back and the input copy of step i+2
        on the copy stream, into the buffer set step i has finished with
        (steps 0 and 1 copy theirs first).  Every step's input and result
        copies are inside the region."""
        with torch.cuda.stream(stream):
            if timed_events:
                timed_events[0].record(stream)
            copy_stream.wait_stream(stream)
            for j in range(min(2, steps)):
                memcpy(bufs[j]["x"].data_ptr(), x_host_all.data_ptr(), x_bytes, H2D)
                bufs[j]["x_ready"].record(copy_stream)
            for i in range(steps):
                bf = bufs[i % 2]
                stream.wait_event(bf["x_ready"])
                outs = [m(xd).view(-1) for m, xd in zip(mods, bf["views"])]
                torch.cat(outs, out=bf["y"])
                bf["y_ready"].record(stream)
                copy_stream.wait_event(bf["y_ready"])
                memcpy(y_host_all[i % 2].data_ptr(), bf["y"].data_ptr(), y_bytes, D2H)
                if i + 2 < steps:
                    memcpy(bf["x"].data_ptr(), x_host_all.data_ptr(), x_bytes, H2D)
                    bf["x_ready"].record(copy_stream)
            stream.wait_stream(copy_stream)
            if timed_events:
                timed_events[1].record(stream)

    e2e_run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2e_run(args.e2e_steps, (e0, e1))
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = t.item()
    e2e_value = world * bytes_step / (ms_e2e * 1e-3) / 1e12

    # ---- prefill (N = 1) ----
    prefill = None
    if world == 1 and not args.no_prefill:
        pl = []
        for i, (K, N) in enumerate(PREFILL_KN):
            g = torch.Generator(device=dev).manual_seed(2000 + i)
            x = torch.randn(PREFILL_M, K, generator=g, device=dev).half()
            q, s = ra.quantize_weight_per_channel(torch.randn(N, K, generator=g, device=dev) * 0.02)
            pl.append((x, q, s.half(), torch.empty(PREFILL_M, N, device=dev, dtype=torch.float16)))

        def pstep():
            for (x, q, s, y) in pl:
                _capi.w8a16_gemm(x, q, s, None, out=y)
        g_pre = capture(pstep)
        pre_steps = max(20, args.steps // 10)
        ms_pre, pclocks = timed(g_pre, pre_steps, args.warmup, sample_clocks=(rank == 0))
        flops = sum(2 * PREFILL_M * N * K for (K, N) in PREFILL_KN)
        tflops = flops / (ms_pre * 1e-3) / 1e12
        prefill = {"value": round(tflops, 2), "unit": "TFLOP/s", "ms_per_step": round(ms_pre, 4),
                   "steps": pre_steps, "gemms": [f"{PREFILL_M}x{K}->{N}" for (K, N) in PREFILL_KN],
                   "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": peaks["bf16_tflops"],
                                "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4),
                                "peak_kind": f"dense bf16/fp16 burst ({peaks['source']})",
                                "traffic": load_traffic("prefill_traffic.json"),
                                "traffic_launch": "M=2048, K=4096, N=11008, w8a16_tc_kernel<256, 4>"},
                   "clocks": pclocks}
        del g_pre

    # ---- config 3: the MLP block (N = 1) ----
    mlp_block = None
    if world == 1 and not args.no_mlp:
        mlp_block = measure_mlp_block(ra, _capi, dev, capture, timed, peaks, args)

    # ---- config 4: the 70B MLP GEMMs, column-parallel over the GPUs ----
    sharded = None
    if not args.no_sharded:
        nl_max = max(-(-N // world) for (_, N) in SHARDED_KN)
        exchange = PeerExchange(max_rows=max(SHARDED_DECODE_M), max_n_local=nl_max) if p2p else None
        pexchange = PrefillExchange(max_rows=SHARDED_PREFILL_M, max_n_local=nl_max) if p2p else None
        sharded = measure_sharded(ra, _capi, dist, dev, world, rank, capture, timed, peaks, args, exchange,
                                  pexchange)

    # ---- CPU baseline (rank 0, N = 1) ----
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        threads = cpu_threads()
        probs = [(L["x"].cpu(), L["q"].cpu(), L["s"].cpu()) for L in layers]   # the GPU arm's own inputs
        time_cpu_gemms(probs[:1], threads)                                    # warm torch's thread pool
        t_cpu = time_cpu_gemms(probs, threads)
        del probs
        cpu = {"value": round(bytes_step / t_cpu / 1e12, 6), "unit": "TB/s", "cores": threads, "kind": "port",
               "sample": f"one pass of the 16-GEMM decode sweep on the GPU arm's inputs ({t_cpu:.2f} s); "
                         + REF_SAMPLE_DESC}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (int8 weights, fp32 accumulate)",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) per-channel int8 weights)",
            "config": {"workload": "decode GEMV sweep, BASELINE config 1: M in {1,4,8,16} x (K,N) in "
                                   "{(4096,4096),(4096,11008),(11008,4096),(4096,14336)}, 16 GEMMs per step",
                       "parallelism": "single GPU" if world == 1 else
                       f"{world} replicas (data-parallel decode: every GPU runs the whole sweep on its own batch, "
                       "no collective); column-parallel sharding is measured on config 4 (the sharded object)",
                       "weights_bytes_per_gpu": sum(L["q"].numel() for L in layers),
                       "l2": "working set > L2: each GEMM has its own weight (663 MB total), no L2 reuse",
                       "timing": "CUDA graph of one step, K replays between CUDA events"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "peak_kind": f"HBM copy ({peaks['source']})",
                         "kernel": "decode kernels per the selector: w8a16_skinny_kernel (every GEMM of this "
                                   "sweep; split-K inside thread-block clusters) and w8a16_stream_kernel "
                                   "(persistent stream-K TMA, layers of 120 MB and more)",
                         "avg_launch_us": round(avg_launch_us, 3), "traffic": traffic},
            "e2e": {"value": round(e2e_value, 4), "unit": "TB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 4),
                    "path": "Int8Linear.forward (public API), eager; per step one pinned host -> device copy "
                            "of all 16 inputs, and all 16 outputs read back in one device -> pinned host copy; "
                            "copies on a copy stream with two device buffer sets (a step's inputs are copied two "
                            "steps ahead, its results read back right after it; both overlap other steps' GEMMs)"
                            + ("" if world == 1 else "; on every GPU, max over ranks")},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if prefill:
            line["prefill"] = prefill
        if mlp_block:
            line["mlp_block"] = mlp_block
        if sharded:
            line["sharded"] = sharded
        print(json.dumps(line), flush=True)

    del g_step
    torch.cuda.synchronize()
    if exchange is not None:
        exchange.close()
    if pexchange is not None:
        pexchange.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
