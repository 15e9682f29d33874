"""The fused peer-to-peer all-gather (rla_w8a16_gemm_allgather) on the GPU.

One GPU:
  * world = 1 (a single-rank gloo group): the fused kernel's output equals the
    plain decode GEMM within the suite's tolerance, for both decode kernels,
    and the call counter advances once per call, also under CUDA-graph
    replay.  (The fused launch is planned with the exchange kernel's own
    occupancy, so its split of K, and with it the fp32 summation order, can
    differ from the plain GEMM's.)
  * failure detection without a fault: a two-rank call whose second "rank"
    never sends anything makes the bounded wait give up (short limit), the
    kernel returns, the device error word reads 7 ("a peer's slice did not
    arrive") and the context stays usable.
  * the prefill pull exchange (PrefillExchange) at world = 1: y equals the
    plain GEMM of the same row blocks bit for bit, eagerly and under graph
    replay; and a two-rank call whose second "rank" never marks its block
    gives up after a short limit with device error 7, then 9 on the next
    call, without a fault.
Two or more GPUs (skipped otherwise): one process per GPU over NCCL, the
column-parallel layer's fused path equals its NCCL path and the fp32
reference within tolerance, call after call, for every decode kernel,
with several layers sharing one exchange and under graph replay; the
prefill pull exchange and the NCCL-overlapped prefill against the fp32
reference, the pull also under graph replay with ragged blocks.
"""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(1, 4096, 4096), (4, 1376, 4096), (8, 2048, 11008), (16, 7168, 4096), (3, 100, 96), (32, 512, 256),
          (5, 7168, 4096)]
# The 70B MLP shards at 2 and 8 ranks (their exchange plans: the one-tile
# 128-thread form with its own register budget, the long-K plan of narrow
# shards, the two-tile form with out-of-line unpacking).
SHARD_SHAPES = [(1, 14336, 8192), (8, 4096, 28672), (1, 3584, 8192), (8, 1024, 28672), (16, 3584, 8192),
                (16, 1024, 28672)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.fixture(scope="module")
def single_rank_group(cuda_lib):
    import torch.distributed as dist
    if dist.is_initialized():
        yield None
        return
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("gloo", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60))
    yield None
    dist.destroy_process_group()


def _problem(M, N, K, seed, bias=False):
    from rotalabs_accel_b200 import quantize_weight_per_channel
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    q, s = quantize_weight_per_channel(torch.randn(N, K, generator=g, device="cuda") * 0.02)
    b = (torch.randn(N, generator=g, device="cuda") * 0.1).half() if bias else None
    return x, q, s.half(), b


def _close(a, b):
    """Within the suite's bar: max |a - b| <= 1e-2 * max(1, max |b|)."""
    a, b = a.float(), b.float()
    return float((a - b).abs().max()) <= 1e-2 * max(1.0, float(b.abs().max()))


@pytest.mark.parametrize("kernel", ["skinny", "stream", "auto"])
def test_world1_fused_equals_plain(single_rank_group, kernel):
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PeerExchange
    _capi.set_decode_kernel(kernel)
    ex = PeerExchange(max_rows=32, max_n_local=14336)
    try:
        calls0 = ex.calls_completed()
        n_calls = 0
        for i, (M, N, K) in enumerate(SHAPES + (SHARD_SHAPES if kernel == "auto" else [])):
            x, q, s, b = _problem(M, N, K, 100 + i, bias=(i % 2 == 1))
            ref = _capi.w8a16_gemm(x, q, s, b)
            out = torch.full((M, N + 8), float("nan"), dtype=torch.float16, device="cuda")   # ldy > N
            for _ in range(3):
                y = ex.gemm(x, q, s, b, out=out)
                n_calls += 1
            torch.cuda.synchronize()
            assert _close(y[:, :N], ref), (M, N, K)
            assert torch.isnan(out[:, N:].float()).all()     # nothing written past the slices
        assert _capi.device_error() == 0
        assert ex.calls_completed() == calls0 + n_calls
    finally:
        ex.close()
        _capi.set_decode_kernel("auto")


def test_world1_fused_cluster_grid_at_residency_estimate(single_rank_group):
    """A skinny exchange launch whose row blocks (74 of 16 rows) times its
    cluster split of K would fill the per-SM residency estimate exactly
    (74 x 8 = 592 CTAs at 4 per SM): its plan counts residency in whole
    clusters, so the grid it launches fits at once and every wait ends
    (no device error)."""
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PeerExchange
    _capi.set_decode_kernel("skinny")
    ex = PeerExchange(max_rows=32, max_n_local=8192)
    try:
        for M, N, K in ((1, 74 * 16, 8192), (4, 74 * 16, 16384), (1, 37 * 16, 28672)):
            x, q, s, b = _problem(M, N, K, 300 + M)
            ref = _capi.w8a16_gemm(x, q, s, b)
            for _ in range(3):
                y = ex.gemm(x, q, s, b)
            torch.cuda.synchronize()
            assert _close(y, ref), (M, N, K)
        assert _capi.device_error() == 0
    finally:
        ex.close()
        _capi.set_decode_kernel("auto")


def test_world1_fused_under_graph_replay(single_rank_group):
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PeerExchange
    ex = PeerExchange(max_rows=16, max_n_local=8192)
    try:
        probs = [_problem(M, N, K, 200 + i) for i, (M, N, K) in enumerate(SHAPES[:4])]
        outs = [torch.empty(p[0].shape[0], p[1].shape[0], dtype=torch.float16, device="cuda") for p in probs]
        refs = [_capi.w8a16_gemm(x, q, s, b) for (x, q, s, b) in probs]
        torch.cuda.synchronize()
        stream = torch.cuda.Stream()

        def step():
            for (x, q, s, b), o in zip(probs, outs):
                ex.gemm(x, q, s, b, out=o)

        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        for o in outs:
            o.zero_()
        calls0 = ex.calls_completed()
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        assert ex.calls_completed() == calls0 + 5 * len(probs)
        for o, r in zip(outs, refs):
            assert _close(o, r)
        assert _capi.device_error() == 0
        del g
    finally:
        ex.close()


@pytest.mark.parametrize("kernel", ["skinny", "stream"])
def test_missing_peer_times_out_with_error_status(single_rank_group, kernel):
    """A two-rank call whose second "rank" is a local buffer that no kernel
    ever fills: the wait for its slice runs out (50 ms), the kernel returns,
    the error word says which wait gave up, and the context stays usable."""
    from rotalabs_accel_b200 import _capi
    _capi.set_decode_kernel(kernel)
    bufs = []
    try:
        _capi.set_peer_wait_limit(0.05)
        M, N, K = 1, 1024, 4096
        x, q, s, _ = _problem(M, N, K, 300)
        recv_bytes = 16 * 2 * 1 * N
        bufs = [_capi.peer_alloc(recv_bytes) for _ in range(2)]
        sync = torch.zeros(_capi.PEER_SYNC_BYTES // 4, dtype=torch.int32, device="cuda")
        out = torch.zeros(M, 2 * N, dtype=torch.float16, device="cuda")
        assert _capi.device_error() == 0
        _capi.w8a16_gemm_allgather(x, q, s, None, out, bufs, recv_bytes, sync.data_ptr(), 0)
        torch.cuda.synchronize()
        assert _capi.device_error() == 7
        # This rank's own slice is complete; the missing peer's columns are not.
        ref = _capi.w8a16_gemm(x, q, s, None)
        torch.cuda.synchronize()
        assert _close(out[:, :N], ref)
        assert _capi.device_error() == 0
    finally:
        _capi.set_peer_wait_limit(1.0)
        _capi.set_decode_kernel("auto")
        torch.cuda.synchronize()
        for p in bufs:
            _capi.peer_free(p)


def _px_blocks(M):
    """Uneven row blocks (the last ragged) for the pull-exchange tests."""
    if M <= 256:
        return [(0, M)]
    a = (M // 3) // 128 * 128 or 128
    return [(0, a), (a, 128), (a + 128, M - a - 128)] if M - a - 128 > 0 else [(0, a), (a, M - a)]


@pytest.mark.parametrize("M,K,N", [(1024, 4096, 4096), (300, 1024, 1000), (517, 2048, 2048), (64, 512, 256)])
def test_world1_prefill_pull_equals_plain(single_rank_group, M, K, N):
    """A single-rank pull exchange: the GEMM of every row block goes through
    the exchange buffer, the pull copies it into y; y equals the plain GEMM
    of the same row blocks bit for bit, and the call number advances once
    per call (eager and under CUDA-graph replay)."""
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PrefillExchange
    ex = PrefillExchange(max_rows=1024, max_n_local=4096)
    try:
        x, q, s, b = _problem(M, N, K, 400 + M, bias=True)
        blocks = _px_blocks(M)
        ref = torch.cat([_capi.w8a16_gemm(x[r0:r0 + r], q, s, b) for r0, r in blocks])
        y = ex.gemm(x, q, s, b, blocks=blocks)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
        assert ex.calls_started() == 1
        out = torch.zeros_like(ref)
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            ex.gemm(x, q, s, b, out=out, blocks=blocks)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            ex.gemm(x, q, s, b, out=out, blocks=blocks)
        out.zero_()
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        assert ex.calls_started() == 7
        assert _capi.device_error() == 0
        ex.check()
        del g
    finally:
        ex.close()


def test_prefill_pull_missing_peer_times_out_with_error_status(single_rank_group):
    """A two-rank pull whose second "rank" is a pair of local buffers that no
    kernel ever marks: the wait for its block runs out (50 ms), the kernel
    returns, the error word reads 7, the sync area keeps the mark, the next
    call records 9 and returns at once, and the context stays usable."""
    from rotalabs_accel_b200 import _capi
    bufs = []
    try:
        _capi.set_peer_wait_limit(0.05)
        M, N, K = 256, 1024, 2048
        x, q, s, _ = _problem(M, N, K, 500)
        bufs = [_capi.peer_alloc(M * N * 2) for _ in range(2)] + [_capi.peer_alloc(_capi.PX_SYNC_BYTES)
                                                                    for _ in range(2)]
        xbs, syncs = bufs[:2], bufs[2:]
        from rotalabs_accel_b200.peer import _device_view
        xb = _device_view(xbs[0], (M, N), torch.float16, torch.device("cuda"))
        words = _device_view(syncs[0], (_capi.PX_SYNC_BYTES // 4,), torch.int32, torch.device("cuda"))
        out = torch.zeros(M, 2 * N, dtype=torch.float16, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        assert _capi.device_error() == 0
        _capi.prefill_exchange_begin(syncs, 0, stream)
        _capi.w8a16_gemm(x, q, s, None, out=xb)
        _capi.prefill_exchange_block(xbs, N, syncs, 0, 0, True, 0, M, N, out, stream)
        torch.cuda.synchronize()
        assert _capi.device_error() == 7
        assert int(words[_capi.PX_SYNC_ABORT_WORD]) == 1
        # this rank's own slice arrived; the missing peer's columns did not
        assert torch.equal(out[:, :N], _capi.w8a16_gemm(x, q, s, None))
        assert int(out[:, N:].abs().max()) == 0
        _capi.prefill_exchange_begin(syncs, 0, stream)
        _capi.prefill_exchange_block(xbs, N, syncs, 0, 0, True, 0, M, N, out, stream)
        torch.cuda.synchronize()
        assert _capi.device_error() == 9
        assert int(words[0]) == 1          # the poisoned call did not advance the call number
        ref = _capi.w8a16_gemm(x, q, s, None)
        torch.cuda.synchronize()
        assert ref.abs().max() > 0 and _capi.device_error() == 0
    finally:
        _capi.set_peer_wait_limit(1.0)
        torch.cuda.synchronize()
        for p in bufs:
            _capi.peer_free(p)


# --------------------------------------------------------------------------
# two or more GPUs
# --------------------------------------------------------------------------

def _worker_multi(rank, world, port, q):
    try:
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from rotalabs_accel_b200 import _capi, int8_gemm_torch, quantize_weight_per_channel
        from rotalabs_accel_b200.peer import PeerExchange
        from rotalabs_accel_b200.sharded import ColumnParallelInt8Linear
        ex = PeerExchange(max_rows=16, max_n_local=-(-28672 // world))
        report = []
        ok = True
        for kernel in ("auto", "skinny", "stream"):
            _capi.set_decode_kernel(kernel)
            for i, (M, K, N, bias) in enumerate([(1, 4096, 14336, False), (4, 4096, 4096, True),
                                                 (16, 11008, 4096, False), (7, 96, 100, True)]):
                g = torch.Generator().manual_seed(10 + i)
                W = torch.randn(N, K, generator=g) * 0.02
                b = (torch.randn(N, generator=g) * 0.1).half() if bias else None
                m_nccl = ColumnParallelInt8Linear(K, N, bias=bias).to(dev)
                m_nccl.quantize_weights(W.to(dev))
                if bias:
                    m_nccl.bias.data[: m_nccl.stop - m_nccl.start].copy_(b[m_nccl.start:m_nccl.stop])
                m_p2p = ColumnParallelInt8Linear(K, N, bias=bias).to(dev)
                m_p2p.load_state_dict(m_nccl.state_dict())
                m_p2p._quantized = True
                m_p2p.enable_peer_exchange(max_tokens=16, exchange=ex)
                wq, s = quantize_weight_per_channel(W)
                for it in range(4):
                    x = torch.randn(M, K, generator=g).half()
                    y_nccl = m_nccl(x.to(dev))
                    y_p2p = m_p2p(x.to(dev))
                    torch.cuda.synchronize()
                    # The fused launch is planned with the exchange kernel's own
                    # occupancy, so its split of K (and thus the fp32 summation
                    # order) can differ from the local GEMM's: compare within the
                    # suite's tolerance, not bit for bit.
                    diff = float((y_p2p.float() - y_nccl.float()).abs().max())
                    same = diff <= 1e-2 * max(1.0, float(y_nccl.float().abs().max()))
                    ref = int8_gemm_torch(x.float(), wq, s, b.float() if b is not None else None)
                    err = float((y_p2p.float().cpu() - ref).abs().max())
                    if not same or err > 1e-2 * max(1.0, float(ref.abs().max())):
                        ok = False
                        report.append((kernel, M, K, N, it, same, err))
        _capi.set_decode_kernel("auto")
        # The benchmark's config 4 shards (Llama-3-70B MLP GEMMs, column-parallel
        # over the world): the fused exchange and the NCCL path both against the
        # fp32 dequant-matmul of the full layer.  The full weight is made on
        # every rank's device from the same seed.
        for (M, K, N) in [(1, 8192, 28672), (16, 8192, 28672), (1, 28672, 8192), (16, 28672, 8192)]:
            g = torch.Generator(device=dev).manual_seed(70 + M + K)
            W = torch.randn(N, K, generator=g, device=dev) * 0.02
            m_nccl = ColumnParallelInt8Linear(K, N).to(dev)
            m_nccl.quantize_weights(W)
            m_p2p = ColumnParallelInt8Linear(K, N).to(dev)
            m_p2p.load_state_dict(m_nccl.state_dict())
            m_p2p._quantized = True
            m_p2p.enable_peer_exchange(max_tokens=16, exchange=ex)
            wq, s = quantize_weight_per_channel(W)
            del W
            for it in range(2):
                x = torch.randn(M, K, generator=g, device=dev).half()
                y_p2p = m_p2p(x)
                y_nccl = m_nccl(x)
                ref = x.float() @ (wq.float() * s.float()[:, None]).t()
                torch.cuda.synchronize()
                tol = 1e-2 * max(1.0, float(ref.abs().max()))
                e_p2p = float((y_p2p.float() - ref).abs().max())
                e_nccl = float((y_nccl.float() - ref).abs().max())
                if e_p2p > tol or e_nccl > tol:
                    ok = False
                    report.append(("config4", M, K, N, it, e_p2p, e_nccl))
            del m_nccl, m_p2p, wq, s
            torch.cuda.empty_cache()
        # Long prefill blocks take the overlapped path (row blocks, each block's
        # all-gather on a communication stream behind the next block's GEMM).
        for (M, K, N) in [(1024, 8192, 28672), (2048, 28672, 8192)]:
            g = torch.Generator(device=dev).manual_seed(90 + K)
            W = torch.randn(N, K, generator=g, device=dev) * 0.02
            m = ColumnParallelInt8Linear(K, N).to(dev)
            m.quantize_weights(W)
            wq, s = quantize_weight_per_channel(W)
            del W
            x = torch.randn(M, K, generator=g, device=dev).half()
            y = m(x)
            ref = x.float() @ (wq.float() * s.float()[:, None]).t()
            torch.cuda.synchronize()
            err = float((y.float() - ref).abs().max())
            if err > 1e-2 * max(1.0, float(ref.abs().max())):
                ok = False
                report.append(("prefill overlapped", M, K, N, err))
            del m, wq, s, x, y, ref
            torch.cuda.empty_cache()
        # The pull exchange (PrefillExchange): every rank's assembled output
        # against the fp32 reference, eagerly and under CUDA-graph replay, with
        # the model's row blocks and with ragged ones.
        from rotalabs_accel_b200.peer import PrefillExchange
        pex = PrefillExchange(max_rows=2048, max_n_local=-(-28672 // world))
        for (M, K, N) in [(1024, 8192, 28672), (2048, 28672, 8192), (333, 4096, 4096)]:
            g = torch.Generator(device=dev).manual_seed(110 + K + M)
            W = torch.randn(N, K, generator=g, device=dev) * 0.02
            m = ColumnParallelInt8Linear(K, N).to(dev)
            m.quantize_weights(W)
            m.enable_peer_exchange(max_tokens=16, exchange=ex, prefill_exchange=pex)
            wq, s = quantize_weight_per_channel(W)
            del W
            x = torch.randn(M, K, generator=g, device=dev).half()
            ref = x.float() @ (wq.float() * s.float()[:, None]).t()
            tol = 1e-2 * max(1.0, float(ref.abs().max()))
            y = m(x)
            torch.cuda.synchronize()
            if float((y.float() - ref).abs().max()) > tol:
                ok = False
                report.append(("prefill pull", M, K, N, float((y.float() - ref).abs().max())))
            out = torch.zeros(M, N, dtype=torch.float16, device=dev)
            ragged = [(0, 128), (128, M - 128)] if M > 128 else [(0, M)]
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                pex.gemm(x, m.weight_int8, m.scale, None, out=out, blocks=ragged)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                pex.gemm(x, m.weight_int8, m.scale, None, out=out, blocks=ragged)
            out.zero_()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            if float((out.float() - ref).abs().max()) > tol:
                ok = False
                report.append(("prefill pull graph", M, K, N, float((out.float() - ref).abs().max())))
            del graph, m, wq, s, x, y, ref, out
            torch.cuda.empty_cache()
        pex.check()
        pex.close()
        # graph replay of several layers sharing the exchange
        layers = []
        for i, (M, K, N) in enumerate([(1, 4096, 4096), (8, 4096, 11008), (16, 4096, 14336)]):
            g = torch.Generator(device=dev).manual_seed(50 + i)
            x = torch.randn(M, K, generator=g, device=dev).half()
            m = ColumnParallelInt8Linear(K, N).to(dev)
            m.quantize_weights((torch.randn(N, K, generator=torch.Generator().manual_seed(60 + i)) * 0.02).to(dev))
            out = torch.empty(M, world * m.n_local, dtype=torch.float16, device=dev)
            layers.append((x, m, out))
        refs = [m(x) for (x, m, _) in layers]       # NCCL path
        torch.cuda.synchronize()
        stream = torch.cuda.Stream()

        def step():
            for (x, m, out) in layers:
                ex.gemm(x, m.weight_int8, m.scale, None, out=out)

        with torch.cuda.stream(stream):
            step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(20):
            graph.replay()
        torch.cuda.synchronize()
        for (x, m, out), r in zip(layers, refs):
            if float((out[:, :m.out_features].float() - r.float()).abs().max()) > 1e-2 * max(1.0, float(r.float().abs().max())):
                ok = False
                report.append(("graph", x.shape[0], m.in_features, m.out_features))
        del graph
        err_word = _capi.device_error()
        if err_word != 0:
            ok = False
            report.append(("device error", err_word))
        ex.close()
        dist.destroy_process_group()
        q.put((rank, ok, report))
    except Exception as e:  # report, never hang the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_fused_equals_nccl_path(cuda_lib, world):
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_multi, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in range(world):
            res.append(q.get(timeout=600))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    res.sort(key=lambda r: r[0])
    assert all(r[1] for r in res), res
