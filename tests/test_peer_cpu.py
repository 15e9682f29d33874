"""Host side of the peer-to-peer output exchange, on CPU only.

The exchange's set-up is collective: the IPC handles travel through one
all-gather of a few bytes over the process group (gloo ranks here).  The C
ABI rejects bad arguments before touching a GPU.  Nothing here launches a
kernel.
"""

import ctypes
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker_blobs(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from rotalabs_accel_b200.peer import exchange_blobs
        blob = bytes([rank]) * 64 + b"end" + bytes([255 - rank])
        got = exchange_blobs(blob, None)
        want = [bytes([r]) * 64 + b"end" + bytes([255 - r]) for r in range(world)]
        q.put((rank, got == want, [len(b) for b in got]))
        dist.destroy_process_group()
    except Exception as e:  # report, never hang the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_blobs_rank_order(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_blobs, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=120) for _ in range(world)), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert all(r[1] for r in res), res


def test_receive_buffer_size():
    from rotalabs_accel_b200.peer import receive_bytes
    # two parity halves x world slots x ceil(M/2) pairs x n_local columns x 8 bytes
    assert receive_bytes(2, 16, 7168) == 2 * 2 * 8 * 7168 * 8
    assert receive_bytes(8, 1, 512) == 2 * 8 * 1 * 512 * 8
    assert receive_bytes(4, 3, 100) == 2 * 4 * 2 * 100 * 8


@pytest.fixture(scope="module")
def lib():
    from rotalabs_accel_b200 import build, _capi
    build.build()
    return _capi.load_library()


def _arr(vals):
    return (ctypes.c_void_p * len(vals))(*vals)


def test_allgather_rejects_bad_arguments(lib):
    from rotalabs_accel_b200 import _capi
    fake = 1 << 20          # never dereferenced: every call below fails validation first
    recv = _arr([fake, fake + 65536])
    enough = 16 * 2 * 1 * 128

    def st(**kw):
        a = dict(x=fake, ldx=64, w=fake, ldw=64, scale=fake, sdt=_capi.DTYPE_F16, bias=None, bdt=0, y=fake, ldy=256,
                 M=1, nl=128, K=64, recv=recv, rb=enough, sync=fake, rank=0, world=2, ws=None, wsb=0)
        a.update(kw)
        return lib.rla_w8a16_gemm_allgather(a["x"], a["ldx"], a["w"], a["ldw"], a["scale"], a["sdt"], a["bias"],
                                            a["bdt"], a["y"], a["ldy"], a["M"], a["nl"], a["K"], a["recv"], a["rb"],
                                            a["sync"], a["rank"], a["world"], a["ws"], a["wsb"], None)

    assert st(world=0) == 1
    assert st(world=9) == 1
    assert st(rank=2) == 1
    assert st(rank=-1) == 1
    assert st(recv=None) == 1
    assert st(recv=_arr([fake, 0])) == 1               # a null receive buffer
    assert st(recv=_arr([fake, fake + 8])) == 1        # a misaligned receive buffer
    assert st(sync=fake + 64) == 1                     # a misaligned sync area
    assert st(y=None) == 1
    assert st(sdt=_capi.DTYPE_BF16) == 1
    assert st(bdt=_capi.DTYPE_F16) == 1                # bias dtype without a bias
    assert st(ldy=200) == 1                            # ldy < world * n_local
    assert st(ldx=32) == 1
    assert st(ws=fake + 16, wsb=4096) == 4             # workspace not 256-byte aligned
    assert st(M=33) == 2                               # not a decode shape: the caller uses NCCL
    assert st(M=0) == 2
    assert st(K=72, ldx=72, ldw=72) == 2               # K % 16 != 0
    assert st(x=fake + 2) == 2                         # x not 16-byte aligned
    assert b"decode" in lib.rla_last_error()
    assert st(M=3, rb=enough) == 4                     # 2 pairs of rows need twice the buffer
    assert b"receive buffers" in lib.rla_last_error()


def test_peer_wait_limit_range(lib):
    assert lib.rla_set_peer_wait_limit(0) == 1
    assert lib.rla_set_peer_wait_limit(61 * 10**9) == 1
    assert lib.rla_set_peer_wait_limit(10**6) == 0
    assert lib.rla_set_peer_wait_limit(10**9) == 0     # back to the default


def test_peer_alloc_and_ipc_reject_null(lib):
    assert lib.rla_peer_alloc(0, None) == 1
    assert lib.rla_ipc_export(None, None) == 1
    assert lib.rla_ipc_open(None, None) == 1
    assert lib.rla_peer_free(None) == 0                # freeing nothing is fine
    assert lib.rla_ipc_close(None) == 0


def test_exchange_needs_a_process_group():
    from rotalabs_accel_b200.peer import PeerExchange
    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    with pytest.raises(RuntimeError, match="process group"):
        PeerExchange()


def test_layer_refuses_peer_exchange_on_cpu():
    from rotalabs_accel_b200.sharded import ColumnParallelInt8Linear
    m = ColumnParallelInt8Linear(64, 32)
    with pytest.raises(RuntimeError, match="GPU"):
        m.enable_peer_exchange(max_tokens=4)
    with pytest.raises(ValueError):
        m.enable_peer_exchange(max_tokens=64)


def test_exchange_refuses_calls_after_a_failed_wait():
    """Once a wait of an exchange call has given up (the abort word of the
    sync area is set), check() raises and gemm() refuses every later call
    until the exchange is set up again.  Host logic only: the exchange object
    is assembled by hand around a CPU sync area."""
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PeerExchange
    ex = PeerExchange.__new__(PeerExchange)
    ex._recv = object()                    # "open"
    ex._failed = None
    ex.max_rows, ex.max_n_local = 16, 128
    ex._sync = torch.zeros(_capi.PEER_SYNC_BYTES // 4, dtype=torch.int32)
    ex.check()                             # a clean sync area passes
    ex._sync[_capi.PEER_SYNC_ABORT_WORD] = 5
    with pytest.raises(RuntimeError, match="call 5 gave up"):
        ex.check()
    x = torch.zeros(1, 64, dtype=torch.float16)
    w = torch.zeros(128, 64, dtype=torch.int8)
    s = torch.ones(128, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="set up a new one"):
        ex.gemm(x, w, s)
    ex._sync[_capi.PEER_SYNC_ABORT_WORD] = 0  # the mark stays on the host side too
    with pytest.raises(RuntimeError, match="PeerExchange failed"):
        ex.check()


def test_prefill_exchange_rejects_bad_arguments(lib):
    """rla_prefill_exchange_begin / _block validate everything before any
    launch (no device is touched by these calls)."""
    fake = 1 << 20
    syncs = _arr([fake, fake + 4096])
    xbs = _arr([fake, fake + (1 << 24)])

    def blk(**kw):
        a = dict(xb=xbs, ld=128, sync=syncs, rank=0, world=2, block=0, last=1, row0=0, rows=256, nl=128, y=fake,
                 ldy=256)
        a.update(kw)
        return lib.rla_prefill_exchange_block(a["xb"], a["ld"], a["sync"], a["rank"], a["world"], a["block"],
                                              a["last"], a["row0"], a["rows"], a["nl"], a["y"], a["ldy"], None)

    assert lib.rla_prefill_exchange_begin(syncs, 0, 0, None) == 1
    assert lib.rla_prefill_exchange_begin(syncs, 2, 2, None) == 1
    assert lib.rla_prefill_exchange_begin(None, 0, 2, None) == 1
    assert lib.rla_prefill_exchange_begin(_arr([fake, fake + 64]), 0, 2, None) == 1   # sync not 128-byte aligned
    assert blk(world=9) == 1
    assert blk(rank=-1) == 1
    assert blk(xb=None) == 1
    assert blk(xb=_arr([fake, fake + 8])) == 1          # exchange buffer not 16-byte aligned
    assert blk(sync=_arr([fake, 0])) == 1
    assert blk(y=fake + 8) == 1
    assert blk(block=16) == 1                           # at most RLA_PX_MAX_BLOCKS blocks
    assert blk(block=-1) == 1
    assert blk(nl=100, ld=100, ldy=200) == 1            # n_local not a multiple of 8
    assert blk(ld=64) == 1                              # ld_xb < n_local
    assert blk(ldy=255) == 1                            # ldy < world * n_local
    assert blk(rows=-1) == 1
    assert blk(rows=1 << 31) == 1                       # rows >= 2^31
    assert b"2^31" in lib.rla_last_error()


def test_prefill_exchange_refuses_calls_after_a_failed_wait():
    """The pull exchange's host-side failure rule, as for the decode exchange:
    a marked sync area makes check() raise and gemm() refuse.  The object is
    assembled by hand around a CPU copy of the sync words."""
    from rotalabs_accel_b200 import _capi
    from rotalabs_accel_b200.peer import PrefillExchange
    ex = PrefillExchange.__new__(PrefillExchange)
    ex._xb = object()
    ex._failed = None
    ex.max_rows, ex.max_n_local, ex._xb_elems = 64, 128, 64 * 128
    ex._sync_words = torch.zeros(_capi.PX_SYNC_BYTES // 4, dtype=torch.int32)
    ex.check()
    assert ex.supports(64, 128) and not ex.supports(65, 128) and not ex.supports(8, 100)
    ex._sync_words[_capi.PX_SYNC_ABORT_WORD] = 3
    with pytest.raises(RuntimeError, match="call 3 gave up"):
        ex.check()
    with pytest.raises(RuntimeError, match="set up a new one"):
        ex.gemm(torch.zeros(64, 32, dtype=torch.float16), torch.zeros(128, 32, dtype=torch.int8),
                torch.ones(128))


def test_prefill_exchange_needs_a_process_group():
    from rotalabs_accel_b200.peer import PrefillExchange
    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    with pytest.raises(RuntimeError, match="process group"):
        PrefillExchange()


def test_exchange_operand_checks():
    """The exchanges pass raw pointers on: wrong dtypes, devices, shapes or
    strides are refused on the host before anything reaches the library."""
    from rotalabs_accel_b200.peer import check_exchange_operands
    x = torch.zeros(4, 64, dtype=torch.float16)
    w = torch.zeros(32, 64, dtype=torch.int8)
    s = torch.ones(32)
    with pytest.raises(TypeError, match="CUDA"):
        check_exchange_operands(x, w, s, None, None, 2)           # CPU tensors never reach the kernels
    with pytest.raises(TypeError, match="float16"):
        check_exchange_operands(x.to(torch.bfloat16), w, s, None, None, 2)
    with pytest.raises(TypeError, match="float16"):
        check_exchange_operands(x[:, ::2], w, s, None, None, 2)   # strided rows
