"""Direct peer-to-peer output exchange for the column-parallel layer.

rotalabs-accel has no distributed code; this is the fused output step of the
sharded ``Int8Linear`` (src/rotalabs_accel/kernels/gemm.py:241-336 with its
output channels split over the ranks).  Instead of "local GEMM, then
``all_gather_into_tensor``, then a reorder kernel", one decode kernel per
rank computes its column slice, writes it into its own output and sends it
to every peer over NVLink as 8-byte flagged words {two fp16 values, call
number}; the kernel's last CTAs unpack the peers' slices from this rank's
receive buffer (``rla_w8a16_gemm_allgather``).  No host synchronisation,
no separate collective, one launch.

Set-up is collective (every rank of the group, one process per GPU, one
node): ``PeerExchange(group, max_rows, max_n_local)`` allocates this rank's
receive buffer with the library's own ``cudaMalloc`` (so an IPC handle covers
exactly that buffer), exchanges the handles in one all-gather of a few bytes
over the process group, maps every peer's buffer, and keeps a local sync
area.  ``exchange.gemm(x2d, weight_int8, scale, bias)`` then runs on every
rank, in the same order and with the same shapes on every rank,
stream-ordered on each rank.  ``close()`` (collective) unmaps and frees.

Failure: every wait inside an exchange call is bounded.  A wait that gives up
(a peer that never sends its slice) marks this rank's sync area, and from then
on every exchange call on it returns at once with its output incomplete
(device errors 7, 8 and then 9).  ``check()`` reads the mark; once it is
seen, ``gemm`` refuses further calls.  Recovery is collective: ``close()`` on
every rank, then a new ``PeerExchange``.
"""

from __future__ import annotations

import struct
from typing import List, Optional

import torch
import torch.distributed as dist

from . import _capi


def exchange_blobs(blob: bytes, group: Optional[dist.ProcessGroup] = None) -> List[bytes]:
    """All-gather one byte string per rank (all the same length) over the
    process group (NCCL or gloo); returns them in rank order."""
    world = dist.get_world_size(group)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    mine = torch.tensor(list(blob), dtype=torch.uint8, device=dev)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    return [bytes(p.cpu().tolist()) for p in parts]


def receive_bytes(world: int, max_rows: int, max_n_local: int) -> int:
    """Receive buffer size for calls of up to ``max_rows`` rows and
    ``max_n_local`` columns per rank: two halves (call parity) of
    ``world * ceil(max_rows / 2) * max_n_local`` 8-byte flagged words."""
    return 16 * world * ((max_rows + 1) // 2) * max_n_local


def check_exchange_operands(x2d: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
                            bias: Optional[torch.Tensor], out: Optional[torch.Tensor], world: int) -> None:
    """The exchanges hand raw pointers to the library: refuse operands the
    kernels would misread (``x2d`` fp16 ``[M, K]`` with unit inner stride,
    ``weight_int8`` int8 ``[n_local, K]`` with unit inner stride, ``scale``
    and ``bias`` contiguous ``[n_local]`` fp32/fp16, ``out`` fp16
    ``[M, >= world * n_local]`` with unit inner stride, all on one CUDA
    device)."""
    if x2d.dim() != 2 or x2d.dtype != torch.float16 or not x2d.is_cuda or (x2d.numel() and x2d.stride(1) != 1):
        raise TypeError("exchange: x must be a 2-D float16 CUDA tensor with unit inner stride")
    dev = x2d.device
    if (weight_int8.dim() != 2 or weight_int8.dtype != torch.int8 or weight_int8.device != dev
            or weight_int8.shape[1] != x2d.shape[1] or (weight_int8.numel() and weight_int8.stride(1) != 1)):
        raise TypeError(f"exchange: weight_int8 must be int8 [n_local, {x2d.shape[1]}] with unit inner stride on "
                        f"{dev}")
    n_local = weight_int8.shape[0]
    for name, t in (("scale", scale), ("bias", bias)):
        if t is None:
            continue
        if (t.shape != (n_local,) or t.dtype not in (torch.float16, torch.float32) or t.device != dev
                or not t.is_contiguous()):
            raise TypeError(f"exchange: {name} must be a contiguous float16/float32 [{n_local}] tensor on {dev}")
    if out is not None and (out.dtype != torch.float16 or out.device != dev or out.dim() != 2
                            or out.shape[0] != x2d.shape[0] or out.shape[1] < world * n_local
                            or (out.numel() and out.stride(1) != 1)):
        raise TypeError(f"exchange: out must be float16 [{x2d.shape[0]}, >= {world * n_local}] with unit inner "
                        f"stride on {dev}")


class _SharedBuffer:
    """One device buffer per rank, every rank's mapped into this process.
    Every step is collective: a rank whose set-up fails still takes part in
    both exchanges, and then every rank raises (none is left half set up)."""

    def __init__(self, nbytes: int, group, rank: int, header: bytes):
        self.local = 0
        self.ptrs: List[int] = []
        self._opened: List[int] = []
        error = None
        handle = bytes(_capi.IPC_HANDLE_BYTES)
        try:
            self.local = _capi.peer_alloc(nbytes)
            handle = _capi.ipc_export(self.local)
        except Exception as e:  # noqa: BLE001 - reported on every rank below
            error = e
        blobs = exchange_blobs(header + handle, group)
        if error is None:
            try:
                for r, b in enumerate(blobs):
                    if b[:len(header)] != header:
                        raise RuntimeError(f"peer exchange: rank {r} set up a different exchange than rank {rank}")
                    if r == rank:
                        self.ptrs.append(self.local)
                    else:
                        p = _capi.ipc_open(b[len(header):])
                        self._opened.append(p)
                        self.ptrs.append(p)
            except Exception as e:  # noqa: BLE001
                error = e
        oks = exchange_blobs(b"\x01" if error is None else b"\x00", group)
        if error is not None or any(o != b"\x01" for o in oks):
            self.release()
            if error is not None:
                raise error
            bad = [r for r, o in enumerate(oks) if o != b"\x01"]
            raise RuntimeError(f"peer exchange: set-up failed on rank(s) {bad}")

    def unmap(self) -> None:
        """Close this process's mappings of the peers' buffers."""
        for p in self._opened:
            _capi.ipc_close(p)
        self._opened = []
        self.ptrs = []

    def release(self) -> None:
        self.unmap()
        if self.local:
            _capi.peer_free(self.local)
            self.local = 0


class PeerExchange:
    """Receive buffers and sync area of a process group for
    ``rla_w8a16_gemm_allgather`` (decode calls of up to ``max_rows`` rows and
    ``max_n_local`` output columns per rank)."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None, max_rows: int = 32, max_n_local: int = 8192):
        if not dist.is_initialized():
            raise RuntimeError("PeerExchange needs an initialised process group")
        if not 1 <= max_rows <= 32 or max_n_local < 1:
            raise ValueError("PeerExchange: need 1 <= max_rows <= 32 (the decode kernels) and max_n_local >= 1")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _capi.MAX_PEERS:
            raise ValueError(f"the peer exchange supports at most {_capi.MAX_PEERS} ranks, got {self.world}")
        self.max_rows, self.max_n_local = max_rows, max_n_local
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.recv_bytes = receive_bytes(self.world, max_rows, max_n_local)
        header = struct.pack("<qqq", self.world, max_rows, max_n_local)
        self._recv = _SharedBuffer(self.recv_bytes, group, self.rank, header)
        self._sync = torch.zeros(_capi.PEER_SYNC_BYTES // 4, dtype=torch.int32, device=self.device)
        self._failed: Optional[str] = None

    def calls_completed(self) -> int:
        """Exchange calls this rank has completed (synchronises)."""
        return int(self._sync[0].item())

    def check(self) -> None:
        """Raise if a wait of an exchange call on this rank gave up
        (synchronises with the device).  From then on ``gemm`` refuses
        further calls: ``close()`` this exchange on every rank and create a
        new one."""
        if self._failed is None and int(self._sync[_capi.PEER_SYNC_ABORT_WORD].item()) != 0:
            self._failed = (f"a wait of exchange call {int(self._sync[_capi.PEER_SYNC_ABORT_WORD].item())} gave up "
                            "(a peer's slice or this launch's CTAs did not arrive in time)")
        if self._failed is not None:
            raise RuntimeError(f"PeerExchange failed: {self._failed}; close() it on every rank and set up a new one")

    def gemm(self, x2d: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
             bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``out[M, world * n_local]``: every rank's slice of ``x2d @
        (weight_int8 * scale[:, None]).T (+ bias)``, this rank's computed
        here from its shard ``weight_int8 [n_local, K]``."""
        if self._recv is None:
            raise RuntimeError("PeerExchange is closed")
        if self._failed is not None:
            raise RuntimeError(f"PeerExchange failed: {self._failed}; close() it on every rank and set up a new one")
        check_exchange_operands(x2d, weight_int8, scale, bias, out, self.world)
        M = x2d.shape[0]
        n_local = weight_int8.shape[0]
        if M > self.max_rows or n_local > self.max_n_local:
            raise ValueError(f"exchange sized for {self.max_rows} rows x {self.max_n_local} columns per rank, "
                             f"got {M} x {n_local}")
        if out is None:
            out = torch.empty((M, self.world * n_local), dtype=torch.float16, device=x2d.device)
        return _capi.w8a16_gemm_allgather(x2d, weight_int8, scale, bias, out, self._recv.ptrs, self.recv_bytes,
                                          self._sync.data_ptr(), self.rank)

    def close(self) -> None:
        """Collective: wait for every rank's work, then unmap and free."""
        if self._recv is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)       # no peer writes into our buffer after this
        self._recv.unmap()
        dist.barrier(group=self.group)       # no rank maps another's buffer any more
        self._recv.release()
        self._recv = None


class _CudaArray:
    """Minimal ``__cuda_array_interface__`` over a raw device pointer, so a
    buffer of the library's own allocation can be viewed as a tensor."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _device_view(ptr: int, shape, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    typestr = {torch.float16: "<f2", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_CudaArray(ptr, shape, typestr), device=device)


_comm_streams: dict = {}


def comm_stream(device: torch.device) -> torch.cuda.Stream:
    """The per-device stream that the overlapped prefill runs its exchange on.
    High priority: when a GEMM CTA leaves an SM, a waiting exchange CTA gets
    the SM before the next GEMM tile (measured at 2 ranks, M = 4096, the
    8192 -> 14336 shard's pull overlapped in two blocks: 1130 -> 1072 us per
    call)."""
    s = _comm_streams.get(device.index)
    if s is None:
        s = _comm_streams[device.index] = torch.cuda.Stream(device=device, priority=-1)
    return s


class PrefillExchange:
    """Exchange buffers and sync areas of a process group for the pull
    exchange of the column-parallel prefill (``rla_prefill_exchange_*``):
    calls of up to ``max_rows`` rows and ``max_n_local`` output columns per
    rank, ``max_n_local`` a multiple of 8.

    One call (``gemm``), on every rank in the same order with the same
    shapes: the rows are cut into blocks; per block, this rank's GEMM writes
    its slice into its own exchange buffer on the current stream, and on a
    communication stream the pull kernel marks the block ready on every rank,
    waits for every rank's mark and copies every rank's slice of those rows
    from its exchange buffer (over NVLink) straight into the output's
    columns, while the next block's GEMM runs.  No collective library call,
    no staging copy, no reorder pass.  The current stream waits for the
    communication stream at the end (the call captures into a CUDA graph).

    Failure: as ``PeerExchange`` -- bounded waits, device error 7 and a mark
    in the sync area; ``check()`` raises once the mark is seen and ``gemm``
    then refuses; recovery is ``close()`` on every rank and a new exchange.
    Unlike the decode exchange, the GEMMs do not read the mark, so a peer
    slower than the wait limit could read a partly overwritten buffer of the
    failed call: the limit must stay far above any call's duration."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None, max_rows: int = 4096, max_n_local: int = 14336):
        if not dist.is_initialized():
            raise RuntimeError("PrefillExchange needs an initialised process group")
        if max_rows < 1 or max_n_local < 8 or max_n_local % 8:
            raise ValueError("PrefillExchange: need max_rows >= 1 and max_n_local a positive multiple of 8")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _capi.MAX_PEERS:
            raise ValueError(f"the peer exchange supports at most {_capi.MAX_PEERS} ranks, got {self.world}")
        self.max_rows, self.max_n_local = max_rows, max_n_local
        self.device = torch.device("cuda", torch.cuda.current_device())
        header = struct.pack("<qqqq", 2, self.world, max_rows, max_n_local)
        self._xb = _SharedBuffer(2 * max_rows * max_n_local, group, self.rank, header)
        try:
            self._sync = _SharedBuffer(_capi.PX_SYNC_BYTES, group, self.rank, header)
        except Exception:
            self._xb.release()
            raise
        self._xb_elems = max_rows * max_n_local
        self._xb_flat = _device_view(self._xb.local, (self._xb_elems,), torch.float16, self.device)
        self._sync_words = _device_view(self._sync.local, (_capi.PX_SYNC_BYTES // 4,), torch.int32, self.device)
        self._failed: Optional[str] = None

    def calls_started(self) -> int:
        """Exchange calls this rank has begun (synchronises)."""
        return int(self._sync_words[0].item())

    def check(self) -> None:
        """Raise if a wait of an exchange call on this rank gave up
        (synchronises); from then on ``gemm`` refuses further calls."""
        if self._failed is None:
            mark = int(self._sync_words[_capi.PX_SYNC_ABORT_WORD].item())
            if mark != 0:
                self._failed = f"a wait of prefill exchange call {mark} gave up (a peer's block did not arrive in time)"
        if self._failed is not None:
            raise RuntimeError(f"PrefillExchange failed: {self._failed}; close() it on every rank and set up a "
                               "new one")

    def supports(self, M: int, n_local: int) -> bool:
        return 1 <= M and n_local % 8 == 0 and M * n_local <= self._xb_elems and n_local <= self.max_n_local

    def gemm(self, x2d: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
             bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None, blocks=None) -> torch.Tensor:
        """``out[M, world * n_local]``: every rank's slice of ``x2d @
        (weight_int8 * scale[:, None]).T (+ bias)``, this rank's computed
        here from its shard ``weight_int8 [n_local, K]``.  ``blocks``: the
        row blocks ``[(row0, rows), ...]`` (default: the pipeline model's
        choice, identical on every rank)."""
        if self._xb is None:
            raise RuntimeError("PrefillExchange is closed")
        if self._failed is not None:
            raise RuntimeError(f"PrefillExchange failed: {self._failed}; close() it on every rank and set up a "
                               "new one")
        check_exchange_operands(x2d, weight_int8, scale, bias, out, self.world)
        M, K = x2d.shape
        n_local = weight_int8.shape[0]
        if not self.supports(M, n_local):
            raise ValueError(f"prefill exchange sized for {self.max_rows} x {self.max_n_local} per rank "
                             f"(n_local a multiple of 8), got {M} x {n_local}")
        dev = x2d.device
        if out is None:
            out = torch.empty((M, self.world * n_local), dtype=torch.float16, device=dev)
        if blocks is None:
            from .sharded import prefill_row_blocks
            blocks = prefill_row_blocks(M, n_local, K, self.world, _capi.device_sm_count(dev.index), "p2p")
        if len(blocks) > _capi.PX_MAX_BLOCKS:
            raise ValueError(f"at most {_capi.PX_MAX_BLOCKS} blocks per call")
        xb = self._xb_flat[:M * n_local].view(M, n_local)
        cur = torch.cuda.current_stream(dev)
        comm = comm_stream(dev)
        _capi.prefill_exchange_begin(self._sync.ptrs, self.rank, cur.cuda_stream)
        for b, (r0, rows) in enumerate(blocks):
            _capi.w8a16_gemm(x2d[r0:r0 + rows], weight_int8, scale, bias, out=xb[r0:r0 + rows])
            done = torch.cuda.Event()
            done.record(cur)
            comm.wait_event(done)
            _capi.prefill_exchange_block(self._xb.ptrs, n_local, self._sync.ptrs, self.rank, b, b == len(blocks) - 1,
                                         r0, rows, n_local, out, comm.cuda_stream)
        cur.wait_stream(comm)
        return out

    def close(self) -> None:
        """Collective: wait for every rank's work, then unmap and free."""
        if self._xb is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._xb.unmap()
        self._sync.unmap()
        dist.barrier(group=self.group)
        self._xb_flat = None
        self._sync_words = None
        self._xb.release()
        self._sync.release()
        self._xb = None
