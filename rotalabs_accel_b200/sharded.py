"""Column-parallel W8A16 layer over several GPUs (one process per GPU).

rotalabs-accel has no distributed code; this is the sharded mode of its
``Int8Linear`` (src/rotalabs_accel/kernels/gemm.py:241-336).  Output
channels are split over the ranks: rank r holds rows
``[r * n_local, (r + 1) * n_local)`` of ``weight_int8`` / ``scale`` (/ ``bias``),
``n_local = ceil(N / world)`` (the last shard is zero-padded when ``world``
does not divide ``N``).  Every rank has the whole activation ``x``.

Forward, per rank, collective path:
  1. ``y_local[M, n_local]`` = the sm_100a W8A16 kernel on the local shard;
  2. one ``all_gather_into_tensor`` of the slices into
     ``staging[world, M, n_local]`` (NCCL over NVLink on GPUs, gloo on the CPU);
  3. ``rla_gather_columns`` reorders the staging buffer into ``y[M, N]``
     (skipped when M == 1: the staging layout already is ``[1, N]``).
On GPUs a long prefill (``prefill_overlapped``) runs these steps per block
of rows: the all-gather and reorder of block i run on a communication stream
while the GEMM of block i+1 runs, so the exchange hides behind the math.

Fused path (after ``enable_peer_exchange``; decode batches of at most
``max_tokens`` rows, K % 16 == 0): one kernel per rank computes its slice,
sends it to every peer over NVLink and unpacks theirs
(``rotalabs_accel_b200.peer``).  The choice depends only on shapes, which
are the same on every rank, so the ranks always take the same path.

Per-channel quantization is row-independent, so quantizing a shard gives
exactly the rows the full quantization would.
"""

from __future__ import annotations

import functools
from typing import Optional

import torch
import torch.distributed as dist

from .gemm import int8_gemm
from .peer import PeerExchange, PrefillExchange, comm_stream
from .quantization import quantize_weight_per_channel


def shard_range(n_total: int, world: int, rank: int):
    """``(start, stop, n_local)`` of rank's output channels; ``stop - start``
    may be below ``n_local`` (or 0) for the last ranks when world does not
    divide ``n_total``."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    n_local = -(-n_total // world)
    start = min(rank * n_local, n_total)
    stop = min(start + n_local, n_total)
    return start, stop, n_local


def assemble_columns(staging: torch.Tensor, n_total: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``staging[world, M, n_local]`` -> ``[M, n_total]`` (CUDA: the library's
    gather kernel; CPU: a torch permute)."""
    world, M, n_local = staging.shape
    if staging.is_cuda:
        from . import _capi
        if n_total == world * n_local:
            if out is None:
                out = torch.empty((M, n_total), dtype=staging.dtype, device=staging.device)
            if M == 1:
                out.copy_(staging.view(1, n_total))
                return out
            return _capi.gather_columns(staging, world, M, n_local, out)
        full = torch.empty((M, world * n_local), dtype=staging.dtype, device=staging.device)
        _capi.gather_columns(staging, world, M, n_local, full)
        y = full[:, :n_total]
        if out is None:
            return y.contiguous()
        out.copy_(y)
        return out
    y = staging.permute(1, 0, 2).reshape(M, world * n_local)[:, :n_total]
    if out is None:
        return y.contiguous()
    out.copy_(y)
    return out


# Block sizes of the overlapped prefill, from a two-stream model fitted to
# B200 measurements of the config-4 shards (M = 512-4096, 2 ranks):
#  * the local GEMM of a block takes whole rounds of tiles (tcgen05 kernel,
#    one tile per SM at a time; blocks on one stream run one after the
#    other); a round of 256-row tiles takes ~7.8 us + K * 7.23 ns, a round of
#    128-row tiles ~0.95 of that, a grid smaller than one round ~0.9 of it
#    (fewer busy SMs under the power cap), plus ~8 us per launch;
#  * the pull exchange moves ~600 GB/s into a rank alone and ~350 GB/s while
#    a GEMM runs beside it, and slows that GEMM by a quarter of the overlap;
#  * the NCCL path: ~15 us + ~650 GB/s of all-gather into each rank, then a
#    reorder at ~5 TB/s.
def _gemm_us(rows: int, n_local: int, K: int, sms: int) -> float:
    nt = -(-n_local // 128)

    def tiles(bm):
        return nt * -(-rows // bm)

    def rounds(bm):
        return -(-tiles(bm) // sms)

    round_us = 7.8 + K * 7.23e-3
    # the library's own choice of tile height (rla_capi.cu, make_plan)
    if rows > 128 and rounds(256) * 256 * 1.0 <= rounds(128) * 128 * 1.9:
        bm, rel = 256, 1.0
    elif rows > 64:
        bm, rel = 128, 0.95
    else:
        bm, rel = 64, 0.95
    if tiles(bm) < sms:
        rel *= 0.9
    return rounds(bm) * rel * round_us + 8.0


def _exchange_us(rows: int, n_local: int, world: int, kind: str = "nccl") -> float:
    """The exchange of one block alone (no GEMM beside it)."""
    if kind == "p2p":
        return 6.0 + (world - 1) * rows * n_local * 2 / 600e9 * 1e6
    ag = 15.0 + (world - 1) * rows * n_local * 2 / 650e9 * 1e6
    reorder = 2.0 * rows * world * n_local * 2 / 5e12 * 1e6
    return ag + reorder


def _pipeline_us(block_rows, n_local: int, K: int, world: int, sms: int, kind: str = "nccl") -> float:
    """Modelled time of one call with these row blocks (see above)."""
    if kind != "p2p":
        t_gemm = t_done = 0.0
        for r in block_rows:
            t_gemm += _gemm_us(r, n_local, K, sms)
            t_done = max(t_gemm, t_done) + _exchange_us(r, n_local, world, kind)
        return t_done
    r_alone, r_ovl, slow = 600e9, 350e9, 0.25
    g_end, t = [], 0.0
    for r in block_rows:
        t += _gemm_us(r, n_local, K, sms)
        g_end.append(t)
    t_pull, extra = 0.0, 0.0
    for i, r in enumerate(block_rows):
        start = max(g_end[i] + extra, t_pull)
        nbytes = (world - 1) * r * n_local * 2
        if i + 1 < len(block_rows):
            window = max(0.0, g_end[i + 1] + extra - start)
            d_ovl = nbytes / r_ovl * 1e6
            if d_ovl <= window:
                dur = d_ovl
                extra += slow * dur
            else:
                dur = window + (nbytes - window * 1e-6 * r_ovl) / r_alone * 1e6
                extra += slow * window
        else:
            dur = nbytes / r_alone * 1e6
        t_pull = start + dur + 6.0
    return max(t_pull, g_end[-1] + extra)


def _compositions(units: int, parts: int):
    if parts == 1:
        yield (units,)
        return
    for first in range(1, units - parts + 2):
        for rest in _compositions(units - first, parts - 1):
            yield (first,) + rest


@functools.lru_cache(maxsize=256)
def prefill_row_blocks(M: int, n_local: int, K: int = 8192, world: int = 2, sms: int = 148, exchange: str = "nccl"):
    """``[(row0, rows), ...]`` covering ``[0, M)`` in order: 1 to 4 blocks of
    rows, each a multiple of 128 rows but the last (which takes the ragged
    tail), at least 512 rows each when there are several, with the least
    modelled time (``_pipeline_us``).  Blocks need not be equal: a block
    split that adds a partly empty round of tiles costs GEMM time (4096 x
    14336 on 148 SMs is 12.1 rounds; halves are 6.05 each, but 3328 + 768 rows
    are 10 + 3), and a short last block leaves little exchange exposed.  One
    block is the serial GEMM -> exchange; more blocks are taken only for a
    clear gain (3 %).  ``exchange``: "nccl" (all-gather, then reorder) or
    "p2p" (``PrefillExchange``'s pull over NVLink)."""
    units = max(1, M // 128)     # a ragged tail of rows joins the last block

    def rows_of(u0, u):
        return M - u0 * 128 if u0 + u == units else u * 128

    best, best_t = None, None
    for c in range(1, min(4, units) + 1):
        c_best, c_t = None, None
        for comp in _compositions(units, c):
            if c > 1 and min(comp) < 4:      # blocks of 512 rows or more (the model is fitted there)
                continue
            rows, u0 = [], 0
            for u in comp:
                rows.append(rows_of(u0, u))
                u0 += u
            t = _pipeline_us(rows, n_local, K, world, sms, exchange)
            if c_t is None or t < c_t:
                c_best, c_t = comp, t
        if c_t is not None and (best_t is None or c_t < best_t * 0.97):
            best, best_t = c_best, c_t
    blocks, u0 = [], 0
    for u in best:
        blocks.append((u0 * 128, rows_of(u0, u)))
        u0 += u
    return blocks


def prefill_overlapped(x2: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor,
                       bias: Optional[torch.Tensor], n_total: int, world: int, group=None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Column-parallel W8A16 GEMM of a long activation block on CUDA:
    ``y[M, n_total]`` on every rank from its shard ``weight_int8 [n_local, K]``.

    Per block of rows (``prefill_row_blocks``): the local GEMM on the current
    stream, then, on a per-device communication stream that waits for it, the
    NCCL all-gather of the block's slices and their reorder into the block's
    rows of ``y``.  The GEMM of the next block runs meanwhile.  The current
    stream waits for the communication stream before returning, so the
    result is ordered like any other stream work (also under CUDA-graph
    capture).  Every rank makes the same calls in the same order."""
    M, K = x2.shape
    n_local = weight_int8.shape[0]
    dev = x2.device
    if out is None:
        out = torch.empty((M, n_total), dtype=torch.float16, device=dev)
    cur = torch.cuda.current_stream(dev)
    comm = comm_stream(dev)
    from . import _capi
    blocks = prefill_row_blocks(M, n_local, K, world, _capi.device_sm_count(dev.index))
    # every buffer is allocated here on the current stream and lives until
    # the communication stream has been joined back (no cross-stream frees)
    staging = torch.empty((world * M * n_local,), dtype=torch.float16, device=dev)   # [world, rows, n_local] per block
    y_loc = torch.empty((M, n_local), dtype=torch.float16, device=dev)
    for r0, rows in blocks:
        _capi.w8a16_gemm(x2[r0:r0 + rows], weight_int8, scale, bias, out=y_loc[r0:r0 + rows])
        done = torch.cuda.Event()
        done.record(cur)
        with torch.cuda.stream(comm):
            comm.wait_event(done)
            st = staging[world * r0 * n_local:world * (r0 + rows) * n_local].view(world, rows, n_local)
            dist.all_gather_into_tensor(st, y_loc[r0:r0 + rows], group=group)
            assemble_columns(st, n_total, out=out[r0:r0 + rows])
    cur.wait_stream(comm)
    return out


class ColumnParallelInt8Linear(torch.nn.Module):
    """``Int8Linear`` with its output channels split over a process group.

    Buffers (local shard): ``weight_int8`` int8 ``[n_local, in]``, ``scale``
    fp32 ``[n_local]``, optional fp16 ``bias`` ``[n_local]``.  ``forward``
    returns the full ``(..., out_features)`` output on every rank.
    """

    def __init__(self, in_features: int, out_features: int, bias: bool = False,
                 group: Optional[dist.ProcessGroup] = None):
        super().__init__()
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.in_features = in_features
        self.out_features = out_features
        self.start, self.stop, self.n_local = shard_range(out_features, self.world, self.rank)
        self.register_buffer("weight_int8", torch.zeros(self.n_local, in_features, dtype=torch.int8))
        self.register_buffer("scale", torch.ones(self.n_local, dtype=torch.float32))
        if bias:
            self.bias = torch.nn.Parameter(torch.zeros(self.n_local, dtype=torch.float16))
        else:
            self.register_parameter("bias", None)
        self._quantized = False
        self._exchange: Optional[PeerExchange] = None
        self._owns_exchange = False
        self._prefill: Optional[PrefillExchange] = None
        self._owns_prefill = False

    def _check_agreement(self) -> None:
        """Every rank must shard the same layer: compare (in, out, world) over
        the group; a mismatch raises on every rank instead of corrupting the
        gather."""
        if self.world == 1:
            return
        dev = self.weight_int8.device
        mine = torch.tensor([self.in_features, self.out_features, self.world], dtype=torch.int64,
                            device=dev if dev.type == "cuda" else "cpu")
        allv = [torch.zeros_like(mine) for _ in range(self.world)]
        dist.all_gather(allv, mine, group=self.group)
        for r, v in enumerate(allv):
            if not torch.equal(v, mine):
                raise RuntimeError(f"ColumnParallelInt8Linear: rank {r} has shape {v.tolist()}, "
                                   f"rank {self.rank} has {mine.tolist()}")

    def quantize_weights(self, weight: torch.Tensor) -> None:
        """Quantize this rank's rows of the full ``[out, in]`` weight."""
        assert weight.shape == (self.out_features, self.in_features)
        self._check_agreement()
        q, s = quantize_weight_per_channel(weight[self.start:self.stop])
        self.weight_int8.zero_()
        self.scale.fill_(1.0)
        rows = self.stop - self.start
        self.weight_int8[:rows].copy_(q.to(self.weight_int8.device))
        self.scale[:rows].copy_(s.to(self.scale.device))
        self._quantized = True

    def load_shard(self, weight_int8: torch.Tensor, scale: torch.Tensor, bias: Optional[torch.Tensor] = None):
        """Install an already-quantized full layer's rows for this rank."""
        assert weight_int8.shape == (self.out_features, self.in_features)
        self._check_agreement()
        rows = self.stop - self.start
        self.weight_int8.zero_()
        self.scale.fill_(1.0)
        self.weight_int8[:rows].copy_(weight_int8[self.start:self.stop])
        self.scale[:rows].copy_(scale[self.start:self.stop].float())
        if bias is not None and self.bias is not None:
            self.bias.data.zero_()
            self.bias.data[:rows].copy_(bias[self.start:self.stop])
        self._quantized = True

    def enable_peer_exchange(self, max_tokens: int = 32, exchange: Optional[PeerExchange] = None,
                             max_prefill_tokens: int = 0, prefill_exchange: Optional[PrefillExchange] = None) -> None:
        """Collective (every rank, module already on its GPU): use the fused
        peer-to-peer path for batches of up to ``max_tokens`` rows (at most
        32), and, with ``max_prefill_tokens`` > 32 (or a ``prefill_exchange``),
        the pull exchange for longer batches of up to that many rows.  Either
        exchange may be shared by several layers (sized for their rows and
        columns per rank); by default the layer makes its own."""
        if not 1 <= max_tokens <= 32:
            raise ValueError("max_tokens must be in [1, 32] (the decode kernels)")
        if not self.weight_int8.is_cuda:
            raise RuntimeError("enable_peer_exchange: move the module to its GPU first")
        if exchange is None:
            exchange = PeerExchange(self.group, max_rows=max_tokens, max_n_local=self.n_local)
            self._owns_exchange = True
        elif exchange.max_rows < max_tokens or exchange.max_n_local < self.n_local:
            raise ValueError("enable_peer_exchange: the shared exchange is too small for this layer")
        self._exchange = exchange
        self._max_tokens = max_tokens
        if prefill_exchange is None and max_prefill_tokens > 32 and self.n_local % 8 == 0:
            prefill_exchange = PrefillExchange(self.group, max_rows=max_prefill_tokens, max_n_local=self.n_local)
            self._owns_prefill = True
        elif prefill_exchange is not None and not prefill_exchange.supports(prefill_exchange.max_rows, self.n_local):
            raise ValueError("enable_peer_exchange: the shared prefill exchange is too small for this layer")
        self._prefill = prefill_exchange

    def close_peer_exchange(self) -> None:
        """Collective: release the peer paths' buffers (those the layer owns)."""
        if self._exchange is not None and self._owns_exchange:
            self._exchange.close()
        if self._prefill is not None and self._owns_prefill:
            self._prefill.close()
        self._exchange = None
        self._owns_exchange = False
        self._prefill = None
        self._owns_prefill = False

    def _fused_ok(self, x2: torch.Tensor) -> bool:
        return (self._exchange is not None and x2.is_cuda and x2.dtype == torch.float16
                and 1 <= x2.shape[0] <= self._max_tokens and self.in_features % 16 == 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self._quantized:
            raise RuntimeError("Weights not quantized. Call quantize_weights() first.")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.in_features)
        M = x2.shape[0]
        if self._fused_ok(x2):
            if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
                x2 = x2.clone(memory_format=torch.contiguous_format)
            y = self._exchange.gemm(x2, self.weight_int8, self.scale, self.bias)
            if y.shape[1] != self.out_features:
                y = y[:, :self.out_features]
            return y.reshape(*lead, self.out_features)
        pull = (self._prefill is not None and M > 32 and self._prefill.supports(M, self.n_local))
        if (self.world > 1 and x2.is_cuda and (M >= 1024 or pull) and x2.dtype == torch.float16
                and x2.stride(1) == 1 and self.weight_int8.stride(1) == 1):
            b = self.bias
            if b is not None and b.dtype not in (torch.float16, torch.float32):
                b = b.half()
            if pull:
                y = self._prefill.gemm(x2, self.weight_int8, self.scale, b)
            else:
                y = prefill_overlapped(x2, self.weight_int8, self.scale, b, self.world * self.n_local, self.world,
                                       group=self.group)
            if y.shape[1] != self.out_features:
                y = y[:, :self.out_features]
            return y.reshape(*lead, self.out_features)
        y_local = int8_gemm(x2, self.weight_int8, self.scale, self.bias)
        if self.world == 1:
            return y_local[:, :self.out_features].reshape(*lead, self.out_features)
        staging = torch.empty((self.world, M, self.n_local), dtype=y_local.dtype, device=y_local.device)
        if y_local.is_cuda:
            dist.all_gather_into_tensor(staging, y_local.contiguous(), group=self.group)
        else:
            dist.all_gather(list(staging.unbind(0)), y_local.contiguous(), group=self.group)
        y = assemble_columns(staging, self.out_features)
        return y.reshape(*lead, self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, world={self.world}, "
                f"rank={self.rank}, rows=[{self.start}, {self.stop}), quantized={self._quantized}")
