"""ctypes binding of the C ABI in ``include/rla_w8a16.h``.

The shared library ``librla_w8a16.so`` is built in-tree
(``rotalabs_accel_b200/build.py``) and loaded from this package directory.
Every CUDA computation of the package goes through here; if the library is
missing or does not load, calls raise instead of computing anything another
way.

The per-token hot calls (``w8a16_gemm``, ``w8a16_gemm_swiglu``) go through
``_rla_fast``, CPython fast-call bindings of the same entry points linked to
the same library (ctypes' generic argument conversion costs more host time
than a decode GEMM takes on the GPU).  Without that module they use ctypes.
A call without a preallocated output goes through ``torch.ops.rla.w8a16_gemm``
(``_rla_torch_ops.so``, a C++ ``torch.library`` registration over the same C
ABI that allocates the output with torch's allocator), when it loads.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librla_w8a16.so")
TORCH_OP_PATH = os.path.join(_HERE, "_rla_torch_ops.so")

RLA_OK = 0
DTYPE_NONE, DTYPE_F16, DTYPE_F32, DTYPE_BF16 = 0, 1, 2, 3
KERNEL_NAMES = {0: "none", 1: "skinny", 2: "tcgen05", 3: "generic", 4: "fill", 5: "stream"}
KERNEL_IDS = {v: k for k, v in KERNEL_NAMES.items()}

EXPORTED_SYMBOLS = (
    "rla_w8a16_gemm", "rla_w8a16_workspace_size", "rla_w8a16_plan", "rla_quantize_per_channel",
    "rla_gather_columns", "rla_launch_count", "rla_get_device_error", "rla_last_error", "rla_version",
    "rla_set_decode_kernel", "rla_w8a16_gemm_allgather", "rla_set_peer_wait_limit", "rla_peer_alloc",
    "rla_peer_free", "rla_ipc_export", "rla_ipc_open", "rla_ipc_close",
    "rla_w8a16_gemm_swiglu", "rla_w8a16_swiglu_workspace_size", "rla_rmsnorm",
    "rla_w8a16_allgather_workspace_size", "rla_prefill_exchange_begin", "rla_prefill_exchange_block",
)

MAX_PEERS = 8
PEER_SYNC_BYTES = 512
PEER_SYNC_ABORT_WORD = 96
IPC_HANDLE_BYTES = 64
PX_SYNC_BYTES = 1024
PX_MAX_BLOCKS = 16
PX_SYNC_ABORT_WORD = 1

_lib = None
_fast = None
_torch_op = None          # torch.ops.rla.w8a16_gemm.default (through the dispatcher)
_torch_op_direct = None   # the same CUDA kernel function, called without the dispatcher
_lib_lock = threading.Lock()


class RlaError(RuntimeError):
    """A C-ABI call returned a non-OK status."""


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load (once) and type the C ABI.  Raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"rotalabs_accel_b200: CUDA library {path} is missing; build it with "
                "`python -m rotalabs_accel_b200.build` (there is no non-CUDA path for CUDA tensors)")
        lib = ctypes.CDLL(path)
        i64, p, sz = ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t
        lib.rla_w8a16_gemm.argtypes = [p, i64, p, i64, p, ctypes.c_int, p, ctypes.c_int, p, i64,
                                       i64, i64, i64, p, sz, p]
        lib.rla_w8a16_gemm.restype = ctypes.c_int
        lib.rla_w8a16_workspace_size.argtypes = [i64, i64, i64]
        lib.rla_w8a16_workspace_size.restype = sz
        lib.rla_w8a16_plan.argtypes = [i64, i64, i64, ctypes.c_int, ctypes.c_int, ctypes.POINTER(i64)]
        lib.rla_w8a16_plan.restype = ctypes.c_int
        lib.rla_quantize_per_channel.argtypes = [p, ctypes.c_int, i64, i64, i64, p, i64, p, p]
        lib.rla_quantize_per_channel.restype = ctypes.c_int
        lib.rla_gather_columns.argtypes = [p, i64, i64, i64, p, i64, p]
        lib.rla_gather_columns.restype = ctypes.c_int
        lib.rla_launch_count.argtypes = []
        lib.rla_launch_count.restype = ctypes.c_uint64
        lib.rla_get_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint)]
        lib.rla_get_device_error.restype = ctypes.c_int
        lib.rla_last_error.argtypes = []
        lib.rla_last_error.restype = ctypes.c_char_p
        lib.rla_version.argtypes = []
        lib.rla_version.restype = ctypes.c_int
        lib.rla_set_decode_kernel.argtypes = [ctypes.c_int]
        lib.rla_set_decode_kernel.restype = ctypes.c_int
        pp = ctypes.POINTER(p)
        lib.rla_w8a16_gemm_allgather.argtypes = [p, i64, p, i64, p, ctypes.c_int, p, ctypes.c_int, p, i64, i64,
                                                 i64, i64, pp, sz, p, ctypes.c_int, ctypes.c_int, p, sz, p]
        lib.rla_w8a16_gemm_allgather.restype = ctypes.c_int
        lib.rla_set_peer_wait_limit.argtypes = [ctypes.c_uint64]
        lib.rla_set_peer_wait_limit.restype = ctypes.c_int
        lib.rla_peer_alloc.argtypes = [sz, pp]
        lib.rla_peer_alloc.restype = ctypes.c_int
        lib.rla_peer_free.argtypes = [p]
        lib.rla_peer_free.restype = ctypes.c_int
        lib.rla_ipc_export.argtypes = [p, p]
        lib.rla_ipc_export.restype = ctypes.c_int
        lib.rla_ipc_open.argtypes = [p, pp]
        lib.rla_ipc_open.restype = ctypes.c_int
        lib.rla_ipc_close.argtypes = [p]
        lib.rla_ipc_close.restype = ctypes.c_int
        lib.rla_w8a16_gemm_swiglu.argtypes = [p, i64, p, p, i64, p, p, ctypes.c_int, p, p, ctypes.c_int, p, i64,
                                              i64, i64, i64, p, sz, p]
        lib.rla_w8a16_gemm_swiglu.restype = ctypes.c_int
        lib.rla_w8a16_swiglu_workspace_size.argtypes = [i64, i64, i64]
        lib.rla_w8a16_swiglu_workspace_size.restype = sz
        lib.rla_rmsnorm.argtypes = [p, i64, p, ctypes.c_int, ctypes.c_float, p, i64, i64, i64, p]
        lib.rla_rmsnorm.restype = ctypes.c_int
        lib.rla_w8a16_allgather_workspace_size.argtypes = [i64, i64, i64]
        lib.rla_w8a16_allgather_workspace_size.restype = sz
        lib.rla_prefill_exchange_begin.argtypes = [p, ctypes.c_int, ctypes.c_int, p]
        lib.rla_prefill_exchange_begin.restype = ctypes.c_int
        lib.rla_prefill_exchange_block.argtypes = [p, i64, p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                   i64, i64, i64, p, i64, p]
        lib.rla_prefill_exchange_block.restype = ctypes.c_int
        if os.path.abspath(path) == LIB_PATH:
            # linked to this library by soname: the loader reuses the copy
            # loaded above, so both bindings share one library state
            try:
                from . import _rla_fast
                globals()["_fast"] = _rla_fast
            except ImportError:
                pass
            if os.path.exists(TORCH_OP_PATH):
                try:
                    # importing the extension module loads the library, whose
                    # static registration defines torch.ops.rla.w8a16_gemm
                    from . import _rla_torch_ops
                    globals()["_torch_op_direct"] = _rla_torch_ops.w8a16_gemm
                    globals()["_torch_op"] = torch.ops.rla.w8a16_gemm.default
                except (ImportError, OSError, RuntimeError, AttributeError):
                    pass
        _lib = lib
        return lib


def _check(status: int, what: str) -> None:
    if status != RLA_OK:
        msg = load_library().rla_last_error().decode(errors="replace")
        raise RlaError(f"{what} failed with status {status}: {msg}")


def _scale_dtype(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return DTYPE_F32
    if t.dtype == torch.float16:
        return DTYPE_F16
    raise TypeError(f"scale must be float32 or float16, got {t.dtype}")


def _bias_dtype(t) -> int:
    if t is None:
        return DTYPE_NONE
    if t.dtype == torch.float16:
        return DTYPE_F16
    if t.dtype == torch.float32:
        return DTYPE_F32
    raise TypeError(f"bias must be float16 or float32, got {t.dtype}")


# Split-K workspaces: one per (device, stream), zero-filled on allocation and
# grown on demand.  Calls on one stream are ordered, so sharing is safe.
_workspaces: dict = {}


def _workspace(device: torch.device, stream_ptr: int, nbytes: int) -> torch.Tensor:
    key = (device.index, stream_ptr)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def plan(M: int, N: int, K: int, aligned: bool = True, have_workspace: bool = True) -> dict:
    """The selector's plan for a shape (no launch)."""
    lib = load_library()
    params = (ctypes.c_int64 * 8)()
    _check(lib.rla_w8a16_plan(M, N, K, int(aligned), int(have_workspace), params), "rla_w8a16_plan")
    keys = ("kernel", "grid_x", "grid_y", "threads", "splits", "w_rows", "x_rows", "smem")
    d = dict(zip(keys, list(params)))
    d["kernel_name"] = KERNEL_NAMES.get(d["kernel"], "?")
    return d


def w8a16_gemm(x2d: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor, bias=None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """``y[M, N] = fp16(x2d @ (weight_int8 * scale[:, None]).T + bias)`` on
    the current CUDA stream through ``rla_w8a16_gemm``.

    ``x2d`` fp16 ``[M, K]`` with unit inner stride; ``weight_int8`` int8
    ``[N, K]`` with unit inner stride; ``scale`` ``[N]`` fp32/fp16
    contiguous; ``bias`` ``[N]`` fp16/fp32 or None."""
    lib = _lib if _lib is not None else load_library()
    if out is None and _torch_op_direct is not None:
        return _torch_op_direct(x2d, weight_int8, scale, bias)
    fast = _fast
    M, K = x2d.shape
    N = weight_int8.shape[0]
    device = x2d.device
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=device)
    index = device.index
    stream = torch._C._cuda_getCurrentRawStream(index)
    need = fast.workspace_size(M, N, K) if fast is not None else lib.rla_w8a16_workspace_size(M, N, K)
    ws_ptr, ws_bytes = 0, 0
    if need:
        ws = _workspace(device, stream, need)
        ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    args = (x2d.data_ptr(), x2d.stride(0) if M > 0 else K, weight_int8.data_ptr(),
            weight_int8.stride(0) if N > 0 else K, scale.data_ptr(), _scale_dtype(scale),
            bias.data_ptr() if bias is not None else 0, _bias_dtype(bias),
            out.data_ptr(), out.stride(0) if M > 0 else N, M, N, K, ws_ptr, ws_bytes, stream)
    call = fast.gemm if fast is not None else lib.rla_w8a16_gemm
    if index == torch.cuda.current_device():
        st = call(*args)
    else:
        with torch.cuda.device(device):
            st = call(*args)
    if st != RLA_OK:
        _check(st, "rla_w8a16_gemm")
    return out


def w8a16_gemm_swiglu(x2d: torch.Tensor, w_gate: torch.Tensor, scale_gate: torch.Tensor, w_up: torch.Tensor,
                      scale_up: torch.Tensor, bias_gate=None, bias_up=None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """``y[M, N] = fp16(silu(g) * u)`` with ``g``, ``u`` the fp16 outputs of
    the gate and up W8A16 GEMMs, in one launch (``rla_w8a16_gemm_swiglu``).
    ``w_gate``/``w_up`` int8 ``[N, K]`` with the same row stride; scales
    (and biases) of one dtype."""
    lib = load_library()
    M, K = x2d.shape
    N = w_gate.shape[0]
    if w_up.shape != w_gate.shape or w_up.stride() != w_gate.stride():
        raise ValueError("w_gate and w_up must have the same shape and strides")
    if scale_up.dtype != scale_gate.dtype:
        raise TypeError("scale_gate and scale_up must have the same dtype")
    if (bias_gate is None) != (bias_up is None) or (bias_gate is not None and bias_gate.dtype != bias_up.dtype):
        raise TypeError("bias_gate and bias_up must both be given (same dtype) or both be None")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=x2d.device)
    index = x2d.device.index
    stream = torch._C._cuda_getCurrentRawStream(index)
    need = lib.rla_w8a16_swiglu_workspace_size(M, N, K)
    ws_ptr, ws_bytes = 0, 0
    if need:
        ws = _workspace(x2d.device, stream, need)
        ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    args = (x2d.data_ptr(), x2d.stride(0) if M > 0 else K, w_gate.data_ptr(), w_up.data_ptr(),
            w_gate.stride(0) if N > 0 else K, scale_gate.data_ptr(), scale_up.data_ptr(), _scale_dtype(scale_gate),
            bias_gate.data_ptr() if bias_gate is not None else 0,
            bias_up.data_ptr() if bias_up is not None else 0, _bias_dtype(bias_gate),
            out.data_ptr(), out.stride(0) if M > 0 else N, M, N, K, ws_ptr, ws_bytes, stream)
    call = _fast.gemm_swiglu if _fast is not None else lib.rla_w8a16_gemm_swiglu
    if index == torch.cuda.current_device():
        st = call(*args)
    else:
        with torch.cuda.device(x2d.device):
            st = call(*args)
    _check(st, "rla_w8a16_gemm_swiglu")
    return out


def rmsnorm(x2d: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp16 rows: ``fp16(x * rsqrt(mean(x^2) + eps) * weight)`` (``rla_rmsnorm``)."""
    lib = load_library()
    dt = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}.get(weight.dtype)
    if dt is None:
        raise TypeError(f"rmsnorm: unsupported weight dtype {weight.dtype}")
    w = weight if weight.is_contiguous() else weight.contiguous()
    M, K = x2d.shape
    if out is None:
        out = torch.empty((M, K), dtype=torch.float16, device=x2d.device)
    stream = torch.cuda.current_stream(x2d.device).cuda_stream
    with torch.cuda.device(x2d.device):
        st = lib.rla_rmsnorm(x2d.data_ptr(), x2d.stride(0) if M > 0 else K, w.data_ptr(), dt, float(eps),
                             out.data_ptr(), out.stride(0) if M > 0 else K, M, K, stream)
    _check(st, "rla_rmsnorm")
    return out


def quantize_per_channel(weight: torch.Tensor):
    """Device per-channel quantization through ``rla_quantize_per_channel``."""
    lib = load_library()
    dt = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}.get(weight.dtype)
    if dt is None:
        raise TypeError(f"quantize_per_channel: unsupported dtype {weight.dtype}")
    w = weight if weight.stride(-1) == 1 else weight.contiguous()
    N, K = w.shape
    q = torch.empty((N, K), dtype=torch.int8, device=w.device)
    s = torch.empty((N,), dtype=torch.float32, device=w.device)
    stream = torch.cuda.current_stream(w.device).cuda_stream
    with torch.cuda.device(w.device):
        st = lib.rla_quantize_per_channel(w.data_ptr(), dt, w.stride(0) if N > 0 else K, N, K, q.data_ptr(),
                                          K, s.data_ptr(), stream)
    _check(st, "rla_quantize_per_channel")
    return q, s


def gather_columns(staging: torch.Tensor, world: int, M: int, n_local: int, out: torch.Tensor) -> torch.Tensor:
    """``staging[world, M, n_local]`` -> ``out[M, world * n_local]``."""
    lib = load_library()
    stream = torch.cuda.current_stream(out.device).cuda_stream
    with torch.cuda.device(out.device):
        st = lib.rla_gather_columns(staging.data_ptr(), world, M, n_local, out.data_ptr(), out.stride(0), stream)
    _check(st, "rla_gather_columns")
    return out


def set_decode_kernel(name: str) -> None:
    """Force the decode (M <= 32) kernel family process-wide: "auto" (the
    selector's choice), "skinny" or "stream".  For A/B runs and tests."""
    kid = 0 if name == "auto" else KERNEL_IDS[name]
    _check(load_library().rla_set_decode_kernel(kid), "rla_set_decode_kernel")


def w8a16_gemm_allgather(x2d: torch.Tensor, weight_int8: torch.Tensor, scale: torch.Tensor, bias,
                         out: torch.Tensor, recv_ptrs, recv_bytes: int, sync_ptr: int, rank: int) -> torch.Tensor:
    """Column-parallel decode GEMM with the peer-to-peer all-gather fused in
    (``rla_w8a16_gemm_allgather``): this rank's slice ``[M, n_local]`` goes to
    columns ``[rank * n_local, (rank + 1) * n_local)`` of ``out`` and, as
    flagged words, into every peer's receive buffer; the peers' slices are
    unpacked from ``recv_ptrs[rank]`` into ``out``.  ``recv_ptrs``: every
    rank's receive buffer as mapped in this process.  Raises ``RlaError``
    (status 2) for shapes that are not decode shapes."""
    lib = load_library()
    M, K = x2d.shape
    n_local = weight_int8.shape[0]
    world = len(recv_ptrs)
    recv = (ctypes.c_void_p * world)(*recv_ptrs)
    stream = torch.cuda.current_stream(x2d.device).cuda_stream
    need = lib.rla_w8a16_allgather_workspace_size(M, n_local, K)
    ws_ptr, ws_bytes = None, 0
    if need:
        ws = _workspace(x2d.device, stream, need)
        ws_ptr, ws_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(x2d.device):
        st = lib.rla_w8a16_gemm_allgather(
            x2d.data_ptr(), x2d.stride(0), weight_int8.data_ptr(), weight_int8.stride(0), scale.data_ptr(),
            _scale_dtype(scale), bias.data_ptr() if bias is not None else None, _bias_dtype(bias),
            out.data_ptr(), out.stride(0), M, n_local, K, recv, recv_bytes, sync_ptr, rank, world,
            ws_ptr, ws_bytes, stream)
    _check(st, "rla_w8a16_gemm_allgather")
    return out


def prefill_exchange_begin(sync_ptrs, rank: int, stream: int) -> None:
    """Start of one pull-exchange call (``rla_prefill_exchange_begin``):
    advance the call number, wait until every peer finished reading this
    rank's exchange buffer in the previous call.  ``sync_ptrs``: every rank's
    sync area as mapped in this process."""
    world = len(sync_ptrs)
    syncs = (ctypes.c_void_p * world)(*sync_ptrs)
    _check(load_library().rla_prefill_exchange_begin(syncs, rank, world, stream), "rla_prefill_exchange_begin")


def prefill_exchange_block(xb_ptrs, ld_xb: int, sync_ptrs, rank: int, block: int, last: bool, row0: int, rows: int,
                           n_local: int, out: torch.Tensor, stream: int) -> None:
    """One block of the pull exchange (``rla_prefill_exchange_block``): mark
    this rank's block ready everywhere, wait for every rank's, copy every
    rank's slice of rows ``[row0, row0 + rows)`` into ``out``'s columns."""
    world = len(xb_ptrs)
    xbs = (ctypes.c_void_p * world)(*xb_ptrs)
    syncs = (ctypes.c_void_p * world)(*sync_ptrs)
    _check(load_library().rla_prefill_exchange_block(xbs, ld_xb, syncs, rank, world, block, 1 if last else 0, row0,
                                                     rows, n_local, out.data_ptr(), out.stride(0), stream),
           "rla_prefill_exchange_block")


def set_peer_wait_limit(seconds: float) -> None:
    """Limit of every wait inside the fused exchange (process-wide)."""
    _check(load_library().rla_set_peer_wait_limit(int(seconds * 1e9)), "rla_set_peer_wait_limit")


def peer_alloc(nbytes: int) -> int:
    """Zeroed device buffer with its own allocation (IPC-exportable as a whole)."""
    ptr = ctypes.c_void_p(0)
    _check(load_library().rla_peer_alloc(nbytes, ctypes.byref(ptr)), "rla_peer_alloc")
    return int(ptr.value)


def peer_free(ptr: int) -> None:
    _check(load_library().rla_peer_free(ptr), "rla_peer_free")


def ipc_export(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(load_library().rla_ipc_export(ptr, buf), "rla_ipc_export")
    return buf.raw


def ipc_open(handle: bytes) -> int:
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle has {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
    buf = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    ptr = ctypes.c_void_p(0)
    _check(load_library().rla_ipc_open(buf, ctypes.byref(ptr)), "rla_ipc_open")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _check(load_library().rla_ipc_close(ptr), "rla_ipc_close")


_sm_counts: dict = {}


def device_sm_count(index: int) -> int:
    """Streaming multiprocessors of CUDA device ``index`` (cached)."""
    n = _sm_counts.get(index)
    if n is None:
        n = _sm_counts[index] = torch.cuda.get_device_properties(index).multi_processor_count
    return n


def torch_op_loaded() -> bool:
    """Whether ``torch.ops.rla.w8a16_gemm`` is registered (``_rla_torch_ops.so``)."""
    load_library()
    return _torch_op is not None


def launch_count() -> int:
    return int(load_library().rla_launch_count())


def device_error() -> int:
    """Read and clear the device-side error word (synchronises)."""
    code = ctypes.c_uint(0)
    _check(load_library().rla_get_device_error(ctypes.byref(code)), "rla_get_device_error")
    return int(code.value)
