// Host side of the direct peer-to-peer all-gather epilogue: device buffers
// with their own allocation (so an IPC handle covers exactly one buffer), IPC
// export / open, and rla_w8a16_gemm_allgather, which runs the decode kernels
// with a PeerOut: each rank's slice goes into its own output and, as flagged
// words, into every peer's receive buffer; the last CTAs unpack the peers'
// slices.  The device protocol is in rla_peer.cuh.
#include <string.h>

#include <atomic>

#include "rla_internal.h"

namespace rla {
// One second, like the pipeline waits inside the decode kernels.
static std::atomic<unsigned long long> g_peer_wait_ns{1000000000ull};
}  // namespace rla

extern "C" {

int rla_set_peer_wait_limit(uint64_t ns) {
  using namespace rla;
  if (ns < 1000000ull || ns > 60000000000ull) {
    set_error("rla_set_peer_wait_limit: limit must be in [1 ms, 60 s], got %llu ns", (unsigned long long)ns);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  g_peer_wait_ns.store(ns, std::memory_order_relaxed);
  return RLA_OK;
}

int rla_peer_alloc(size_t bytes, void** ptr) {
  using namespace rla;
  if (!ptr || bytes == 0) {
    set_error("rla_peer_alloc: need bytes > 0 and a result pointer");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // zeroed before any peer can map it
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_error("rla_peer_alloc(%zu): %s", bytes, cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  *ptr = p;
  return RLA_OK;
}

int rla_peer_free(void* ptr) {
  using namespace rla;
  if (!ptr) return RLA_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("rla_peer_free: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  return RLA_OK;
}

int rla_ipc_export(const void* ptr, void* handle) {
  using namespace rla;
  static_assert(sizeof(cudaIpcMemHandle_t) == RLA_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) {
    set_error("rla_ipc_export: null pointer");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) {
    set_error("rla_ipc_export: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  return RLA_OK;
}

int rla_ipc_open(const void* handle, void** ptr) {
  using namespace rla;
  if (!handle || !ptr) {
    set_error("rla_ipc_open: null pointer");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_error("rla_ipc_open: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  return RLA_OK;
}

int rla_ipc_close(void* ptr) {
  using namespace rla;
  if (!ptr) return RLA_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_error("rla_ipc_close: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  return RLA_OK;
}

size_t rla_w8a16_allgather_workspace_size(int64_t M, int64_t n_local, int64_t K) {
  using namespace rla;
  if (M < 0 || n_local < 0 || K < 0) return 0;
  return make_plan(M, n_local, K, true, true, /*peer=*/true).workspace;
}

int rla_w8a16_gemm_allgather(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                             int scale_dtype, const void* bias, int bias_dtype, void* y, int64_t ldy, int64_t M,
                             int64_t n_local, int64_t K, void* const* recv_peers, size_t recv_bytes, void* sync,
                             int rank, int world, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace rla;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) {
    set_error("rla_w8a16_gemm_allgather: need 1 <= world <= %d and 0 <= rank < world (got rank %d, world %d)",
              kMaxPeers, rank, world);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (M < 0 || n_local < 0 || K < 0 || M > INT32_MAX || n_local > INT32_MAX || K > INT32_MAX) {
    set_error("rla_w8a16_gemm_allgather: M, n_local, K must be in [0, 2^31)");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (!recv_peers || !sync || !y || (reinterpret_cast<uintptr_t>(sync) & 127u)) {
    set_error("rla_w8a16_gemm_allgather: need y, a host array of %d receive buffers and a 128-byte aligned "
              "sync area", world);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  for (int d = 0; d < world; ++d)
    if (!recv_peers[d] || (reinterpret_cast<uintptr_t>(recv_peers[d]) & 15u)) {
      set_error("rla_w8a16_gemm_allgather: receive buffer %d is null or not 16-byte aligned", d);
      return RLA_ERR_INVALID_ARGUMENT;
    }
  if (scale_dtype != RLA_DTYPE_F16 && scale_dtype != RLA_DTYPE_F32) {
    set_error("rla_w8a16_gemm_allgather: scale_dtype must be F16 or F32");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (bias_dtype != RLA_DTYPE_NONE && bias_dtype != RLA_DTYPE_F16 && bias_dtype != RLA_DTYPE_F32) {
    set_error("rla_w8a16_gemm_allgather: bias_dtype must be NONE, F16 or F32");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if ((bias_dtype != RLA_DTYPE_NONE && !bias) || !x || !w || !scale) {
    set_error("rla_w8a16_gemm_allgather: null x, w, scale or bias");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (ldy < (int64_t)world * n_local || ldx < K || ldw < K) {
    set_error("rla_w8a16_gemm_allgather: need ldy >= world * n_local, ldx >= K, ldw >= K");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u)) {
    set_error("rla_w8a16_gemm_allgather: workspace must be 256-byte aligned");
    return RLA_ERR_WORKSPACE;
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                       ldx % 8 == 0 && ldw % 16 == 0;
  if (M < 1 || M > 32 || n_local < 1 || K == 0 || K % 16 != 0 || !aligned) {
    set_error("rla_w8a16_gemm_allgather: only decode shapes are fused (1 <= M <= 32, n_local >= 1, "
              "K %% 16 == 0, 16-byte aligned x and w, ldx %% 8 == 0, ldw %% 16 == 0; got M=%lld n_local=%lld K=%lld)",
              (long long)M, (long long)n_local, (long long)K);
    return RLA_ERR_UNSUPPORTED;
  }
  const int64_t slot_words = ((M + 1) / 2) * n_local;
  if ((int64_t)world * slot_words >= (int64_t(1) << 32)) {
    set_error("rla_w8a16_gemm_allgather: %d ranks x %lld flagged words per slice exceed 2^32",
              world, (long long)slot_words);
    return RLA_ERR_UNSUPPORTED;
  }
  const int64_t half_words = static_cast<int64_t>(recv_bytes / 16);
  if ((int64_t)world * slot_words > half_words) {
    set_error("rla_w8a16_gemm_allgather: receive buffers of %zu bytes hold less than 2 x %d x %lld flagged words",
              recv_bytes, world, (long long)slot_words);
    return RLA_ERR_WORKSPACE;
  }
  // planned with the exchange kernel's own occupancy (it holds more
  // registers than the plain kernel, so fewer of its CTAs fit per SM)
  Plan p = make_plan(M, n_local, K, true, workspace != nullptr && workspace_bytes > 0, /*peer=*/true);
  if (p.workspace > workspace_bytes) p = make_plan(M, n_local, K, true, false, /*peer=*/true);
  if (p.kernel != RLA_KERNEL_SKINNY && p.kernel != RLA_KERNEL_STREAM) {
    set_error("rla_w8a16_gemm_allgather: the plan for this shape is not a decode kernel");
    return RLA_ERR_UNSUPPORTED;
  }

  GemmArgs a{x, ldx, w, ldw, scale, scale_dtype == RLA_DTYPE_F32 ? 1 : 0, bias,
             bias_dtype == RLA_DTYPE_NONE ? 0 : bias_dtype == RLA_DTYPE_F16 ? 1 : 2,
             y, ldy, (int)M, (int)n_local, (int)K};
  for (int d = 0; d < world; ++d) a.peer.recv[d] = static_cast<uint2*>(recv_peers[d]);
  a.peer.sync = static_cast<unsigned int*>(sync);
  a.peer.half_words = half_words;
  a.peer.slot_words = slot_words;
  a.peer.wait_ns = g_peer_wait_ns.load(std::memory_order_relaxed);
  a.peer.unpackers = 0;  // set by the launcher from its grid and occupancy
  a.peer.world = world;
  a.peer.rank = rank;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = p.kernel == RLA_KERNEL_STREAM ? launch_stream(a, p, workspace, s)
                                                      : launch_skinny(a, p, workspace, s);
  if (e != cudaSuccess) {
    set_error("rla_w8a16_gemm_allgather: launch of kernel family %d failed: %s", p.kernel, cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

}  // extern "C"
