// Allocation-free decode GEMM: the split-K decode kernel (rla_skinny.cu) with
// its scratch in a file-scope device array instead of a caller workspace.
//
// Who needs this: code that must not allocate GPU memory on the path that
// runs the GEMM.  cudaMalloc can synchronise the device (stalling every
// stream, which a serving loop cannot afford between decode steps), it can
// fail once a process has reserved its memory up front for a KV cache or a
// custom pool, and some host frameworks (plugin or "enqueue" callbacks of
// inference runtimes) hand a kernel no workspace and forbid allocation in the
// call.  Such callers still pass x, w, scale, bias and y; the split-K partial
// sums and arrival counters live in `rla_noalloc_scratch` below.
//
// Contract:
//   * capacity: kNoAllocScratchBytes (1 MiB) per GPU, held by every GPU that
//     loads the library until the process exits.  A shape whose plan needs
//     more is rejected with RLA_ERR_WORKSPACE (nothing launched).
//   * the first call on a device sets up that device: it looks up the array's
//     device address (cudaGetSymbolAddress) and zeroes its counter region on
//     the caller's stream.  Make that first call before any stream capture.
//   * every call shares the one array and leaves the last call's contents in
//     it.  The counters are back at zero after each call; the partial sums are
//     always written before they are read.  Calls that overlap on the GPU
//     (other streams, other host threads) race on the array and must be
//     ordered by the caller.
//   * no cudaMalloc, cudaFree or other allocating routine is called.
#include <mutex>

#include "rla_common.cuh"
#include "rla_internal.h"

namespace rla {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB
constexpr int kNoAllocMaxDevices = 128;

static __device__ __align__(256) unsigned char rla_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mutex;
static void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (set up on the
// first call per device).  In host code `rla_noalloc_scratch` is only a
// host-side stand-in, never a device address, so kernels get this pointer.
static int noalloc_scratch_for_current_device(cudaStream_t stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("rla_w8a16_gemm_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return RLA_ERR_DEVICE;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    set_error("rla_w8a16_gemm_noalloc: device index %d out of range", dev);
    return RLA_ERR_DEVICE;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, rla_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("rla_w8a16_gemm_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return RLA_ERR_CUDA;
    }
    e = cudaMemsetAsync(p, 0, kSplitCounterBytes, stream);  // counters start at zero
    if (e != cudaSuccess) {
      set_error("rla_w8a16_gemm_noalloc: clearing the counters: %s", cudaGetErrorString(e));
      return RLA_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return RLA_OK;
}

}  // namespace rla

extern "C" int rla_w8a16_gemm_noalloc(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                                      int scale_dtype, const void* bias, int bias_dtype, void* y, int64_t ldy,
                                      int64_t M, int64_t N, int64_t K, void* stream) {
  using namespace rla;
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) {
    set_error("rla_w8a16_gemm_noalloc: M, N, K must be in [0, 2^31)");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (M == 0 || N == 0) return RLA_OK;
  if (scale_dtype != RLA_DTYPE_F16 && scale_dtype != RLA_DTYPE_F32) {
    set_error("rla_w8a16_gemm_noalloc: scale_dtype must be F16 or F32");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (bias_dtype != RLA_DTYPE_NONE && bias_dtype != RLA_DTYPE_F16 && bias_dtype != RLA_DTYPE_F32) {
    set_error("rla_w8a16_gemm_noalloc: bias_dtype must be NONE, F16 or F32");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if ((bias_dtype != RLA_DTYPE_NONE && !bias) || !x || !w || !scale || !y) {
    set_error("rla_w8a16_gemm_noalloc: null pointer");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (ldy < N || ldx < K || ldw < K) {
    set_error("rla_w8a16_gemm_noalloc: leading dimensions must be >= the row length");
    return RLA_ERR_INVALID_ARGUMENT;
  }
  const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0 &&
                       ldx % 8 == 0 && ldw % 16 == 0;
  if (M > 32 || K == 0 || K % 16 != 0 || !aligned) {
    set_error("rla_w8a16_gemm_noalloc: only the decode kernel is allocation-free: needs 1 <= M <= 32, "
              "K %% 16 == 0, 16-byte aligned x and w, ldx %% 8 == 0, ldw %% 16 == 0 (got M=%lld K=%lld)",
              (long long)M, (long long)K);
    return RLA_ERR_UNSUPPORTED;
  }
  Plan p;
  skinny_shape(p, M, N, K, /*have_ws=*/true, device_sm_count());
  if (p.workspace > kNoAllocScratchBytes) {
    set_error("rla_w8a16_gemm_noalloc: this shape needs %zu bytes of split-K scratch; the static scratch "
              "holds %zu bytes (M=%lld N=%lld K=%lld); use rla_w8a16_gemm with a workspace",
              p.workspace, kNoAllocScratchBytes, (long long)M, (long long)N, (long long)K);
    return RLA_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  const int st = noalloc_scratch_for_current_device(s, &scratch);  // set-up on the first call per device
  if (st != RLA_OK) return st;
  GemmArgs a{x, ldx, w, ldw, scale, scale_dtype == RLA_DTYPE_F32 ? 1 : 0, bias,
             bias_dtype == RLA_DTYPE_NONE ? 0 : bias_dtype == RLA_DTYPE_F16 ? 1 : 2,
             y, ldy, (int)M, (int)N, (int)K};
  const cudaError_t e = launch_skinny(a, p, scratch, s);
  if (e != cudaSuccess) {
    set_error("rla_w8a16_gemm_noalloc: launch failed: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}
