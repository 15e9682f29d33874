// torch.library registration of the W8A16 GEMM: rla::w8a16_gemm.
//
// A thin C++ layer over the C ABI of include/rla_w8a16.h (rla_w8a16_gemm):
// it checks the tensors, allocates the fp16 output with torch's caching
// allocator on the input's device, picks the current torch CUDA stream and a
// per-(device, stream) split-K workspace, and calls the library.  No
// arithmetic happens here.  It replaces the launcher of rotalabs-accel's
// Triton path (src/rotalabs_accel/kernels/gemm.py:140-186, called from
// int8_gemm at :232) for 2-D fp16 activations; the Python int8_gemm keeps the
// reference's shape handling around it.
//
//   rla::w8a16_gemm(Tensor x, Tensor weight_int8, Tensor scale, Tensor? bias=None) -> Tensor
//     x       fp16 [M, K], unit inner stride (any row stride)
//     weight  int8 [N, K], unit inner stride
//     scale   fp32 or fp16 [N], contiguous
//     bias    fp16 or fp32 [N], contiguous, or None
//     -> fp16 [M, N], contiguous
//
// The Meta kernel gives the output's shape and dtype without computing, so
// the op traces under FakeTensor / torch.compile as an opaque call.
//
// The same file is also a Python extension module (_rla_torch_ops) whose
// w8a16_gemm calls the CUDA kernel function directly: the per-token hot path
// (Int8Linear.forward) takes it to skip the dispatcher's schema parsing and
// dispatch, a few microseconds of host time per call.  Same checks, same
// launch, same result as the op.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/rla_w8a16.h"

namespace {

// Split-K workspaces, one per (device, stream), zero-filled when made and
// grown on demand.  Calls on one stream are ordered, so they share it.
at::Tensor workspace_for(const at::Device& dev, cudaStream_t stream, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, at::Tensor> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto& ws = cache[{dev.index(), stream}];
  if (!ws.defined() || static_cast<size_t>(ws.numel()) < bytes) {
    const int64_t n = static_cast<int64_t>(bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes);
    ws = at::zeros({n}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  return ws;
}

void check_args(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale,
                const std::optional<at::Tensor>& bias) {
  TORCH_CHECK(x.dim() == 2 && x.scalar_type() == at::kHalf, "rla::w8a16_gemm: x must be a 2-D float16 tensor");
  TORCH_CHECK(w.dim() == 2 && w.scalar_type() == at::kChar, "Weight must be INT8");
  TORCH_CHECK(w.size(1) == x.size(1), "Weight shape mismatch: ", w.sizes(), " vs (", w.size(0), ", ", x.size(1), ")");
  TORCH_CHECK(scale.dim() == 1 && scale.size(0) == w.size(0), "Scale shape mismatch: ", scale.sizes(), " vs (",
              w.size(0), ",)");
  TORCH_CHECK(scale.scalar_type() == at::kFloat || scale.scalar_type() == at::kHalf,
              "rla::w8a16_gemm: scale must be float32 or float16");
  if (bias.has_value()) {
    TORCH_CHECK(bias->dim() == 1 && bias->size(0) == w.size(0), "rla::w8a16_gemm: bias must be [N]");
    TORCH_CHECK(bias->scalar_type() == at::kHalf || bias->scalar_type() == at::kFloat,
                "rla::w8a16_gemm: bias must be float16 or float32");
  }
}

at::Tensor w8a16_gemm_cuda(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale,
                           const std::optional<at::Tensor>& bias) {
  check_args(x, w, scale, bias);
  const at::Device dev = x.device();
  TORCH_CHECK(dev.is_cuda() && w.device() == dev && scale.device() == dev &&
                  (!bias.has_value() || bias->device() == dev),
              "rla::w8a16_gemm: all tensors must be on the same CUDA device");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(M == 0 || K == 0 || x.stride(1) == 1, "rla::w8a16_gemm: x needs a unit inner stride");
  TORCH_CHECK(N == 0 || K == 0 || w.stride(1) == 1, "rla::w8a16_gemm: weight_int8 needs a unit inner stride");
  TORCH_CHECK(scale.is_contiguous(), "rla::w8a16_gemm: scale must be contiguous");
  TORCH_CHECK(!bias.has_value() || bias->is_contiguous(), "rla::w8a16_gemm: bias must be contiguous");
  c10::cuda::CUDAGuard guard(dev);
  at::Tensor y = at::empty({M, N}, x.options());
  if (M == 0 || N == 0) return y;
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  const size_t need = rla_w8a16_workspace_size(M, N, K);
  void* ws_ptr = nullptr;
  size_t ws_bytes = 0;
  if (need) {
    at::Tensor ws = workspace_for(dev, stream, need);
    ws_ptr = ws.data_ptr();
    ws_bytes = static_cast<size_t>(ws.numel());
  }
  const int sdt = scale.scalar_type() == at::kFloat ? RLA_DTYPE_F32 : RLA_DTYPE_F16;
  const int bdt = !bias.has_value() ? RLA_DTYPE_NONE : bias->scalar_type() == at::kFloat ? RLA_DTYPE_F32 : RLA_DTYPE_F16;
  const int st = rla_w8a16_gemm(x.data_ptr(), K > 0 ? x.stride(0) : 0, static_cast<const int8_t*>(w.data_ptr()),
                                K > 0 ? w.stride(0) : 0, scale.data_ptr(), sdt,
                                bias.has_value() ? bias->data_ptr() : nullptr, bdt, y.data_ptr(), N, M, N, K,
                                ws_ptr, ws_bytes, stream);
  TORCH_CHECK(st == RLA_OK, "rla_w8a16_gemm failed with status ", st, ": ", rla_last_error());
  return y;
}

at::Tensor w8a16_gemm_meta(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scale,
                           const std::optional<at::Tensor>& bias) {
  check_args(x, w, scale, bias);
  return at::empty({x.size(0), w.size(0)}, x.options());
}

}  // namespace

PYBIND11_MODULE(_rla_torch_ops, m) {
  m.def("w8a16_gemm", &w8a16_gemm_cuda, "rla::w8a16_gemm's CUDA kernel function, called without the dispatcher",
        pybind11::arg("x"), pybind11::arg("weight_int8"), pybind11::arg("scale"),
        pybind11::arg("bias") = pybind11::none());
}

TORCH_LIBRARY(rla, m) {
  m.def("w8a16_gemm(Tensor x, Tensor weight_int8, Tensor scale, Tensor? bias=None) -> Tensor");
}
TORCH_LIBRARY_IMPL(rla, CUDA, m) { m.impl("w8a16_gemm", &w8a16_gemm_cuda); }
TORCH_LIBRARY_IMPL(rla, Meta, m) { m.impl("w8a16_gemm", &w8a16_gemm_meta); }
