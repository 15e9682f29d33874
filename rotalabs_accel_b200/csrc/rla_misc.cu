// Small kernels around the W8A16 GEMM: the any-shape fallback kernel, the
// K == 0 fill, per-channel int8 quantization and the column-parallel output
// assembly.
#include <cuda_bf16.h>

#include <algorithm>

#include "rla_common.cuh"
#include "rla_internal.h"

namespace rla {

__device__ __forceinline__ float load_scale(const void* p, int is_f32, int n) {
  return is_f32 ? static_cast<const float*>(p)[n] : __half2float(static_cast<const __half*>(p)[n]);
}
__device__ __forceinline__ float load_bias(const void* p, int kind, int n) {
  return kind == 0 ? 0.f : kind == 1 ? __half2float(static_cast<const __half*>(p)[n]) : static_cast<const float*>(p)[n];
}

// ---------------------------------------------------------------------------
// Generic W8A16 kernel: any K, any strides, any alignment.  One warp per
// (output channel n, block of 8 tokens); lanes stride over k, fp32
// accumulation, warp-shuffle reduction.  Used only for shapes the fast
// kernels' 16-byte vector / TMA rules exclude (ragged K, odd strides).
// Gated form (GLU): the warp also accumulates the up projection's row n and
// writes fp16(silu(gate) * up).
// ---------------------------------------------------------------------------
template <bool GLU>
__global__ void w8a16_generic_kernel(const __half* __restrict__ x, int64_t ldx, const int8_t* __restrict__ w,
                                     int64_t ldw, const void* __restrict__ scale, int scale_f32,
                                     const void* __restrict__ bias, int bias_kind, __half* __restrict__ y,
                                     int64_t ldy, int M, int N, int K, const int8_t* __restrict__ w_up,
                                     const void* __restrict__ scale_up, const void* __restrict__ bias_up) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t mblocks = (M + 7) / 8;
  if (gw >= mblocks * N) return;
  const int n = static_cast<int>(gw % N);
  const int mb = static_cast<int>(gw / N);
  float acc[8], accu[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = accu[j] = 0.f;
  const int8_t* wr = w + static_cast<int64_t>(n) * ldw;
  const int8_t* wu = GLU ? w_up + static_cast<int64_t>(n) * ldw : nullptr;
  for (int k = lane; k < K; k += 32) {
    const float wv = static_cast<float>(wr[k]);
    const float uv = GLU ? static_cast<float>(wu[k]) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = mb * 8 + j;
      if (m < M) {
        const float xv = __half2float(x[static_cast<int64_t>(m) * ldx + k]);
        acc[j] = fmaf(xv, wv, acc[j]);
        if (GLU) accu[j] = fmaf(xv, uv, accu[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
      if (GLU) accu[j] += __shfl_xor_sync(0xffffffffu, accu[j], o);
    }
  if (lane == 0) {
    const float sc = load_scale(scale, scale_f32, n);
    const float bi = load_bias(bias, bias_kind, n);
    const float scu = GLU ? load_scale(scale_up, scale_f32, n) : 0.f;
    const float biu = GLU ? load_bias(bias_up, bias_kind, n) : 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = mb * 8 + j;
      if (m >= M) continue;
      if (GLU)
        y[static_cast<int64_t>(m) * ldy + n] = rla_swiglu(fmaf(acc[j], sc, bi), fmaf(accu[j], scu, biu));
      else
        y[static_cast<int64_t>(m) * ldy + n] = __float2half_rn(fmaf(acc[j], sc, bi));
    }
  }
}

cudaError_t launch_generic(const GemmArgs& a, cudaStream_t s) {
  const int64_t warps = (int64_t)((a.M + 7) / 8) * a.N;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  auto kern = a.w_up ? w8a16_generic_kernel<true> : w8a16_generic_kernel<false>;
  rla_clear_stale_launch_error();
  kern<<<(unsigned)blocks, 256, 0, s>>>(static_cast<const __half*>(a.x), a.ldx, a.w, a.ldw, a.scale, a.scale_f32,
                                        a.bias, a.bias_kind, static_cast<__half*>(a.y), a.ldy, a.M, a.N, a.K,
                                        a.w_up, a.scale_up, a.bias_up);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// SwiGLU of two fp16 [M, N] tensors: y = fp16(silu(gate) * up) in fp32.  The
// prefill form of the gated GEMM (two tcgen05 GEMMs into the workspace, then
// this pass): a streaming kernel at full occupancy hides the latency of the
// exp / reciprocal that a GEMM epilogue with four warps cannot.
// ---------------------------------------------------------------------------
__global__ void swiglu_rows_kernel(const __half* __restrict__ gate, const __half* __restrict__ up, int64_t ld,
                                   __half* __restrict__ y, int64_t ldy, int M, int N, int vec) {
  const int64_t per_row = vec ? N / 8 : N;
  const int64_t total = per_row * M;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / per_row;
    const int64_t c = i - m * per_row;
    if (vec) {
      const uint4 g = *reinterpret_cast<const uint4*>(gate + m * ld + c * 8);
      const uint4 u = *reinterpret_cast<const uint4*>(up + m * ld + c * 8);
      const __half* gh = reinterpret_cast<const __half*>(&g);
      const __half* uh = reinterpret_cast<const __half*>(&u);
      uint4 o;
      __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int k = 0; k < 8; ++k) oh[k] = rla_swiglu(__half2float(gh[k]), __half2float(uh[k]));
      *reinterpret_cast<uint4*>(y + m * ldy + c * 8) = o;
    } else {
      y[m * ldy + c] = rla_swiglu(__half2float(gate[m * ld + c]), __half2float(up[m * ld + c]));
    }
  }
}

cudaError_t launch_swiglu(const void* gate, const void* up, int64_t ld, void* y, int64_t ldy, int M, int N,
                          cudaStream_t s) {
  const bool vec = N % 8 == 0 && ld % 8 == 0 && ldy % 8 == 0 && (reinterpret_cast<uintptr_t>(gate) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(up) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  const int64_t work = (vec ? (int64_t)N / 8 : (int64_t)N) * M;
  const int64_t blocks = std::min<int64_t>((work + 255) / 256, 148 * 16);
  rla_clear_stale_launch_error();
  swiglu_rows_kernel<<<(unsigned)std::max<int64_t>(blocks, 1), 256, 0, s>>>(
      static_cast<const __half*>(gate), static_cast<const __half*>(up), ld, static_cast<__half*>(y), ldy, M, N,
      vec ? 1 : 0);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// RMSNorm of fp16 rows, the arithmetic of rotalabs-accel's CUDA RMSNorm
// (kernels/normalization.py:66-101): per row, the mean of x^2 in fp32,
// rrms = rsqrt(mean + eps), y = fp16(x * rrms * w) computed in fp32.  One CTA
// per row; 16-byte loads when the row is aligned.  Launched with
// programmatic dependent launch, so the next GEMM's prologue overlaps it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_weight(const void* w, int dtype, int k) {
  return dtype == RLA_DTYPE_F32  ? static_cast<const float*>(w)[k]
         : dtype == RLA_DTYPE_F16 ? __half2float(static_cast<const __half*>(w)[k])
                                  : __bfloat162float(static_cast<const __nv_bfloat16*>(w)[k]);
}

__global__ void rmsnorm_rows_kernel(const __half* __restrict__ x, int64_t ldx, const void* __restrict__ weight,
                                    int weight_dtype, float eps, __half* __restrict__ y, int64_t ldy, int K,
                                    int vec) {
  // Programmatic dependent launch: the GEMM that follows (the MLP block's
  // gate/up projection) may start now and stream its weights while this
  // kernel runs; it reads y only after this grid completes.  Nothing is read
  // or written here before the previous kernel in the stream has finished.
  rla_griddep_launch_dependents();
  rla_griddep_wait();
  const __half* xr = x + static_cast<int64_t>(blockIdx.x) * ldx;
  __half* yr = y + static_cast<int64_t>(blockIdx.x) * ldy;
  float ss = 0.f;
  if (vec) {
    for (int k = threadIdx.x * 8; k < K; k += blockDim.x * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
      const float f = __half2float(xr[k]);
      ss = fmaf(f, f, ss);
    }
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rrms = rsqrtf(red[0] / static_cast<float>(K) + eps);
  if (vec) {
    for (int k = threadIdx.x * 8; k < K; k += blockDim.x * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
      const __half2* h = reinterpret_cast<const __half2*>(&v);
      uint4 o;
      __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        oh[i] = __floats2half2_rn(f.x * rrms * load_weight(weight, weight_dtype, k + 2 * i),
                                  f.y * rrms * load_weight(weight, weight_dtype, k + 2 * i + 1));
      }
      *reinterpret_cast<uint4*>(yr + k) = o;
    }
  } else {
    for (int k = threadIdx.x; k < K; k += blockDim.x)
      yr[k] = __float2half_rn(__half2float(xr[k]) * rrms * load_weight(weight, weight_dtype, k));
  }
}

cudaError_t launch_rmsnorm(const void* x, int64_t ldx, const void* weight, int weight_dtype, float eps, void* y,
                           int64_t ldy, int M, int K, cudaStream_t s) {
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  const int threads = K >= 4096 ? 512 : 256;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)M);
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rmsnorm_rows_kernel, static_cast<const __half*>(x), ldx, weight, weight_dtype, eps,
                            static_cast<__half*>(y), ldy, K, vec ? 1 : 0);
}

// K == 0: the empty sum; y = bias (or 0).
__global__ void w8a16_fill_kernel(const void* __restrict__ bias, int bias_kind, __half* __restrict__ y, int64_t ldy,
                                  int M, int N) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(M) * N) return;
  const int n = static_cast<int>(i % N);
  const int m = static_cast<int>(i / N);
  y[static_cast<int64_t>(m) * ldy + n] = __float2half_rn(load_bias(bias, bias_kind, n));
}

cudaError_t launch_fill(const GemmArgs& a, cudaStream_t s) {
  const int64_t total = static_cast<int64_t>(a.M) * a.N;
  rla_clear_stale_launch_error();
  w8a16_fill_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(a.bias, a.bias_kind,
                                                                     static_cast<__half*>(a.y), a.ldy, a.M, a.N);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Per-output-channel symmetric quantization, bit-identical to the CPU path:
//   scale = T(max|w_row| / 127)      (T = the input dtype; the quotient is
//                                     computed in fp32 and rounded to T, as
//                                     torch does for fp16 / bf16 tensors)
//   scale = 1 where scale == 0
//   q = clamp(rint(T(w / scale)), -128, 127)   (rint: round half to even)
// One CTA per row: a max-reduction pass, then a quantize pass.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ float round_to_t(float v);
template <>
__device__ __forceinline__ float round_to_t<float>(float v) { return v; }
template <>
__device__ __forceinline__ float round_to_t<__half>(float v) { return __half2float(__float2half_rn(v)); }
template <>
__device__ __forceinline__ float round_to_t<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

template <typename T>
__global__ void quantize_rows_kernel(const T* __restrict__ w, int64_t ldw, int K, int8_t* __restrict__ q,
                                     int64_t ldq, float* __restrict__ scale_out) {
  const int64_t row = blockIdx.x;
  const T* wr = w + row * ldw;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_f<T>(wr[k])));
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  // max|w| is exact in T; the division is IEEE fp32 (round to nearest),
  // then rounded to T.
  float sc = round_to_t<T>(__fdiv_rn(red[0], 127.0f));
  if (sc == 0.f) sc = 1.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float r = rintf(round_to_t<T>(__fdiv_rn(to_f<T>(wr[k]), sc)));
    q[row * ldq + k] = static_cast<int8_t>(fminf(fmaxf(r, -128.f), 127.f));
  }
  if (threadIdx.x == 0) scale_out[row] = sc;
}

cudaError_t launch_quantize(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int8_t* q, int64_t ldq,
                            float* scale, cudaStream_t s) {
  const unsigned blocks = static_cast<unsigned>(N);
  switch (w_dtype) {
    case RLA_DTYPE_F32:
      rla_clear_stale_launch_error();
      quantize_rows_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(w), ldw, (int)K, q, ldq, scale);
      break;
    case RLA_DTYPE_F16:
      rla_clear_stale_launch_error();
      quantize_rows_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(w), ldw, (int)K, q, ldq, scale);
      break;
    case RLA_DTYPE_BF16:
      rla_clear_stale_launch_error();
      quantize_rows_kernel<__nv_bfloat16>
          <<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), ldw, (int)K, q, ldq, scale);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Column-parallel output assembly: staging[r][m][j] -> y[m][r * n_local + j].
// 16-byte vectors when every row boundary is 16-byte aligned, else halves.
// ---------------------------------------------------------------------------
__global__ void gather_columns_vec_kernel(const uint4* __restrict__ staging, int64_t world, int64_t M,
                                          int64_t nl_vec, uint4* __restrict__ y, int64_t ldy_vec) {
  const int64_t total = world * M * nl_vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = i % nl_vec;
    const int64_t m = (i / nl_vec) % M;
    const int64_t r = i / (nl_vec * M);
    y[m * ldy_vec + r * nl_vec + j] = staging[i];
  }
}
__global__ void gather_columns_kernel(const __half* __restrict__ staging, int64_t world, int64_t M, int64_t nl,
                                      __half* __restrict__ y, int64_t ldy) {
  const int64_t total = world * M * nl;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = i % nl;
    const int64_t m = (i / nl) % M;
    const int64_t r = i / (nl * M);
    y[m * ldy + r * nl + j] = staging[i];
  }
}

cudaError_t launch_gather(const void* staging, int64_t world, int64_t M, int64_t nl, void* y, int64_t ldy,
                          cudaStream_t s) {
  const bool vec = (nl % 8 == 0) && (ldy % 8 == 0) && ((reinterpret_cast<uintptr_t>(staging) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(y) & 15) == 0);
  const int64_t elems = vec ? world * M * (nl / 8) : world * M * nl;
  int64_t blocks = (elems + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  rla_clear_stale_launch_error();
  if (vec)
    gather_columns_vec_kernel<<<(unsigned)blocks, 256, 0, s>>>(static_cast<const uint4*>(staging), world, M, nl / 8,
                                                               static_cast<uint4*>(y), ldy / 8);
  else
    gather_columns_kernel<<<(unsigned)blocks, 256, 0, s>>>(static_cast<const __half*>(staging), world, M, nl,
                                                           static_cast<__half*>(y), ldy);
  return cudaGetLastError();
}

}  // namespace rla
