// Small kernels around the W8A16 GEMM: the any-shape fallback kernel, the
// K == 0 fill, per-channel int8 quantization and the column-parallel output
// assembly.
#include <cuda_bf16.h>

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
// ---------------------------------------------------------------------------
__global__ void w8a16_generic_kernel(const __half* __restrict__ x, int64_t ldx, const int8_t* __restrict__ w,
                                     int64_t ldw, const void* __restrict__ scale, int scale_f32,
                                     const void* __restrict__ bias, int bias_kind, __half* __restrict__ y,
                                     int64_t ldy, int M, int N, int K) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t mblocks = (M + 7) / 8;
  if (gw >= mblocks * N) return;
  const int n = static_cast<int>(gw % N);
  const int mb = static_cast<int>(gw / N);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  const int8_t* wr = w + static_cast<int64_t>(n) * ldw;
  for (int k = lane; k < K; k += 32) {
    const float wv = static_cast<float>(wr[k]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = mb * 8 + j;
      if (m < M) acc[j] = fmaf(__half2float(x[static_cast<int64_t>(m) * ldx + k]), wv, acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  if (lane == 0) {
    const float sc = load_scale(scale, scale_f32, n);
    const float bi = load_bias(bias, bias_kind, n);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = mb * 8 + j;
      if (m < M) y[static_cast<int64_t>(m) * ldy + n] = __float2half_rn(fmaf(acc[j], sc, bi));
    }
  }
}

cudaError_t launch_generic(const GemmArgs& a, cudaStream_t s) {
  const int64_t warps = (int64_t)((a.M + 7) / 8) * a.N;
  const int64_t blocks = (warps * 32 + 255) / 256;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  w8a16_generic_kernel<<<(unsigned)blocks, 256, 0, s>>>(static_cast<const __half*>(a.x), a.ldx, a.w, a.ldw,
                                                        a.scale, a.scale_f32, a.bias, a.bias_kind,
                                                        static_cast<__half*>(a.y), a.ldy, a.M, a.N, a.K);
  return cudaGetLastError();
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
      quantize_rows_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(w), ldw, (int)K, q, ldq, scale);
      break;
    case RLA_DTYPE_F16:
      quantize_rows_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(w), ldw, (int)K, q, ldq, scale);
      break;
    case RLA_DTYPE_BF16:
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
  if (vec)
    gather_columns_vec_kernel<<<(unsigned)blocks, 256, 0, s>>>(static_cast<const uint4*>(staging), world, M, nl / 8,
                                                               static_cast<uint4*>(y), ldy / 8);
  else
    gather_columns_kernel<<<(unsigned)blocks, 256, 0, s>>>(static_cast<const __half*>(staging), world, M, nl,
                                                           static_cast<__half*>(y), ldy);
  return cudaGetLastError();
}

}  // namespace rla
