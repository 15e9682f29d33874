// Decode-regime W8A16 kernel (M <= 32): stream the int8 weight once from HBM.
//
// Work split.  A CTA owns 16*WN consecutive weight rows (output channels n)
// and one slice of K (split-K across CTAs when gridDim.y > 1).  Inside the
// CTA, warp (wn, wk) owns rows [16*wn, 16*wn + 16) and every WK-th 64-wide
// chunk of the CTA's K slice.  Partial sums of the WK warps are added in
// shared memory in a fixed order; partial sums of the CTAs along K go
// through the caller's workspace and are added, again in a fixed order, by
// whichever CTA of the row block finishes last.  Results are therefore
// bit-reproducible from run to run.
//
// Inner product on the tensor cores, "swap-AB": the weight rows are the MMA
// rows (m16) and the <= 8*NT activation rows are the MMA columns (n8), so a
// 16x8x16 MMA carries 16 output channels of up to 8 tokens.  Because a dot
// product does not care in which order its k terms are visited, each lane
// loads 16 *contiguous* weight bytes per row with one 128-bit load and the
// k order inside the MMA fragment is permuted to match; the activation
// fragment is loaded with the same permutation (32 contiguous bytes of x).
// Lane (g = lane/4, q = lane%4) of a chunk starting at kb covers
// k in [kb + 16q, kb + 16q + 16) for weight rows g and g+8 and x row g:
//   MMA step s (0..3), fragment k columns {2q, 2q+1} <- k = kb+16q+4s+{0,1}
//                                         {2q+8, 2q+9} <- k = kb+16q+4s+{2,3}
// int8 -> fp16 happens in registers (rla_i8x4_to_h2x2).
//
// Launched with programmatic dependent launch: a CTA warms L2 with its first
// weight bytes while the previous kernel in the stream finishes, and reads
// nothing before that kernel is done (rla_griddep_wait).
//
// Gated form (GLU, rla_w8a16_gemm_swiglu): a warp's 16 MMA rows are 8 gate
// rows (A rows 0-7) and the same 8 rows of the up projection (A rows 8-15),
// so one lane holds gate and up of the same output and the epilogue computes
// fp16(silu(gate) * up) in registers; a CTA covers 8 * WN outputs.
//
// With a peer exchange (PEER, rla_w8a16_gemm_allgather) the epilogue stores
// pairs of rows into y and, as flagged words, into every peer's receive
// buffer, and every CTA ends with peer_finish (rla_peer.cuh).
#include <atomic>

#include "rla_common.cuh"
#include "rla_internal.h"
#include "rla_peer.cuh"

namespace rla {

template <int NT>
struct XFrag {
  uint4 v[NT][2];
};

// One 64-wide k chunk of a warp: rows g and g+8 (wa[0], wa[1]: 16 int8 each)
// times the chunk's activation fragments, four m16n8k16 steps per 8-token tile.
template <int NT>
RLA_DEVFN void skinny_chunk_mma(float (&acc)[NT][4], const uint4 (&wa)[2], const XFrag<NT>& xb) {
  const uint32_t* w0 = reinterpret_cast<const uint32_t*>(&wa[0]);
  const uint32_t* w1 = reinterpret_cast<const uint32_t*>(&wa[1]);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    uint32_t a0, a1, a2, a3;
    rla_i8x4_to_h2x2(w0[s], a0, a2);  // row g:   k {2q,2q+1} and {2q+8,2q+9}
    rla_i8x4_to_h2x2(w1[s], a1, a3);  // row g+8
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xb.v[t][0]);
      rla_mma_16816(acc[t], a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
    }
  }
}

// The unpacking phase of the exchange form: out of line for two or more
// token tiles (see peer_finish_call).
template <int NT>
RLA_DEVFN void skinny_peer_finish(const PeerOut& po, unsigned int s, __half* y, int64_t ldy, int M, int N, int* slot) {
  if constexpr (NT >= 2)
    peer_finish_call(po, s, y, ldy, M, N, threadIdx.x, blockDim.x, 0, slot);
  else
    peer_finish(po, s, y, ldy, M, N, threadIdx.x, blockDim.x, 0, slot);
}

template <int NT, int WN, int WK, int U, bool PEER, bool GLU, bool XJ>
RLA_DEVFN void skinny_body(const __half* __restrict__ x, int64_t ldx, const int8_t* __restrict__ w, int64_t ldw,
                           const void* __restrict__ scale, int scale_f32, const void* __restrict__ bias,
                           int bias_kind, __half* __restrict__ y, int64_t ldy, int M, int N, int K,
                           int chunks_per_split, float* __restrict__ partial, unsigned int* __restrict__ counters,
                           const PeerOut& po, const int8_t* __restrict__ w_up, const void* __restrict__ scale_up,
                           const void* __restrict__ bias_up) {
  static_assert(!(PEER && GLU), "the gated form has no peer exchange");
  constexpr int OUTS = GLU ? 8 * WN : 16 * WN;  // output channels per CTA
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int wn = warp % WN;
  const int wk = warp / WN;
  const int g = lane >> 2;
  const int q = lane & 3;

  const int row_base = blockIdx.x * OUTS;
  const int n0 = row_base + wn * (GLU ? 8 : 16);
  const int r0 = min(n0 + g, N - 1);
  const int r1 = GLU ? r0 : min(n0 + g + 8, N - 1);
  const int8_t* wrow0 = w + (int64_t)r0 * ldw + q * 16;
  const int8_t* wrow1 = (GLU ? w_up : w) + (int64_t)r1 * ldw + q * 16;

  bool xrow_ok[NT];
  const __half* xrow[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int xr = t * 8 + g;
    xrow_ok[t] = xr < M;
    xrow[t] = x + (int64_t)(xrow_ok[t] ? xr : 0) * ldx + q * 16;
  }

  const int total_chunks = (K + 63) >> 6;
  const int c_begin = blockIdx.y * chunks_per_split;
  const int c_end = min(total_chunks, c_begin + chunks_per_split);

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

  // Let the next launch in the stream start, warm L2 with this lane's first
  // batch of weight bytes (and k-warp 0 with the scales and biases of its
  // outputs, read by the epilogue), then wait for the predecessor before any
  // real read.
  rla_griddep_launch_dependents();
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int cc = c_begin + wk + u * WK;
    if (cc < c_end && cc * 64 + q * 16 < K) {
      rla_prefetch_l2(wrow0 + cc * 64);
      rla_prefetch_l2(wrow1 + cc * 64);
    }
  }
  if (wk == 0 && q == 0) {
    const int esz = scale_f32 ? 4 : 2, bsz = bias_kind == 2 ? 4 : 2;
    rla_prefetch_l2(static_cast<const char*>(scale) + (int64_t)r0 * esz);
    rla_prefetch_l2(static_cast<const char*>(GLU ? scale_up : scale) + (int64_t)r1 * esz);
    if (bias_kind != 0) {
      rla_prefetch_l2(static_cast<const char*>(bias) + (int64_t)r0 * bsz);
      rla_prefetch_l2(static_cast<const char*>(GLU ? bias_up : bias) + (int64_t)r1 * bsz);
    }
  }
  rla_griddep_wait();
  unsigned int call = 0;
  if constexpr (PEER) call = peer_call(po);
  __shared__ int peer_slot;

  // The epilogue's scales and biases (already warmed in L2 above) are pulled
  // into this SM's L1 now, so that the epilogue's loads hit L1 instead of
  // adding an L2 round trip after the weight stream.
  if (wk == 0 && q == 0) {
    const int esz = scale_f32 ? 4 : 2, bsz = bias_kind == 2 ? 4 : 2;
    rla_prefetch_l1(static_cast<const char*>(scale) + (int64_t)r0 * esz);
    rla_prefetch_l1(static_cast<const char*>(GLU ? scale_up : scale) + (int64_t)r1 * esz);
    if (bias_kind != 0) {
      rla_prefetch_l1(static_cast<const char*>(bias) + (int64_t)r0 * bsz);
      rla_prefetch_l1(static_cast<const char*>(GLU ? bias_up : bias) + (int64_t)r1 * bsz);
    }
  }

  const uint4 zero4 = make_uint4(0, 0, 0, 0);
  // XJIT: each chunk's activation fragments are loaded just before its MMAs
  // instead of with the batch's weight loads, so that all the weight loads
  // issue first.  Chosen per launch shape (XJ) from measurements; the gated
  // and exchange forms keep the batch order.
  constexpr bool XJIT = XJ && !PEER && !GLU;
  for (int c = c_begin + wk; c < c_end; c += WK * U) {
    uint4 wa[U][2];
    XFrag<NT> xb[U];
    // Issue every load of U chunks before any math: U*2 streaming 16-byte
    // weight loads (plus the L1-resident activation loads) in flight per lane.
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int cc = c + u * WK;
      const int kofs = cc * 64;
      const bool ok = (cc < c_end) && (kofs + q * 16 < K);
      wa[u][0] = ok ? rla_ldg_stream(wrow0 + kofs) : zero4;
      wa[u][1] = ok ? rla_ldg_stream(wrow1 + kofs) : zero4;
      if constexpr (!XJIT) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const bool okx = ok && xrow_ok[t];
          xb[u].v[t][0] = okx ? rla_ldg_keep(xrow[t] + kofs) : zero4;
          xb[u].v[t][1] = okx ? rla_ldg_keep(xrow[t] + kofs + 8) : zero4;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if constexpr (XJIT) {
        const int cc = c + u * WK;
        const int kofs = cc * 64;
        const bool ok = (cc < c_end) && (kofs + q * 16 < K);
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const bool okx = ok && xrow_ok[t];
          xb[u].v[t][0] = okx ? rla_ldg_keep(xrow[t] + kofs) : zero4;
          xb[u].v[t][1] = okx ? rla_ldg_keep(xrow[t] + kofs + 8) : zero4;
        }
      }
      skinny_chunk_mma<NT>(acc, wa[u], xb[u]);
    }
  }

  // ---- reduce the WK k-slicing warps (fixed order) ----
  __shared__ __align__(16) float red[(WK > 1 ? WK - 1 : 1) * WN * NT * 4 * 32];
  if constexpr (WK > 1) {
    if (wk > 0) {
      float* dst = red + (((wk - 1) * WN + wn) * NT * 4) * 32;
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[(t * 4 + i) * 32 + lane] = acc[t][i];
    }
    __syncthreads();
    if (wk == 0) {
      for (int j = 0; j < WK - 1; ++j) {
        const float* src = red + ((j * WN + wn) * NT * 4) * 32;
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[t][i] += src[(t * 4 + i) * 32 + lane];
      }
    }
  }

  // ---- split-K inside a thread-block cluster (no workspace) ----
  // The CTAs of a row block form one cluster along y, cluster rank = K slice.
  // Ranks 1.. leave k-warp 0's partial sums in shared memory; rank 0 adds
  // them in rank order (the order of the workspace path below, so the sums
  // are the same) and runs the single-CTA epilogue.
  const bool cluster_split = gridDim.y > 1 && partial == nullptr;
  if (cluster_split) {
    static_assert(WK >= 2, "the exchange reuses the k-warp reduction buffer");
    float* mine = red + (wn * 32 + lane) * (NT * 4);  // (WN x 32 lanes) x (NT x 4) floats
    const uint32_t rank = rla_cluster_ctarank();
    __syncwarp();  // this warp's reads of the reduction buffer are done
    if (wk == 0 && rank != 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
        *reinterpret_cast<float4*>(mine + 4 * t) = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
    }
    rla_cluster_sync();
    if (wk == 0 && rank == 0) {
      const uint32_t ranks = rla_cluster_nctarank();
      for (uint32_t r = 1; r < ranks; ++r) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4 v = rla_ld_dsmem_f4(mine + 4 * t, r);
          acc[t][0] += v.x;
          acc[t][1] += v.y;
          acc[t][2] += v.z;
          acc[t][3] += v.w;
        }
      }
    }
    rla_cluster_sync();  // no CTA exits while rank 0 may still read its shared memory
    if (rank != 0) {
      if constexpr (PEER) skinny_peer_finish<NT>(po, call, y, ldy, M, N, &peer_slot);
      return;
    }
  }

  // Accumulator element (t, i): row n = n0 + g + 8*(i>>1), token m = 8t + 2q + (i&1).
  // Gated form: i>>1 = 0 is the gate, 1 the up projection of output n0 + g.
  if (gridDim.y == 1 || cluster_split) {
    if constexpr (GLU) {
      const int n = n0 + g;
      if (wk == 0 && n < N) {
        const float scg = scale_f32 ? static_cast<const float*>(scale)[n]
                                    : __half2float(static_cast<const __half*>(scale)[n]);
        const float scu = scale_f32 ? static_cast<const float*>(scale_up)[n]
                                    : __half2float(static_cast<const __half*>(scale_up)[n]);
        const float big = bias_kind == 0 ? 0.f
                          : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias)[n])
                                           : static_cast<const float*>(bias)[n];
        const float biu = bias_kind == 0 ? 0.f
                          : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias_up)[n])
                                           : static_cast<const float*>(bias_up)[n];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int m = t * 8 + 2 * q + j;
            if (m < M) y[(int64_t)m * ldy + n] = rla_swiglu(fmaf(acc[t][j], scg, big), fmaf(acc[t][2 + j], scu, biu));
          }
      }
      return;
    }
    if (wk == 0) {
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int n = n0 + g + 8 * hi;
        if (n >= N) continue;
        const float sc = scale_f32 ? static_cast<const float*>(scale)[n]
                                   : __half2float(static_cast<const __half*>(scale)[n]);
        const float bi = bias_kind == 0 ? 0.f
                         : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias)[n])
                                          : static_cast<const float*>(bias)[n];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if constexpr (PEER) {
            // rows 8t + 2q and 8t + 2q + 1 form pair 4t + q
            if (t * 8 + 2 * q < M)
              peer_store_pair(po, call, y, ldy, M, N, 4 * t + q, n, __float2half_rn(fmaf(acc[t][2 * hi], sc, bi)),
                              __float2half_rn(fmaf(acc[t][2 * hi + 1], sc, bi)));
          } else {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int m = t * 8 + 2 * q + j;
              if (m < M) y[(int64_t)m * ldy + n] = __float2half_rn(fmaf(acc[t][2 * hi + j], sc, bi));
            }
          }
        }
      }
    }
    if constexpr (PEER) skinny_peer_finish<NT>(po, call, y, ldy, M, N, &peer_slot);
    return;
  }

  // ---- split-K across CTAs: publish this slice, the last CTA adds them all ----
  // Partial sums [splits][M][NP]; the gated form keeps gate in columns
  // [0, N) and up in [N, 2N).
  constexpr int NPF = GLU ? 2 : 1;
  if (wk == 0) {
    float* part = partial + (int64_t)blockIdx.y * M * N * NPF;
#pragma unroll
    for (int hi = 0; hi < 2; ++hi) {
      const int n = GLU ? n0 + g : n0 + g + 8 * hi;
      if (n >= N) continue;
      const int col = GLU ? hi * N + n : n;
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int m = t * 8 + 2 * q + j;
          if (m < M) __stcg(part + (int64_t)m * N * NPF + col, acc[t][2 * hi + j]);
        }
    }
  }
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    const unsigned int prev = rla_arrive_acq_rel_gpu(counters + blockIdx.x);
    is_last = (prev == gridDim.y - 1);
  }
  __syncthreads();
  if (!is_last) {
    if constexpr (PEER) skinny_peer_finish<NT>(po, call, y, ldy, M, N, &peer_slot);
    return;
  }

  const int rows_here = min(OUTS, N - row_base);
  if constexpr (GLU) {
    for (int idx = threadIdx.x; idx < rows_here * M; idx += blockDim.x) {
      const int n = row_base + idx % rows_here;
      const int m = idx / rows_here;
      float sg = 0.f, su = 0.f;
      for (int sidx = 0; sidx < (int)gridDim.y; ++sidx) {
        const float* row = partial + ((int64_t)sidx * M + m) * 2 * N;
        sg += __ldcg(row + n);
        su += __ldcg(row + N + n);
      }
      const float scg =
          scale_f32 ? static_cast<const float*>(scale)[n] : __half2float(static_cast<const __half*>(scale)[n]);
      const float scu =
          scale_f32 ? static_cast<const float*>(scale_up)[n] : __half2float(static_cast<const __half*>(scale_up)[n]);
      const float big = bias_kind == 0 ? 0.f
                        : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias)[n])
                                         : static_cast<const float*>(bias)[n];
      const float biu = bias_kind == 0 ? 0.f
                        : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias_up)[n])
                                         : static_cast<const float*>(bias_up)[n];
      y[(int64_t)m * ldy + n] = rla_swiglu(fmaf(sg, scg, big), fmaf(su, scu, biu));
    }
    if (threadIdx.x == 0) counters[blockIdx.x] = 0u;  // leave the workspace re-usable
    return;
  }
  // Plain output: one element per step; exchange: one pair of rows per step.
  const int steps = PEER ? (M + 1) / 2 : M;
  for (int idx = threadIdx.x; idx < rows_here * steps; idx += blockDim.x) {
    const int n = row_base + idx % rows_here;
    const int m = (PEER ? 2 : 1) * (idx / rows_here);
    float sum = 0.f;
    for (int sidx = 0; sidx < (int)gridDim.y; ++sidx) sum += __ldcg(partial + ((int64_t)sidx * M + m) * N + n);
    const float sc =
        scale_f32 ? static_cast<const float*>(scale)[n] : __half2float(static_cast<const __half*>(scale)[n]);
    const float bi = bias_kind == 0 ? 0.f
                     : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias)[n])
                                      : static_cast<const float*>(bias)[n];
    if constexpr (PEER) {
      float sum1 = 0.f;
      if (m + 1 < M)
        for (int sidx = 0; sidx < (int)gridDim.y; ++sidx)
          sum1 += __ldcg(partial + ((int64_t)sidx * M + m + 1) * N + n);
      peer_store_pair(po, call, y, ldy, M, N, m / 2, n, __float2half_rn(fmaf(sum, sc, bi)),
                      __float2half_rn(fmaf(sum1, sc, bi)));
    } else {
      y[(int64_t)m * ldy + n] = __float2half_rn(fmaf(sum, sc, bi));
    }
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = 0u;  // leave the workspace re-usable
  if constexpr (PEER) skinny_peer_finish<NT>(po, call, y, ldy, M, N, &peer_slot);
}

#define RLA_SKINNY_PARAMS                                                                                     \
  const __half* __restrict__ x, int64_t ldx, const int8_t* __restrict__ w, int64_t ldw,                         \
      const void* __restrict__ scale, int scale_f32, const void* __restrict__ bias, int bias_kind,               \
      __half* __restrict__ y, int64_t ldy, int M, int N, int K, int chunks_per_split, float* __restrict__ partial, \
      unsigned int* __restrict__ counters, const __grid_constant__ PeerOut po, const int8_t* __restrict__ w_up,   \
      const void* __restrict__ scale_up, const void* __restrict__ bias_up
#define RLA_SKINNY_ARGS                                                                                   \
  x, ldx, w, ldw, scale, scale_f32, bias, bias_kind, y, ldy, M, N, K, chunks_per_split, partial, counters, po, \
      w_up, scale_up, bias_up

template <int NT, int WN, int WK, int U, bool PEER, bool GLU, bool XJ>
__global__ void __launch_bounds__(32 * WN * WK) w8a16_skinny_kernel(RLA_SKINNY_PARAMS) {
  skinny_body<NT, WN, WK, U, PEER, GLU, XJ>(RLA_SKINNY_ARGS);
}

// The one-tile exchange form of the 128-thread CTA with the register budget
// of seven resident CTAs per SM: left to itself the compiler gives that form
// 56 registers, too few to keep a whole batch of loads in flight (the plain
// form gets 72); with this bound it gets 72.  One GPU, world-1 exchange,
// 8192 -> 14336 at M = 1: 28.7 -> 24.6 us.
template <int NT, int WN, int WK, int U, bool PEER, bool GLU, bool XJ>
__global__ void __launch_bounds__(32 * WN * WK, 7) w8a16_skinny_kernel_b7(RLA_SKINNY_PARAMS) {
  skinny_body<NT, WN, WK, U, PEER, GLU, XJ>(RLA_SKINNY_ARGS);
}

// One row group of 16 k-warps (512 threads) with the register budget of two
// resident CTAs per SM (64 registers): for M <= 8 on layers of at most two
// row blocks per SM, every warp's K share is in flight in one batch of loads
// and the slices add up in shared memory, with no split of K across CTAs.
template <int NT, int U, bool XJ>
__global__ void __launch_bounds__(512, 2) w8a16_skinny16_kernel(RLA_SKINNY_PARAMS) {
  skinny_body<NT, 1, 16, U, false, false, XJ>(RLA_SKINNY_ARGS);
}

// ---------------------------------------------------------------------------
// Host side.  Per-device facts about an instantiation (its dynamic
// shared-memory attribute, its occupancy) are cached per device, lock-free:
// a race only repeats a query.
// ---------------------------------------------------------------------------
constexpr int kSkMaxDevices = 64;

static int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kSkMaxDevices) return -1;
  return d;
}

// The kernel instance of a configuration and form (0 plain, 1 gated, 2 with
// the peer exchange).
template <int NT, int WN, int WK, bool XJ>
struct SkinnyInst {
  static constexpr int U = NT >= 4 ? 2 : 4;
  static constexpr int THREADS = 32 * WN * WK;
  static constexpr size_t SMEM = 0;
  using KernT = void (*)(const __half*, int64_t, const int8_t*, int64_t, const void*, int, const void*, int,
                         __half*, int64_t, int, int, int, int, float*, unsigned int*, const PeerOut, const int8_t*,
                         const void*, const void*);
  static KernT kernel(int form) {
    if constexpr (WN * WK == 16) {
      (void)form;  // plain form only (the plan never asks for the others)
      return w8a16_skinny16_kernel<NT, U, XJ>;
    } else {
      if (form == 2) {
        if constexpr (NT == 1 && WN * WK == 4) return w8a16_skinny_kernel_b7<NT, WN, WK, U, true, false, XJ>;
        return w8a16_skinny_kernel<NT, WN, WK, U, true, false, XJ>;
      }
      return form == 1 ? w8a16_skinny_kernel<NT, WN, WK, U, false, true, XJ>
                       : w8a16_skinny_kernel<NT, WN, WK, U, false, false, XJ>;
    }
  }
  // CTAs that can be resident on the whole device at once when the K slices
  // of a row block form clusters of `cluster` CTAs (1: no cluster).  With
  // clusters this counts whole clusters that fit (all CTAs of a cluster sit
  // in one GPC), not just CTAs per SM.  0 when the device cannot be asked.
  static int resident(int form, int cluster) {
    static std::atomic<int> cache[kSkMaxDevices][3][kMaxClusterSplits + 1];
    const int d = current_device();
    if (d < 0 || cluster < 1 || cluster > kMaxClusterSplits) return 0;
    const int cached = cache[d][form][cluster].load(std::memory_order_relaxed);
    if (cached > 0) return cached;
    int v = 0;
    cudaError_t e;
    if (cluster == 1) {
      int per_sm = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel(form), THREADS, SMEM);
      v = per_sm * device_sm_count();
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, cluster);
      cfg.blockDim = dim3(THREADS);
      cfg.dynamicSmemBytes = SMEM;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 1;
      attr[0].val.clusterDim.y = static_cast<unsigned int>(cluster);
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, kernel(form), &cfg);
      v = clusters * cluster;
    }
    if (e != cudaSuccess || v < 1) {
      (void)cudaGetLastError();
      return 0;
    }
    cache[d][form][cluster].store(v, std::memory_order_relaxed);
    return v;
  }
};

template <int NT, int WN, int WK, bool XJ>
static cudaError_t launch_cfg(const GemmArgs& a, const Plan& p, void* workspace, cudaStream_t s) {
  using I = SkinnyInst<NT, WN, WK, XJ>;
  const int form = a.w_up ? 1 : a.peer.world > 0 ? 2 : 0;
  const int total_chunks = (a.K + 63) / 64;
  const int cps = (total_chunks + p.splits - 1) / p.splits;
  unsigned int* counters = nullptr;
  float* partial = nullptr;
  if (p.splits > 1 && !p.cluster) {
    counters = static_cast<unsigned int*>(workspace);
    partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kSplitCounterBytes);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid_x, p.splits);
  cfg.blockDim = dim3(I::THREADS);
  cfg.dynamicSmemBytes = I::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see rla_griddep_wait
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int cluster = p.splits > 1 && p.cluster ? p.splits : 1;
  if (cluster > 1) {
    // the K slices of a row block are one cluster (split-K through
    // distributed shared memory)
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = static_cast<unsigned int>(cluster);
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  PeerOut po = a.peer;
  if (po.world > 0) {
    // Unpacking CTAs: the whole grid when it is resident at once (counted in
    // whole clusters), else at most (resident + 1) / 2 so that the CTAs still
    // to run find room.
    int resident = I::resident(form, cluster);
    if (resident < 1) resident = 1;
    const unsigned int ctas = static_cast<unsigned int>(p.grid_x) * static_cast<unsigned int>(p.splits);
    po.unpackers = ctas <= (unsigned)resident ? ctas : ((unsigned)resident + 1) / 2;
  }
  return cudaLaunchKernelEx(&cfg, I::kernel(form), static_cast<const __half*>(a.x), a.ldx, a.w, a.ldw, a.scale,
                            a.scale_f32, a.bias, a.bias_kind, static_cast<__half*>(a.y), a.ldy, a.M, a.N, a.K, cps,
                            partial, counters, po, a.w_up, a.scale_up, a.bias_up);
}

// Instantiated configurations: NT in {1, 2, 4}; (WN, WK) in {(1, 8), (2, 4),
// (4, 2), (1, 4)}.  Activation loads just before the MMAs (XJ): always for
// NT = 1 with (1, 8); for NT = 2 with (1, 4) when the plan asks for it.
template <int NT>
static cudaError_t launch_nt(const GemmArgs& a, const Plan& p, void* ws, cudaStream_t s) {
  if (p.wn == 1 && p.wk == 8) return launch_cfg<NT, 1, 8, NT == 1>(a, p, ws, s);
  if constexpr (NT == 1) {
    if (p.wn == 1 && p.wk == 16) {
      if (a.w_up || a.peer.world > 0) return cudaErrorInvalidConfiguration;
      return launch_cfg<NT, 1, 16, true>(a, p, ws, s);
    }
  }
  if (p.wn == 2 && p.wk == 4) return launch_cfg<NT, 2, 4, false>(a, p, ws, s);
  if (p.wn == 4 && p.wk == 2) return launch_cfg<NT, 4, 2, false>(a, p, ws, s);
  if (p.wn == 1 && p.wk == 4) {
    if constexpr (NT == 2) {
      if (p.xjit) return launch_cfg<NT, 1, 4, true>(a, p, ws, s);
    }
    return launch_cfg<NT, 1, 4, false>(a, p, ws, s);
  }
  return cudaErrorInvalidConfiguration;
}

template <int NT>
static int resident_nt(int wn, int wk, int form, bool xjit, int cluster) {
  if (wn == 1 && wk == 8) return SkinnyInst<NT, 1, 8, NT == 1>::resident(form, cluster);
  if constexpr (NT == 1) {
    if (wn == 1 && wk == 16) return form == 0 ? SkinnyInst<NT, 1, 16, true>::resident(form, cluster) : 0;
  }
  if (wn == 2 && wk == 4) return SkinnyInst<NT, 2, 4, false>::resident(form, cluster);
  if (wn == 4 && wk == 2) return SkinnyInst<NT, 4, 2, false>::resident(form, cluster);
  if (wn == 1 && wk == 4) {
    if constexpr (NT == 2) {
      if (xjit) return SkinnyInst<NT, 1, 4, true>::resident(form, cluster);
    }
    return SkinnyInst<NT, 1, 4, false>::resident(form, cluster);
  }
  return 0;
}

int skinny_resident_ctas(int nt, int wn, int wk, bool gated, bool xjit, bool peer, int cluster) {
  const int form = gated ? 1 : peer ? 2 : 0;
  int v = 0;
  switch (nt) {
    case 1: v = resident_nt<1>(wn, wk, form, xjit, cluster); break;
    case 2: v = resident_nt<2>(wn, wk, form, xjit, cluster); break;
    case 4: v = resident_nt<4>(wn, wk, form, xjit, cluster); break;
    default: break;
  }
  // no device to ask (e.g. planning on a CPU-only host): two CTAs per SM
  return v > 0 ? v : 2 * device_sm_count();
}

int skinny_ctas_per_sm(int nt, int wn, int wk, bool gated, bool xjit, bool peer) {
  return skinny_resident_ctas(nt, wn, wk, gated, xjit, peer, 1) / device_sm_count();
}

cudaError_t launch_skinny(const GemmArgs& a, const Plan& p, void* workspace, cudaStream_t s) {
  switch (p.nt) {
    case 1: return launch_nt<1>(a, p, workspace, s);
    case 2: return launch_nt<2>(a, p, workspace, s);
    case 4: return launch_nt<4>(a, p, workspace, s);
    default: return cudaErrorInvalidConfiguration;
  }
}

}  // namespace rla
