// Decode-regime W8A16 kernel, persistent and stream-K (M <= 32).
//
// The decode GEMM is a stream of N*K int8 weight bytes; everything else is
// small.  This kernel keeps every SM's share of that stream in flight for
// the whole launch:
//
//  * Work space.  Units are (row block of 128 weight rows) x (128-wide k
//    box); there are U = ceil(N/128) * ceil(K/128) of them, ordered row block
//    by row block.  The persistent grid has P CTAs (one per SM) and CTA p takes
//    the contiguous unit range [U*p/P, U*(p+1)/P): every CTA streams the same
//    number of bytes (to one unit), so there is no wave tail.
//  * Producer warp (one thread).  Walks its range in stages of up to SB boxes
//    of one row block.  Per box it issues TMA tensor loads of the int8 weight
//    box [128 rows x 128 k] and of two fp16 activation boxes [8*NT rows x 64 k],
//    all with the 128-byte swizzle, into a STAGES-deep shared-memory ring; a
//    transaction-count mbarrier per stage completes when the bytes land.
//    Rows past N, k past K and tokens past M are zero-filled by TMA, so the
//    consumers need no bounds checks.  Few, large TMA operations: per-row
//    bulk copies were measured to serialise in the copy engine.
//  * Consumer warps (8).  Warp w owns weight rows [16w, 16w+16) of the row
//    block, so no cross-warp reduction is ever needed.  Per box a lane reads
//    32 contiguous int8 (k = 32q .. 32q+31 of the box) of rows g and g+8 --
//    16-byte chunks 2q and 2q+1 -- and the matching 64 bytes of x; the chunk
//    addresses follow the swizzle and the x chunk order is rotated per lane
//    so that every shared-memory read is bank-conflict-free.  int8 -> fp16
//    in registers, then mma.sync.m16n8k16 with the weight rows as the MMA's
//    M and the tokens as its N (the k order inside the fragment is permuted
//    to match the contiguous bytes; x uses the same permutation).  Two
//    accumulator sets (even / odd k steps) halve the MMA dependency chain.
//  * Row-block end.  A row block wholly inside the CTA's range is written out
//    (x scale, + bias, fp16; scale and bias were fetched when the row block
//    started).  A row block split between CTAs leaves one fp32 piece per CTA
//    in the workspace; the CTA that arrives last (atomic counter) adds the
//    pieces in CTA order, so results are bit-reproducible.  A CTA that finds
//    every other piece already published skips publishing its own.
//  * Programmatic dependent launch.  A CTA lets the next kernel in the stream
//    start launching as soon as it runs, and asks L2 for its first weight
//    boxes before waiting for the previous kernel (griddepcontrol): L2 is
//    coherent, so the prefetch can never yield stale data, while every real
//    read (TMA into shared memory, x, scale, workspace) waits for the
//    predecessor to finish.  (Prefetching a whole range from a second,
//    co-resident CTA was measured slower: the prefetches queue in the SM's
//    copy engine ahead of the running kernel's loads.)
//
// Waits are bounded (rla_mbar_wait); on a timeout the CTA records a device
// error and raises its abort flag: the producer stops issuing copies (and
// waits, bounded, for those in flight), the consumers run the rest of their
// loop without waiting or computing, so every named barrier still completes.
//
// With a peer exchange (PEER, rla_w8a16_gemm_allgather) the epilogue stores
// pairs of rows into y and, as flagged words, into every peer's receive
// buffer, and the consumer warps end with peer_finish (rla_peer.cuh), also
// after an abort.
#include "rla_common.cuh"
#include "rla_internal.h"
#include "rla_peer.cuh"
#include "rla_tmap.cuh"

namespace rla {

namespace sk {
constexpr int RB = 128;                    // weight rows per row block
constexpr int BOXK = 128;                  // k per weight box (128 bytes of int8)
constexpr int GROUPS = RB / 16;            // 16-row groups per row block
constexpr int NCW = GROUPS;                // consumer warps, one 16-row group each
constexpr int THREADS = 32 * (1 + NCW);
constexpr int W_BOX = RB * BOXK;           // 16 KB
// Weight boxes a CTA asks L2 for before its dependency wait.
constexpr int PREFETCH_BOXES = 4;
}  // namespace sk

template <int NT>
struct StreamCfg {
  static constexpr int XR = 8 * NT;                    // token rows per x box
  static constexpr int X_BOX = XR * 128;               // 64 fp16 x XR rows
  static constexpr int SB = 2;                         // weight boxes per stage
  static constexpr int STAGE = SB * sk::W_BOX + 2 * SB * X_BOX;
  static constexpr int STAGES = NT == 4 ? 4 : 5;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE + 2 * STAGES * 8 + 64 + 1024;
};

RLA_DEVFN void rla_tma_prefetch_l2_2d(const void* desc, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(desc), "r"(c0), "r"(c1)
               : "memory");
}
RLA_DEVFN void rla_named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

RLA_DEVFN unsigned int rla_ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

RLA_DEVFN int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
RLA_DEVFN int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }
// First unit of CTA p's range.
RLA_DEVFN int64_t sk_bound(int64_t units, int p, int P) { return units * p / P; }
// CTA whose range holds unit u.
RLA_DEVFN int sk_owner(int64_t units, int64_t u, int P) {
  int p = static_cast<int>((u * P) / units);
  while (p + 1 < P && sk_bound(units, p + 1, P) <= u) ++p;
  while (p > 0 && sk_bound(units, p, P) > u) --p;
  return p;
}

template <int NT, bool PEER>
__global__ void __launch_bounds__(sk::THREADS, 1)
    w8a16_stream_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                        const void* __restrict__ scale, int scale_f32, const void* __restrict__ bias, int bias_kind,
                        __half* __restrict__ y, int64_t ldy, int M, int N, int K, float* __restrict__ partial,
                        unsigned int* __restrict__ counters, const __grid_constant__ PeerOut po) {
  using Cfg = StreamCfg<NT>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int SB = Cfg::SB;
  constexpr int NCW = sk::NCW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + (size_t)STAGES * Cfg::STAGE);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + STAGES);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int P = gridDim.x;
  const int p = blockIdx.x;
  const int64_t C = (K + sk::BOXK - 1) / sk::BOXK;
  const int64_t R = (N + sk::RB - 1) / sk::RB;
  const int64_t U = R * C;
  const int64_t f_begin = sk_bound(U, p, P);
  const int64_t f_end = sk_bound(U, p + 1, P);
  // Stage cursor (row block, box within it), advanced without divisions.
  const int c_count = static_cast<int>(C);
  const int rb_begin = static_cast<int>(f_begin / C);
  const int c_begin = static_cast<int>(f_begin - (int64_t)rb_begin * C);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      rla_mbar_init(&full[s], 1);
      rla_mbar_init(&empty[s], NCW);
    }
    *abort_flag = 0;
    *last_flag = 0;
    rla_fence_barrier_init();
  }
  __syncthreads();
  rla_griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      rla_tma_prefetch_desc(&tmap_w);
      rla_tma_prefetch_desc(&tmap_x);
      // Ask L2 for the first weight boxes before the dependency wait (the
      // wait covers the predecessor's tail; L2 is coherent).
      {
        int64_t f = f_begin;
        int rb = rb_begin, c0 = c_begin;
        for (int n = 0; f < f_end && n < sk::PREFETCH_BOXES; ++n) {
          rla_tma_prefetch_l2_2d(&tmap_w, c0 * sk::BOXK, rb * sk::RB);
          ++f;
          if (++c0 == c_count) { c0 = 0; ++rb; }
        }
      }
      rla_griddep_wait();
      int64_t f = f_begin;
      int rb = rb_begin, c0 = c_begin;
      int issued = 0;
      for (int it = 0; f < f_end; ++it) {
        const int nb = static_cast<int>(imin64(min(SB, c_count - c0), f_end - f));
        const int s = it % STAGES;
        if (it >= STAGES &&
            !rla_mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, RLA_DEVERR_TIMEOUT_SLOT_EMPTY, abort_flag))
          break;
        uint8_t* stg = stages + (size_t)s * Cfg::STAGE;
        rla_mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nb * (sk::W_BOX + 2 * Cfg::X_BOX)));
        for (int b = 0; b < nb; ++b) {
          const int32_t k = (c0 + b) * sk::BOXK;
          rla_tma_load_2d(stg + b * sk::W_BOX, &tmap_w, &full[s], k, rb * sk::RB);
          uint8_t* xb = stg + SB * sk::W_BOX + (2 * b) * Cfg::X_BOX;
          rla_tma_load_2d(xb, &tmap_x, &full[s], k, 0);
          rla_tma_load_2d(xb + Cfg::X_BOX, &tmap_x, &full[s], k + 64, 0);
        }
        f += nb;
        c0 += nb;
        if (c0 == c_count) { c0 = 0; ++rb; }
        issued = it + 1;
      }
      if (*abort_flag) {
        // Let the copies already issued land before the CTA exits.
        for (int it = max(0, issued - STAGES); it < issued; ++it)
          rla_mbar_wait(&full[it % STAGES], (it / STAGES) & 1, RLA_DEVERR_TIMEOUT_TMA_FULL, nullptr);
      }
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int cw = warp - 1;                  // 16-row group of the row block
  const int g = lane >> 2;
  const int q = lane & 3;
  // Weight rows cw*16 + g and cw*16 + g + 8 both sit at swizzle phase g.
  const int wrowA = (cw * 16 + g) * sk::BOXK;
  const int wrowB = wrowA + 8 * sk::BOXK;
  const int wc0 = ((2 * q) ^ g) << 4;        // chunk 2q, swizzled
  const int wc1 = ((2 * q + 1) ^ g) << 4;    // chunk 2q + 1, swizzled
  // x: lane q reads fp16 k [32q, 32q + 32) of the box = 8-wide chunks 4q..4q+3,
  // from x box (q / 2); the issue order is rotated for q >= 2 (conflict-free).
  int xoff[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int lc = 4 * (q & 1) + ((i + 2 * (q >> 1)) & 3);
    xoff[i] = (q >> 1) * Cfg::X_BOX + g * 128 + ((lc ^ g) << 4);
  }
  const bool rot = q >= 2;

  float acc[2][NT][4];
#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[e][t][0] = acc[e][t][1] = acc[e][t][2] = acc[e][t][3] = 0.f;

  rla_griddep_wait();
  unsigned int call = 0;
  if constexpr (PEER) call = peer_call(po);
  int64_t f = f_begin;
  int rb = rb_begin, c0 = c_begin;
  int rb_loaded = -1;
  float sc_pre[2] = {0.f, 0.f}, bi_pre[2] = {0.f, 0.f};
  for (int it = 0; f < f_end; ++it) {
    const int nb = static_cast<int>(imin64(min(SB, c_count - c0), f_end - f));
    const int s = it % STAGES;
    // After an abort (a wait that gave up, here or in another warp) the warp
    // skips the stage's math but keeps the loop's control flow, so every
    // consumer warp still takes every named barrier of the CTA.
    int ok = 1;
    if (lane == 0) ok = rla_mbar_wait(&full[s], (it / STAGES) & 1, RLA_DEVERR_TIMEOUT_TMA_FULL, abort_flag) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (rb != rb_loaded) {
      // Start of a row block: fetch its scale / bias now, used at its end.
      rb_loaded = rb;
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int n = min(rb * sk::RB + cw * 16 + g + 8 * hi, N - 1);
        sc_pre[hi] = scale_f32 ? static_cast<const float*>(scale)[n]
                               : __half2float(static_cast<const __half*>(scale)[n]);
        bi_pre[hi] = bias_kind == 0 ? 0.f
                     : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias)[n])
                                      : static_cast<const float*>(bias)[n];
      }
    }
    const uint8_t* stg = stages + (size_t)s * Cfg::STAGE;
#pragma unroll
    for (int b = 0; b < SB; ++b) {
      if (b >= nb || !ok) break;
      const uint8_t* wb = stg + b * sk::W_BOX;
      const uint4 a0 = *reinterpret_cast<const uint4*>(wb + wrowA + wc0);
      const uint4 a1 = *reinterpret_cast<const uint4*>(wb + wrowA + wc1);
      const uint4 b0 = *reinterpret_cast<const uint4*>(wb + wrowB + wc0);
      const uint4 b1 = *reinterpret_cast<const uint4*>(wb + wrowB + wc1);
      uint4 xv[NT][4];
      const uint8_t* xb = stg + SB * sk::W_BOX + (2 * b) * Cfg::X_BOX;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        uint4 r[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = *reinterpret_cast<const uint4*>(xb + t * 8 * 128 + xoff[i]);
        // undo the rotated issue order: xv[t][j] = fp16 k [32q + 8j, +8)
        xv[t][0] = rot ? r[2] : r[0];
        xv[t][1] = rot ? r[3] : r[1];
        xv[t][2] = rot ? r[0] : r[2];
        xv[t][3] = rot ? r[1] : r[3];
      }
      const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint32_t wbw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int st = 0; st < 8; ++st) {
        uint32_t a0r, a1r, a2r, a3r;
        rla_i8x4_to_h2x2(wa[st], a0r, a2r);    // row g:   k {2q,2q+1}, {2q+8,2q+9}
        rla_i8x4_to_h2x2(wbw[st], a1r, a3r);   // row g+8
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[t][st >> 1]);
          rla_mma_16816(acc[st & 1][t], a0r, a1r, a2r, a3r, xw[2 * (st & 1)], xw[2 * (st & 1) + 1]);
        }
      }
    }
    __syncwarp();
    if (lane == 0 && ok) rla_mbar_arrive(&empty[s]);
    f += nb;
    c0 += nb;
    const bool rb_done = c0 == c_count;
    const int rb_cur = rb;
    if (rb_done) { c0 = 0; ++rb; }
    if (!rb_done && f != f_end) continue;  // the row block continues in the next stage

    // ---------------- the row block (this CTA's piece of it) is done ----------------
    float sum[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) sum[t][i] = acc[0][t][i] + acc[1][t][i];
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[e][t][0] = acc[e][t][1] = acc[e][t][2] = acc[e][t][3] = 0.f;
    constexpr int NOUT = sk::GROUPS;     // warps taking part in the piece exchange
    const int64_t piece_lo = imax64((int64_t)rb_cur * C, f_begin);
    const int64_t piece_hi = imin64((int64_t)(rb_cur + 1) * C, f_end);
    const bool whole = piece_lo == (int64_t)rb_cur * C && piece_hi == (int64_t)(rb_cur + 1) * C;   // uniform over the CTA
    const int rl0 = cw * 16 + g;            // row within the row block (and +8)
    bool write_out = true;
    if (!whole) {
      const int p_first = sk_owner(U, (int64_t)rb_cur * C, P);
      const int p_last = sk_owner(U, (int64_t)(rb_cur + 1) * C - 1, P);
      const unsigned others = static_cast<unsigned>(p_last - p_first);
      // If every other contributor has already published its piece, this CTA is
      // certainly the last one: no need to publish its own piece first.
      if (cw == 0 && lane == 0) *last_flag = rla_ld_acquire_gpu(counters + p_first) == others ? 2 : 0;
      rla_named_bar_sync(2, NOUT * 32);
      int mode = *last_flag;
      if (mode == 0) {
        // Publish this CTA's piece, then count it; the last contributor adds up.
        const int which = (rb_cur == rb_begin) ? 0 : 1;
        float* dst = partial + ((int64_t)p * 2 + which) * sk::RB * M;
#pragma unroll
        for (int hi = 0; hi < 2; ++hi)
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int m = t * 8 + 2 * q + jj;
              if (m < M) __stcg(dst + (rl0 + 8 * hi) * M + m, sum[t][2 * hi + jj]);
            }
        rla_named_bar_sync(2, NOUT * 32);       // every row group's piece is written
        if (cw == 0 && lane == 0) {
          // releases the CTA's pieces, acquires the others'
          *last_flag = rla_arrive_acq_rel_gpu(counters + p_first) == others ? 1 : 0;
        }
        rla_named_bar_sync(2, NOUT * 32);
        mode = *last_flag;
      }
      write_out = mode != 0;
      if (write_out) {
        // Add the pieces in CTA order (this CTA's own piece from registers).
        float own[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            own[t][i] = sum[t][i];
            sum[t][i] = 0.f;
          }
        for (int pp = p_first; pp <= p_last; ++pp) {
          if (pp == p) {
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int i = 0; i < 4; ++i) sum[t][i] += own[t][i];
            continue;
          }
          const int wh = ((int64_t)rb_cur == sk_bound(U, pp, P) / C) ? 0 : 1;
          const float* src = partial + ((int64_t)pp * 2 + wh) * sk::RB * M;
#pragma unroll
          for (int hi = 0; hi < 2; ++hi)
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int jj = 0; jj < 2; ++jj) {
                const int m = t * 8 + 2 * q + jj;
                if (m < M) sum[t][2 * hi + jj] += __ldcg(src + (rl0 + 8 * hi) * M + m);
              }
        }
        if (cw == 0 && lane == 0) counters[p_first] = 0u;  // leave the workspace re-usable
      }
      rla_named_bar_sync(2, NOUT * 32);         // last_flag may be rewritten at the next row block
    }
    if (write_out) {
      // y[m, n] = fp16(sum * scale[n] + bias[n]); scale and bias were loaded
      // when the row block started.
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int n = rb_cur * sk::RB + rl0 + 8 * hi;
        if (n >= N) continue;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if constexpr (PEER) {
            // rows 8t + 2q and 8t + 2q + 1 form pair 4t + q
            if (t * 8 + 2 * q < M)
              peer_store_pair(po, call, y, ldy, M, N, 4 * t + q, n,
                              __float2half_rn(fmaf(sum[t][2 * hi], sc_pre[hi], bi_pre[hi])),
                              __float2half_rn(fmaf(sum[t][2 * hi + 1], sc_pre[hi], bi_pre[hi])));
          } else {
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int m = t * 8 + 2 * q + jj;
              if (m < M) y[(int64_t)m * ldy + n] = __float2half_rn(fmaf(sum[t][2 * hi + jj], sc_pre[hi], bi_pre[hi]));
            }
          }
        }
      }
    }
  }
  if constexpr (PEER) {
    // Every consumer warp gets here (after the loop, also after an abort: all
    // its waits are bounded), so the barriers over the consumers complete.
    __shared__ int peer_slot;
    peer_finish(po, call, y, ldy, M, N, threadIdx.x - 32, NCW * 32, 3, &peer_slot);
  }
}

size_t stream_workspace_bytes(int64_t M, int ctas) {
  return kSplitCounterBytes + (size_t)ctas * 2 * sk::RB * (size_t)M * sizeof(float);
}

template <int NT>
static cudaError_t launch_stream_nt(const GemmArgs& a, const Plan& p, void* workspace, cudaStream_t s) {
  using Cfg = StreamCfg<NT>;
  CUtensorMap tw, tx;
  if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.ldw,
                    sk::BOXK, sk::RB, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.ldx * 2,
                    64, Cfg::XR, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  auto kern = a.peer.world > 0 ? w8a16_stream_kernel<NT, true> : w8a16_stream_kernel<NT, false>;
  // At most one CTA per SM, all resident at once: every CTA unpacks a share.
  PeerOut po = a.peer;
  if (po.world > 0) po.unpackers = static_cast<unsigned int>(p.grid_x);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM);
  if (e != cudaSuccess) return e;
  unsigned int* counters = static_cast<unsigned int*>(workspace);
  float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + kSplitCounterBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid_x);
  cfg.blockDim = dim3(sk::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tw, tx, a.scale, a.scale_f32, a.bias, a.bias_kind, static_cast<__half*>(a.y),
                            a.ldy, a.M, a.N, a.K, partial, counters, po);
}

cudaError_t launch_stream(const GemmArgs& a, const Plan& p, void* workspace, cudaStream_t s) {
  switch (p.nt) {
    case 1: return launch_stream_nt<1>(a, p, workspace, s);
    case 2: return launch_stream_nt<2>(a, p, workspace, s);
    case 4: return launch_stream_nt<4>(a, p, workspace, s);
    default: return cudaErrorInvalidConfiguration;
  }
}

size_t stream_smem_bytes(int nt) {
  return nt == 1 ? StreamCfg<1>::SMEM : nt == 2 ? StreamCfg<2>::SMEM : StreamCfg<4>::SMEM;
}

}  // namespace rla
