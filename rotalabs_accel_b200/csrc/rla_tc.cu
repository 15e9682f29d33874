// Prefill-regime W8A16 kernel (M > 32): TMA -> int8->fp16 into Tensor Memory
// -> tcgen05.mma with fp32 accumulators in Tensor Memory.
//
// Orientation ("swap-AB"): a tile is 128 weight rows (output channels n) x BM
// activation rows (tokens m).  The weight tile is the MMA's A operand
// (M = 128 = the 128 TMEM lanes), the activation tile the B operand
// (N = BM), so D[n, m] lives in TMEM with one output channel per lane and the
// per-channel scale is a single register per epilogue thread.
//
// Warp roles (320 threads, one CTA per SM):
//   warp 0      TMA producer: per 64-wide k block, one fp16 x tile
//               [BM x 64] (128-byte swizzle, UMMA canonical K-major layout)
//               and one int8 w tile [128 x 64] (64-byte swizzle) into a
//               STAGES-deep shared-memory ring, completion on mbarriers.
//   warp 1      TMEM allocator + MMA issuer (one thread): 4 x
//               tcgen05.mma.kind::f16 (128 x BM x 16) per k block, A from
//               TMEM, B from shared memory; tcgen05.commit frees the ring
//               slot and the TMEM operand slot.
//   warps 2-9   converters, then epilogue, two per TMEM lane quarter.  Thread
//               i of warp w owns TMEM lane 32*(w%4)+i = weight row i of the
//               tile: it reads its half (32 int8) of the row's 64-byte k block
//               from shared memory (swizzle-aware, bank-conflict-free),
//               converts to fp16 in registers and writes them with tcgen05.st
//               into its half of an A-operand slot of TMEM (ASTAGES slots).
//               After the last k block: tcgen05.ld of every other 32-token
//               block of its row of D, x scale[n] (+ bias[n]), fp16, store.
// No operand is ever converted into shared memory: shared-memory traffic is
// the TMA writes, one read of the int8 tile and the MMA's read of x.
//
// All waits are bounded (rla_mbar_wait); a timeout records a device error,
// raises a CTA-wide abort flag and unwinds to the TMEM release.
#include "rla_common.cuh"
#include "rla_internal.h"
#include "rla_tmap.cuh"

namespace rla {

namespace tc {
constexpr int BN = 128;          // weight rows per tile (MMA M, TMEM lanes)
constexpr int BK = 64;           // k per pipeline stage
constexpr int ASTAGES = 4;       // TMEM A-operand slots (32 columns each)
constexpr int CONVW = 8;         // converter (then epilogue) warps: 2 per TMEM lane quarter
constexpr int THREADS = 64 + 32 * CONVW;
constexpr int W_TILE_BYTES = BN * BK;  // int8
}  // namespace tc

template <int BM, int STAGES>
struct TcShared {
  alignas(1024) uint8_t x[STAGES][BM * 128];
  alignas(1024) uint8_t w[STAGES][tc::W_TILE_BYTES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t afull[tc::ASTAGES];
  uint64_t aempty[tc::ASTAGES];
  uint64_t dfull;
  uint32_t tmem_base;
  int abort_flag;
};

template <int BM>
__host__ __device__ constexpr int tmem_cols_for() {
  // D: BM fp32 columns; A ring: ASTAGES x 32 columns (64 fp16 k per slot).
  return (BM + tc::ASTAGES * 32) <= 256 ? 256 : 512;
}

template <int BM, int STAGES>
__global__ void __launch_bounds__(tc::THREADS, 1)
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                    const void* __restrict__ scale, int scale_f32, const void* __restrict__ bias, int bias_kind,
                    __half* __restrict__ y, int64_t ldy, int M, int N, int K) {
  using Smem = TcShared<BM, STAGES>;
  constexpr int TMEM_COLS = tmem_cols_for<BM>();
  constexpr uint32_t STAGE_TX = BM * 128 + tc::W_TILE_BYTES;

  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * tc::BN;
  const int m0 = blockIdx.y * BM;
  const int num_kb = (K + tc::BK - 1) / tc::BK;
  volatile int* abort_flag = &sm.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      rla_mbar_init(&sm.full[s], 1);
      rla_mbar_init(&sm.empty[s], 1);
    }
    for (int a = 0; a < tc::ASTAGES; ++a) {
      rla_mbar_init(&sm.afull[a], tc::CONVW);  // one arrival per converter warp
      rla_mbar_init(&sm.aempty[a], 1);
    }
    rla_mbar_init(&sm.dfull, 1);
    sm.abort_flag = 0;
    rla_fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    rla_tma_prefetch_desc(&tmap_x);
    rla_tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    rla_tmem_alloc(&sm.tmem_base, TMEM_COLS);
    rla_tmem_relinquish();
  }
  rla_tc_fence_before();
  __syncthreads();
  rla_tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t a_col0 = BM;  // A slots follow the accumulator columns

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int issued_until = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES) {
          if (!rla_mbar_wait(&sm.empty[s], ((kb / STAGES) - 1) & 1, RLA_DEVERR_TIMEOUT_SLOT_EMPTY, abort_flag))
            break;
        }
        rla_mbar_arrive_expect_tx(&sm.full[s], STAGE_TX);
        rla_tma_load_2d(sm.x[s], &tmap_x, &sm.full[s], kb * tc::BK, m0);
        rla_tma_load_2d(sm.w[s], &tmap_w, &sm.full[s], kb * tc::BK, n0);
        issued_until = kb + 1;
      }
      if (*abort_flag) {
        // Do not leave the CTA while our copies may still land in shared memory.
        for (int kb = max(0, issued_until - STAGES); kb < issued_until; ++kb)
          rla_mbar_wait(&sm.full[kb % STAGES], (kb / STAGES) & 1, RLA_DEVERR_TIMEOUT_TMA_FULL, nullptr);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = rla_idesc_f16_f32(tc::BN, BM);
      bool ok = true;
      for (int kb = 0; kb < num_kb && ok; ++kb) {
        const int s = kb % STAGES;
        const int a = kb % tc::ASTAGES;
        ok = rla_mbar_wait(&sm.full[s], (kb / STAGES) & 1, RLA_DEVERR_TIMEOUT_TMA_FULL, abort_flag) &&
             rla_mbar_wait(&sm.afull[a], (kb / tc::ASTAGES) & 1, RLA_DEVERR_TIMEOUT_A_FULL, abort_flag);
        if (!ok) break;
        rla_tc_fence_after();
        const uint32_t xbase = rla_smem_u32(sm.x[s]);
#pragma unroll
        for (int ks = 0; ks < tc::BK / 16; ++ks) {
          const uint64_t bdesc = rla_smem_desc_sw128(xbase + ks * 32);
          rla_umma_ts_f16(tmem, tmem + a_col0 + a * 32 + ks * 8, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
        }
        rla_umma_commit(&sm.empty[s]);
        rla_umma_commit(&sm.aempty[a]);
      }
      rla_umma_commit(&sm.dfull);
      // On the abort path nobody else waits for the accumulator: make sure
      // no MMA is still writing TMEM before it is released.
      if (!ok) rla_mbar_wait(&sm.dfull, 0, RLA_DEVERR_TIMEOUT_ACCUM, nullptr);
    }
    __syncwarp();
  } else {
    // ---------------- converters, then epilogue ----------------
    // Warps 2 .. 2 + CONVW - 1: quarter = warp % 4 (the TMEM lanes a warp may
    // touch), half = which 32 of the k block's 64 bytes it converts (and
    // which 32-token column blocks it writes out in the epilogue).
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;  // TMEM lane == weight row within the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int swz = (row >> 1) & 3;       // 64-byte swizzle of the int8 tile
    bool ok = true;
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % STAGES;
      const int a = kb % tc::ASTAGES;
      ok = rla_mbar_wait(&sm.full[s], (kb / STAGES) & 1, RLA_DEVERR_TIMEOUT_TMA_FULL, abort_flag);
      if (ok && kb >= tc::ASTAGES)
        ok = rla_mbar_wait(&sm.aempty[a], ((kb / tc::ASTAGES) - 1) & 1, RLA_DEVERR_TIMEOUT_A_EMPTY, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      rla_tc_fence_after();
      const uint8_t* wrow = sm.w[s] + row * 64;
      uint32_t v[16];
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;      // 16-byte chunk of the row
        const uint4 q4 = *reinterpret_cast<const uint4*>(wrow + ((c ^ swz) << 4));
        rla_i8x4_to_h2x2(q4.x, v[cc * 8 + 0], v[cc * 8 + 1]);
        rla_i8x4_to_h2x2(q4.y, v[cc * 8 + 2], v[cc * 8 + 3]);
        rla_i8x4_to_h2x2(q4.z, v[cc * 8 + 4], v[cc * 8 + 5]);
        rla_i8x4_to_h2x2(q4.w, v[cc * 8 + 6], v[cc * 8 + 7]);
      }
      rla_tmem_st_32x32b_x16(tmem + lane_addr + a_col0 + a * 32 + half * 16, v);
      rla_tmem_wait_st();
      rla_tc_fence_before();
      __syncwarp();
      if (lane == 0) rla_mbar_arrive(&sm.afull[a]);
    }
    if (ok) ok = rla_mbar_wait(&sm.dfull, 0, RLA_DEVERR_TIMEOUT_ACCUM, abort_flag);
    if (__all_sync(0xffffffffu, ok)) {
      rla_tc_fence_after();
      const int n = n0 + row;
      float sc = 0.f, bi = 0.f;
      if (n < N) {
        sc = scale_f32 ? static_cast<const float*>(scale)[n] : __half2float(static_cast<const __half*>(scale)[n]);
        bi = bias_kind == 0 ? 0.f
             : bias_kind == 1 ? __half2float(static_cast<const __half*>(bias)[n])
                              : static_cast<const float*>(bias)[n];
      }
#pragma unroll 1
      for (int j = half; j < BM / 32; j += 2) {
        if (m0 + j * 32 >= M) break;
        uint32_t d[32];
        rla_tmem_ld_32x32b_x32(tmem + lane_addr + j * 32, d);
        rla_tmem_wait_ld();
        if (n < N) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int m = m0 + j * 32 + i;
            if (m < M) y[(int64_t)m * ldy + n] = __float2half_rn(fmaf(__uint_as_float(d[i]), sc, bi));
          }
        }
      }
    }
  }

  rla_tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    rla_tc_fence_after();
    rla_tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
size_t tcgen05_smem_bytes(int bm, int stages) {
  size_t per_stage = (size_t)bm * 128 + tc::W_TILE_BYTES;
  return per_stage * stages + 1024 /* barriers etc. */ + 1024 /* alignment slack */;
}
int tcgen05_tmem_cols(int bm) { return (bm + tc::ASTAGES * 32) <= 256 ? 256 : 512; }

template <int BM, int STAGES>
static cudaError_t launch_tc_cfg(const GemmArgs& a, const Plan& p, cudaStream_t s) {
  CUtensorMap tx, tw;
  if (!make_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.x, (uint64_t)a.K, (uint64_t)a.M,
                    (uint64_t)a.ldx * 2, tc::BK, BM, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, a.w, (uint64_t)a.K, (uint64_t)a.N, (uint64_t)a.ldw,
                    tc::BK, tc::BN, CU_TENSOR_MAP_SWIZZLE_64B))
    return cudaErrorInvalidValue;
  const size_t smem = sizeof(TcShared<BM, STAGES>) + 1024;
  auto kern = w8a16_tc_kernel<BM, STAGES>;
  // Per device and cheap: set on every launch rather than tracking devices.
  cudaError_t attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (attr_err != cudaSuccess) return attr_err;
  dim3 grid(p.grid_x, p.grid_y);
  rla_clear_stale_launch_error();
  kern<<<grid, tc::THREADS, smem, s>>>(tx, tw, a.scale, a.scale_f32, a.bias, a.bias_kind,
                                        static_cast<__half*>(a.y), a.ldy, a.M, a.N, a.K);
  return cudaGetLastError();
}

cudaError_t launch_tcgen05(const GemmArgs& a, const Plan& p, cudaStream_t s) {
  if (p.bm == 256 && p.stages == 4) return launch_tc_cfg<256, 4>(a, p, s);
  if (p.bm == 128 && p.stages == 6) return launch_tc_cfg<128, 6>(a, p, s);
  if (p.bm == 64 && p.stages == 8) return launch_tc_cfg<64, 8>(a, p, s);
  return cudaErrorInvalidConfiguration;
}

}  // namespace rla
