// Pull exchange of the column-parallel prefill (one process per GPU, every
// rank's exchange buffer and sync area IPC-mapped into every other rank).
//
// Rank r computes output columns [r * n_local, (r + 1) * n_local) of a long
// activation block.  One call of the exchange, on rank r:
//
//  * begin (one small kernel, current stream): advance the call number c in
//    r's sync area, then wait (bounded) until every peer has announced that
//    it finished reading r's exchange buffer in call c - 1 (done[peer] >= c-1).
//    Only then may r's GEMM overwrite its exchange buffer.
//  * per block of rows: the library's GEMM writes r's slice of the block's
//    rows into r's exchange buffer xb[r] (current stream); then, on a
//    communication stream ordered after that GEMM, pull:
//      - every CTA marks the block ready in every rank's sync area
//        (ready[r][block] = c; a release store at system scope, ordered after
//        the GEMM's stores by the stream and the kernel boundary);
//      - it waits (bounded) for ready[src][block] >= c of the source rank it
//        copies from, then reads that rank's rows of the block from xb[src]
//        over NVLink (16-byte loads that bypass L1) and stores them into
//        y[rows, src * n_local : (src + 1) * n_local];
//      - on the call's last block, the last CTA to finish tells every peer
//        that r's reads of call c are over (done[r] = c in the peer's sync
//        area).
//
// The next block's GEMM runs on the current stream while a block is pulled,
// so the exchange overlaps the compute.  One exchange buffer per rank is
// enough: a rank's GEMM of call c + 1 starts only after begin(c + 1) saw
// every peer's done of call c.  The ready flags need no reset: a source's
// ready[src][block] can only be c while a reader is in call c (the source
// cannot start call c + 1 before the reader's done of call c), so ">= c"
// means "this call's block is in xb[src]".
//
// No cross-GPU deadlock: a pull waits only for peers' GEMMs of the same call
// and block, which wait on nothing but their own begin, which waits only on
// reads of the previous call.  Pull CTAs need no shared memory and few
// registers, so they fit beside the tcgen05 GEMM's CTAs on the same SM.
//
// Every wait is bounded by the limit of rla_set_peer_wait_limit.  A wait that
// gives up records device error 7 and marks the sync area aborted (the call
// number, never cleared); every kernel of a later call on that sync area then
// records device error 9 and returns at once (y incomplete).  Recovery is
// collective: free and re-create the buffers on every rank.
#include <algorithm>
#include <atomic>

#include "rla_common.cuh"
#include "rla_internal.h"

namespace rla {

namespace px {
constexpr int kSeq = 0;       // call number of the running (or last) call
constexpr int kAbort = RLA_PX_SYNC_ABORT_WORD;  // call number whose wait gave up (never cleared)
constexpr int kTicket = 2;    // CTAs of the last block's pull that finished
constexpr int kDone = 16;     // + src: last call whose reads of this rank's buffer src finished
constexpr int kReady = 32;    // + src * kMaxBlocks + block: call number of src's block
constexpr int kMaxBlocks = RLA_PX_MAX_BLOCKS;
static_assert(kReady + kMaxPeers * kMaxBlocks <= RLA_PX_SYNC_BYTES / 4, "prefill exchange sync area layout");
constexpr int kPullThreads = 256;
}  // namespace px

struct PxArgs {
  const uint4* xb[kMaxPeers];   // every rank's exchange buffer (this rank's is local)
  unsigned int* sync[kMaxPeers];  // every rank's sync area
  uint4* y;                     // this rank's output, row stride ldy16 16-byte units
  int64_t ld_xb16;              // exchange buffer row stride in 16-byte units
  int64_t ldy16;
  int64_t row0;
  int rows;
  int chunks;                   // 16-byte units per row of a slice (n_local / 8)
  int rank, world, block, last;
  int ctas_per_src;
  unsigned long long wait_ns;
};

RLA_DEVFN unsigned int px_ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
RLA_DEVFN void px_st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
RLA_DEVFN uint4 px_ld_cg(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
// a >= b for call numbers that may wrap
RLA_DEVFN bool px_reached(unsigned int a, unsigned int b) { return static_cast<int>(a - b) >= 0; }

// Bounded wait until *flag >= c.  Gives up when the limit passes or when
// another wait of the same call has given up.
RLA_DEVFN bool px_wait(const unsigned int* flag, unsigned int c, unsigned int* sync_local, uint64_t wait_ns) {
  if (px_reached(px_ld_acquire_sys(flag), c)) return true;
  const uint64_t t0 = rla_globaltimer();
  while (true) {
    __nanosleep(200);
    if (px_reached(px_ld_acquire_sys(flag), c)) return true;
    if (rla_ld_relaxed_gpu_u32(sync_local + px::kAbort) != 0u) return false;
    if (rla_globaltimer() - t0 > wait_ns) {
      rla_record_error(RLA_DEVERR_TIMEOUT_PEER_DATA);
      atomicCAS(sync_local + px::kAbort, 0u, c);
      return false;
    }
  }
}

// One warp.  Lane 0 advances the call number; lanes < world wait for their
// peer's done of the previous call.
__global__ void __launch_bounds__(32) px_begin_kernel(PxArgs a) {
  unsigned int* sync = a.sync[a.rank];
  __shared__ unsigned int s_c;
  if (threadIdx.x == 0) {
    if (rla_ld_relaxed_gpu_u32(sync + px::kAbort) != 0u) {
      rla_record_error(RLA_DEVERR_PEER_POISONED);
      s_c = 0u;
    } else {
      const unsigned int c = sync[px::kSeq] + 1u;
      sync[px::kSeq] = c;
      sync[px::kTicket] = 0u;
      s_c = c;
    }
  }
  __syncwarp();
  const unsigned int c = s_c;
  if (c == 0u) return;
  const int src = threadIdx.x;
  if (src < a.world && src != a.rank) (void)px_wait(sync + px::kDone + src, c - 1u, sync, a.wait_ns);
}

// Grid: world * ctas_per_src CTAs; CTA b copies from source rank
// b / ctas_per_src.
template <int UNR>
__global__ void __launch_bounds__(px::kPullThreads) px_pull_kernel(PxArgs a) {
  unsigned int* sync = a.sync[a.rank];
  __shared__ unsigned int s_c;
  __shared__ int s_ok;
  const int src = blockIdx.x / a.ctas_per_src;
  const int part = blockIdx.x % a.ctas_per_src;
  if (threadIdx.x == 0) {
    const unsigned int c = rla_ld_relaxed_gpu_u32(sync + px::kSeq);
    const unsigned int aborted = rla_ld_relaxed_gpu_u32(sync + px::kAbort);
    s_c = c;
    s_ok = aborted == 0u;
    if (aborted != 0u && aborted != c) rla_record_error(RLA_DEVERR_PEER_POISONED);
  }
  __syncthreads();
  const unsigned int c = s_c;
  if (s_ok) {
    // announce this rank's block to every rank (idempotent across CTAs)
    if (threadIdx.x < a.world)
      px_st_release_sys(a.sync[threadIdx.x] + px::kReady + a.rank * px::kMaxBlocks + a.block, c);
    if (threadIdx.x == 0)
      s_ok = px_wait(sync + px::kReady + src * px::kMaxBlocks + a.block, c, sync, a.wait_ns) ? 1 : 0;
    __syncthreads();
  }
  if (s_ok) {
    // One warp per row of the source's slice: 16-byte loads, UNR in flight
    // per lane, consecutive lanes on consecutive 16-byte units (no index
    // division, a few instructions per unit, so the copy leaves the SM's
    // issue slots to the GEMM running beside it).
    constexpr int kWarps = px::kPullThreads / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunks = a.chunks;
    const uint4* __restrict__ from0 = a.xb[src] + a.row0 * a.ld_xb16;
    uint4* __restrict__ to0 = a.y + a.row0 * a.ldy16 + static_cast<int64_t>(src) * chunks;
    for (int r = part * kWarps + warp; r < a.rows; r += a.ctas_per_src * kWarps) {
      const uint4* __restrict__ from = from0 + static_cast<int64_t>(r) * a.ld_xb16;
      uint4* __restrict__ to = to0 + static_cast<int64_t>(r) * a.ldy16;
      int ch = lane;
      for (; ch + 32 * (UNR - 1) < chunks; ch += 32 * UNR) {
        uint4 v[UNR];
#pragma unroll
        for (int u = 0; u < UNR; ++u) v[u] = px_ld_cg(from + ch + 32 * u);
#pragma unroll
        for (int u = 0; u < UNR; ++u) to[ch + 32 * u] = v[u];
      }
      for (; ch < chunks; ch += 32) to[ch] = px_ld_cg(from + ch);
    }
  }
  if (a.last) {
    // The last CTA of the call's last pull tells every peer that this rank's
    // reads of call c are over (the earlier blocks' pulls completed before
    // this launch started).  Aborted calls send nothing: the peers' begin
    // then gives up too.
    __syncthreads();
    if (threadIdx.x == 0) {
      const unsigned int old = rla_arrive_acq_rel_gpu(sync + px::kTicket);
      if (old + 1u == gridDim.x && rla_ld_relaxed_gpu_u32(sync + px::kAbort) == 0u) {
        for (int d = 0; d < a.world; ++d)
          if (d != a.rank) px_st_release_sys(a.sync[d] + px::kDone + a.rank, c);
      }
    }
  }
}

}  // namespace rla

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace rla {
// The pull kernel runs beside the tcgen05 GEMM on the same SMs.  An SM's
// split between L1 and shared memory changes only when the SM is idle, so a
// pull CTA that lands on an idle SM with the default (small shared memory)
// split would keep the GEMM's CTAs (about 166 KB of shared memory each) off
// that SM until every pull CTA there has finished.  Asking for the largest
// shared-memory split keeps the SMs ready for the GEMM.  Once per device.
template <int UNR>
static cudaError_t px_prepare_pull_kernel() {
  static std::atomic<unsigned long long> done_mask{0};
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = d >= 0 && d < 64 ? (1ull << d) : 0ull;
  if (bit && (done_mask.load(std::memory_order_relaxed) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(px_pull_kernel<UNR>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess && bit) done_mask.fetch_or(bit, std::memory_order_relaxed);
  return e;
}

template <int UNR>
static cudaError_t px_launch_pull(const PxArgs& a, cudaStream_t stream) {
  const cudaError_t prep = px_prepare_pull_kernel<UNR>();
  if (prep != cudaSuccess) return prep;
  rla_clear_stale_launch_error();
  px_pull_kernel<UNR><<<a.world * a.ctas_per_src, px::kPullThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

static int px_fill_common(PxArgs& a, void* const* sync_peers, int rank, int world, const char* fn) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) {
    set_error("%s: need 1 <= world <= %d and 0 <= rank < world (got rank %d, world %d)", fn, kMaxPeers, rank, world);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (!sync_peers) {
    set_error("%s: need a host array of %d sync areas", fn, world);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  for (int d = 0; d < world; ++d) {
    if (!sync_peers[d] || (reinterpret_cast<uintptr_t>(sync_peers[d]) & 127u)) {
      set_error("%s: sync area %d is null or not 128-byte aligned", fn, d);
      return RLA_ERR_INVALID_ARGUMENT;
    }
    a.sync[d] = static_cast<unsigned int*>(sync_peers[d]);
  }
  a.rank = rank;
  a.world = world;
  a.wait_ns = g_peer_wait_ns.load(std::memory_order_relaxed);
  return RLA_OK;
}
}  // namespace rla

extern "C" {

int rla_prefill_exchange_begin(void* const* sync_peers, int rank, int world, void* stream) {
  using namespace rla;
  PxArgs a{};
  const int st = px_fill_common(a, sync_peers, rank, world, "rla_prefill_exchange_begin");
  if (st != RLA_OK) return st;
  rla_clear_stale_launch_error();
  px_begin_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("rla_prefill_exchange_begin: launch failed: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

int rla_prefill_exchange_block(const void* const* xb_peers, int64_t ld_xb, void* const* sync_peers, int rank,
                               int world, int block, int last, int64_t row0, int64_t rows, int64_t n_local, void* y,
                               int64_t ldy, void* stream) {
  using namespace rla;
  PxArgs a{};
  const char* fn = "rla_prefill_exchange_block";
  const int st = px_fill_common(a, sync_peers, rank, world, fn);
  if (st != RLA_OK) return st;
  if (!xb_peers || !y || (reinterpret_cast<uintptr_t>(y) & 15u)) {
    set_error("%s: need a host array of %d exchange buffers and a 16-byte aligned y", fn, world);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  for (int d = 0; d < world; ++d) {
    if (!xb_peers[d] || (reinterpret_cast<uintptr_t>(xb_peers[d]) & 15u)) {
      set_error("%s: exchange buffer %d is null or not 16-byte aligned", fn, d);
      return RLA_ERR_INVALID_ARGUMENT;
    }
    a.xb[d] = static_cast<const uint4*>(xb_peers[d]);
  }
  if (block < 0 || block >= RLA_PX_MAX_BLOCKS) {
    set_error("%s: block must be in [0, %d), got %d", fn, RLA_PX_MAX_BLOCKS, block);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  if (row0 < 0 || rows < 0 || n_local < 1 || n_local % 8 != 0 || ld_xb < n_local || ld_xb % 8 != 0 ||
      ldy < (int64_t)world * n_local || ldy % 8 != 0) {
    set_error("%s: need row0, rows >= 0, n_local a positive multiple of 8, ld_xb >= n_local and "
              "ldy >= world * n_local, both multiples of 8 (got row0=%lld rows=%lld n_local=%lld ld_xb=%lld "
              "ldy=%lld)", fn, (long long)row0, (long long)rows, (long long)n_local, (long long)ld_xb,
              (long long)ldy);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  const int64_t chunks = n_local / 8;
  if (rows >= (int64_t(1) << 31) || chunks >= (int64_t(1) << 30)) {
    set_error("%s: a block of %lld rows x %lld columns is too large (rows < 2^31, n_local < 2^33)", fn,
              (long long)rows, (long long)n_local);
    return RLA_ERR_INVALID_ARGUMENT;
  }
  a.y = static_cast<uint4*>(y);
  a.ld_xb16 = ld_xb / 8;
  a.ldy16 = ldy / 8;
  a.row0 = row0;
  a.rows = static_cast<int>(rows);
  a.chunks = static_cast<int>(chunks);
  a.block = block;
  a.last = last ? 1 : 0;
  // about one CTA per SM in all (it fits beside a GEMM CTA), one warp per
  // row, fewer CTAs when a block has fewer rows than that
  const int warps = px::kPullThreads / 32;
  const int64_t want = (device_sm_count() + world - 1) / world;
  a.ctas_per_src = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, (rows + warps - 1) / warps)));
  int unroll = 4;
#ifdef RLA_EXPERIMENTS
  unroll = exp_int("RLA_PX_UNROLL", unroll);
  if (const int c = exp_int("RLA_PX_CTAS", 0); c > 0)
    a.ctas_per_src = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((c + world - 1) / world,
                                                                            (rows + warps - 1) / warps)));
#endif
  const cudaError_t e = unroll == 8 ? px_launch_pull<8>(a, static_cast<cudaStream_t>(stream))
                                    : px_launch_pull<4>(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", fn, cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

}  // extern "C"
