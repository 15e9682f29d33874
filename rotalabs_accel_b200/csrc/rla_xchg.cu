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
//        copies from, then moves that rank's rows of the block from xb[src]
//        (over NVLink for a peer) into y[rows, src * n_local : (src + 1) *
//        n_local] with bulk copies through shared memory;
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
// reads of the previous call.  A pull CTA is one warp with 48 KB of shared
// memory, so it fits beside a tcgen05 GEMM CTA on the same SM.
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
constexpr int kSlots = 3;             // pull ring: slots of shared memory per CTA
constexpr int kSlotBytes = 16384;
constexpr int kPullSmem = kSlots * kSlotBytes;
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

// ---------------------------------------------------------------------------
// The pull moves bytes with the SM's bulk-copy engine (TMA, untiled): one warp
// per CTA, its lane 0 streams the source's rows through a ring of
// shared-memory slots -- a bulk load from the source's exchange buffer (over
// NVLink for a peer) completing on an mbarrier, then a bulk store into y.
// Few instructions per byte and no load/store-unit traffic, so the pull
// costs the GEMM running beside it on the same SMs as little as it can.
// Plain loads, no multicast.  A CTA's rows are one contiguous range; a slot
// holds whole rows when they fit (one load for several rows, one store per
// row), else one piece of a row.
// ---------------------------------------------------------------------------
RLA_DEVFN void px_bulk_load(void* smem, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  rla_mbar_arrive_expect_tx(bar, bytes);
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   rla_smem_u32(smem)),
               "l"(gsrc), "r"(bytes), "r"(rla_smem_u32(bar))
               : "memory");
}
RLA_DEVFN void px_bulk_store(void* gdst, const void* smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(rla_smem_u32(smem)),
               "r"(bytes)
               : "memory");
}
RLA_DEVFN void px_bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
RLA_DEVFN void px_bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
RLA_DEVFN void px_bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// After a failed wait: wait (bounded again) for a bulk load this CTA issued,
// so that no copy into its shared memory is in flight when it exits.
RLA_DEVFN void px_drain_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = rla_globaltimer();
  while (!rla_mbar_try_wait_sleep(bar, parity, 1000u))
    if (rla_globaltimer() - t0 > limit_ns) return;
}

// Piece walker over rows [r, re) of one CTA: a piece is `nr` whole rows
// (rows_per_slot of them at most) or bytes [off, off + len) of one row.
struct PxPiece {
  int r, re, nr;
  uint32_t off, len;
  uint32_t rowbytes;
  uint32_t slot_bytes;
  int rows_per_slot;  // 0: rows larger than a slot
  RLA_DEVFN bool valid() const { return r < re; }
  RLA_DEVFN void settle() {
    if (rows_per_slot > 0) {
      nr = min(rows_per_slot, re - r);
      off = 0;
      len = static_cast<uint32_t>(nr) * rowbytes;
    } else {
      nr = 1;
      len = min(slot_bytes, rowbytes - off);
    }
  }
  RLA_DEVFN void next() {
    if (rows_per_slot > 0) {
      r += nr;
    } else {
      off += len;
      if (off >= rowbytes) {
        off = 0;
        ++r;
      }
    }
    settle();
  }
};

__global__ void __launch_bounds__(32) px_pull_kernel(PxArgs a) {
  extern __shared__ __align__(128) unsigned char px_ring[];
  __shared__ __align__(8) uint64_t bars[px::kSlots];
  __shared__ int s_abort;
  unsigned int* sync = a.sync[a.rank];
  const int src = blockIdx.x / a.ctas_per_src;
  const int part = blockIdx.x % a.ctas_per_src;
  const int lane = threadIdx.x;
  unsigned int c = 0;
  bool ok = false;
  if (lane == 0) {
    c = rla_ld_relaxed_gpu_u32(sync + px::kSeq);
    const unsigned int aborted = rla_ld_relaxed_gpu_u32(sync + px::kAbort);
    ok = aborted == 0u;
    if (aborted != 0u && aborted != c) rla_record_error(RLA_DEVERR_PEER_POISONED);
  }
  c = __shfl_sync(0xffffffffu, c, 0);
  ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
  if (ok && lane < a.world) px_st_release_sys(a.sync[lane] + px::kReady + a.rank * px::kMaxBlocks + a.block, c);
  if (ok && lane == 0) {
    ok = px_wait(sync + px::kReady + src * px::kMaxBlocks + a.block, c, sync, a.wait_ns);
    s_abort = 0;
    for (int i = 0; i < px::kSlots; ++i) rla_mbar_init(&bars[i], 1);
    rla_fence_barrier_init();
    // the source's rows were written by generic stores (its GEMM) and are
    // read here by the bulk-copy (async) proxy
    asm volatile("fence.proxy.async;" ::: "memory");
  }
  if (ok && lane == 0) {
    const int per = (a.rows + a.ctas_per_src - 1) / a.ctas_per_src;
    const int rb = min(a.rows, part * per), re = min(a.rows, rb + per);
    const uint32_t rowbytes = static_cast<uint32_t>(a.chunks) * 16u;
    const bool packed = a.ld_xb16 == a.chunks && rowbytes <= static_cast<uint32_t>(px::kSlotBytes);
    const int rps = packed ? static_cast<int>(px::kSlotBytes / rowbytes) : 0;
    const char* from = reinterpret_cast<const char*>(a.xb[src] + a.row0 * a.ld_xb16);
    char* to = reinterpret_cast<char*>(a.y + a.row0 * a.ldy16 + static_cast<int64_t>(src) * a.chunks);
    const int64_t ld_from = a.ld_xb16 * 16, ld_to = a.ldy16 * 16;
    PxPiece li{rb, re, 0, 0u, 0u, rowbytes, static_cast<uint32_t>(px::kSlotBytes), rps};
    li.settle();
    PxPiece si = li;
    int issued = 0, done = 0;
    while (issued < px::kSlots && li.valid()) {
      px_bulk_load(px_ring + issued * px::kSlotBytes, from + li.r * ld_from + li.off, li.len, &bars[issued]);
      li.next();
      ++issued;
    }
    bool good = true;
    while (done < issued) {
      const int slot = done % px::kSlots;
      const uint32_t parity = static_cast<uint32_t>(done / px::kSlots) & 1u;
      if (good && !rla_mbar_wait(&bars[slot], parity, RLA_DEVERR_TIMEOUT_PEER_DATA, &s_abort)) good = false;
      if (!good) px_drain_wait(&bars[slot], parity, a.wait_ns);  // a load in flight must land before exit
      if (good) {
        const unsigned char* sm = px_ring + slot * px::kSlotBytes;
        for (int i = 0; i < si.nr; ++i)
          px_bulk_store(to + (si.r + i) * ld_to + si.off, sm + i * si.rowbytes, si.nr > 1 ? si.rowbytes : si.len);
        px_bulk_commit();
        si.next();
      }
      ++done;
      if (good && li.valid()) {
        px_bulk_wait_read_all();  // the slot's data has left for y: reuse it
        px_bulk_load(px_ring + slot * px::kSlotBytes, from + li.r * ld_from + li.off, li.len, &bars[slot]);
        li.next();
        ++issued;
      }
    }
    px_bulk_wait_all();
    asm volatile("fence.proxy.async;" ::: "memory");
    if (!good) atomicCAS(sync + px::kAbort, 0u, c);
  }
  if (a.last) {
    __syncwarp();
    if (lane == 0) {
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
// The pull kernel runs beside the tcgen05 GEMM on the same SMs (48 KB of
// shared memory next to the GEMM's ~166 KB).  An SM's split between L1 and
// shared memory changes only when the SM is idle, so the kernel asks for the
// largest shared-memory split: a pull CTA that lands on an idle SM then
// leaves room for a GEMM CTA.  Attributes set once per device.
static cudaError_t px_launch_pull(PxArgs a, int ctas_total, cudaStream_t stream) {
  static std::atomic<unsigned long long> done_mask{0};
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = d >= 0 && d < 64 ? (1ull << d) : 0ull;
  if (!bit || !(done_mask.load(std::memory_order_relaxed) & bit)) {
    e = cudaFuncSetAttribute(px_pull_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, px::kPullSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(px_pull_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    if (bit) done_mask.fetch_or(bit, std::memory_order_relaxed);
  }
  // one single-warp CTA per SM in all, each over a contiguous range of rows
  a.ctas_per_src = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>((ctas_total + a.world - 1) / a.world, a.rows)));
  rla_clear_stale_launch_error();
  px_pull_kernel<<<a.world * a.ctas_per_src, 32, px::kPullSmem, stream>>>(a);
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
  int ctas_total = device_sm_count();
#ifdef RLA_EXPERIMENTS
  ctas_total = exp_int("RLA_PX_CTAS", ctas_total);
#endif
  const cudaError_t e = px_launch_pull(a, ctas_total, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", fn, cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

}  // extern "C"
