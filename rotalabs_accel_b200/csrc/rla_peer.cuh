// Device side of the direct peer-to-peer output exchange (column-parallel
// decode over several GPUs, one process per GPU).
//
// Every rank runs the same sequence of exchange calls; rank r computes output
// columns [r * n_local, (r + 1) * n_local) of every row.  Call s of rank r:
//
//  * Phase 1 (the GEMM's epilogue).  Each output element of r's slice goes
//    to r's own y with a plain store, and to every peer d as part of an 8-byte
//    "flagged word" {fp16 y[2p][n], fp16 y[2p+1][n], s} stored over NVLink into
//    d's receive buffer.  An aligned 8-byte store is seen whole or not at
//    all, so a reader that finds the flag s in a word has its data: no fence,
//    no separate completion flag (the low-latency protocol NCCL calls LL).
//  * Phase 2 (unpacking).  When the whole grid is resident at once, every
//    CTA unpacks its share right after its own phase 1.  Otherwise every CTA
//    takes a ticket when its phase 1 is done, and the last R CTAs to finish
//    wait until all CTAs of the launch have taken one.  Unpacking CTAs poll
//    the receive buffer for every peer's words of call s and write them into
//    y.  When the kernel completes, y holds all slices.
//
// Reuse without a handshake: receive buffers are double-buffered by the
// parity of s.  A rank writes a peer's parity-p half in call s only after its
// own call s - 1 has completed, which needed the peer's words of call s - 1,
// which the peer wrote after its call s - 2 -- the last reader of that half --
// had completed.  Stale words carry older call numbers.  (Every phase-1 store
// comes after the kernel's dependency wait, so this holds with programmatic
// dependent launch too.)
//
// No cross-GPU deadlock: phase 1 waits on nothing outside the GPU.  With the
// whole grid resident, every CTA of a launch runs its phase 1 whatever the
// others wait for.  Otherwise a CTA waits on peers only after every CTA of
// its own launch has finished phase 1, and R <= (resident CTAs + 1) / 2
// leaves room for every CTA that has not yet run.  (Programmatic dependent
// launch does not change this: a dependent grid starts only after every CTA
// of this grid has started.)
//
// The call number s is one more than the calls this rank has completed (a
// counter in its sync area, advanced by the last unpacking CTA).  Every wait is
// bounded by PeerOut::wait_ns; a wait that gives up records a device error and
// marks the exchange aborted: the other waits of the call stop at once (y is
// then incomplete), and so do those of every later call on the same sync area
// (device error RLA_DEVERR_PEER_POISONED), until the exchange is set up again.
#pragma once

#include "rla_common.cuh"
#include "rla_internal.h"

namespace rla {

RLA_DEVFN unsigned int rla_ld_relaxed_gpu_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// One flagged word {data (low 32 bits), flag (high 32 bits)}: one aligned
// scalar 64-bit access each way.  A naturally aligned scalar access is
// single-copy atomic in the PTX memory model, so a reader sees the flag and
// the data of the same store.  (A vector access such as v2.u32 is two 32-bit
// accesses in unspecified order, which would not give this guarantee.)
RLA_DEVFN void rla_st_flagged(uint2* p, uint32_t data, uint32_t flag) {
  const uint64_t v = static_cast<uint64_t>(data) | (static_cast<uint64_t>(flag) << 32);
  asm volatile("st.volatile.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
RLA_DEVFN uint2 rla_ld_flagged(const uint2* p) {
  uint64_t v;
  asm volatile("ld.volatile.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return make_uint2(static_cast<uint32_t>(v), static_cast<uint32_t>(v >> 32));
}
// Two consecutive flagged words (16-byte aligned) in one load: two 64-bit
// elements, each single-copy atomic on its own; each word carries its own
// flag, so the pair needs no more than that.
RLA_DEVFN void rla_ld_flagged2(const uint2* p, uint2& a, uint2& b) {
  uint64_t u, v;
  asm volatile("ld.volatile.global.v2.b64 {%0, %1}, [%2];" : "=l"(u), "=l"(v) : "l"(p) : "memory");
  a = make_uint2(static_cast<uint32_t>(u), static_cast<uint32_t>(u >> 32));
  b = make_uint2(static_cast<uint32_t>(v), static_cast<uint32_t>(v >> 32));
}

// This launch's call number.  Read after the dependency wait: the previous
// exchange call in the stream has completed and advanced the counter.
RLA_DEVFN unsigned int peer_call(const PeerOut& po) { return rla_ld_relaxed_gpu_u32(po.sync + kSyncSeq) + 1u; }

// Flagged word (pair p, column n) of `src`'s slice in rank d's receive buffer.
RLA_DEVFN uint2* peer_word(const PeerOut& po, int d, unsigned int s, int src, int64_t pair_col) {
  return po.recv[d] + (int64_t)(s & 1u) * po.half_words + (int64_t)src * po.slot_words + pair_col;
}

// Phase 1 for rows (2p, 2p+1) of local column n: this rank's y directly,
// every peer one flagged word.  v1 is ignored when row 2p+1 does not exist.
RLA_DEVFN void peer_store_pair(const PeerOut& po, unsigned int s, __half* y, int64_t ldy, int M, int n_local, int p,
                               int n, __half v0, __half v1) {
  const int m = 2 * p;
  const int64_t col = (int64_t)po.rank * n_local + n;
  y[(int64_t)m * ldy + col] = v0;
  if (m + 1 < M) y[(int64_t)(m + 1) * ldy + col] = v1;
  const uint32_t data = static_cast<uint32_t>(__half_as_ushort(v0)) |
                        (static_cast<uint32_t>(__half_as_ushort(v1)) << 16);
  const int64_t pc = (int64_t)p * n_local + n;
  for (int d = 0; d < po.world; ++d)
    if (d != po.rank) rla_st_flagged(peer_word(po, d, s, po.rank, pc), data, s);
}

// Bounded wait for one flagged word of call s (t0: start of the wait phase).
RLA_DEVFN bool peer_wait_word(const PeerOut& po, const uint2* w, unsigned int s, uint2& out, uint64_t t0) {
  out = rla_ld_flagged(w);
  if (out.y == s) return true;
  const unsigned int* abort_word = po.sync + kSyncAbort;
  while (true) {
    __nanosleep(100);
    out = rla_ld_flagged(w);
    if (out.y == s) return true;
    if (rla_ld_relaxed_gpu_u32(abort_word) != 0u) return false;  // a wait of this call gave up
    if (rla_globaltimer() - t0 > po.wait_ns) {
      rla_record_error(RLA_DEVERR_TIMEOUT_PEER_DATA);
      atomicExch(po.sync + kSyncAbort, s);
      return false;
    }
  }
}

// One received flagged word (pair p, column n of source rank src; pc = p *
// n_local + n < 2^31) into y.
RLA_DEVFN void peer_unpack_word(uint2 v, __half* y, int64_t ldy, int M, int n_local, int src, uint32_t pc) {
  const uint32_t p = pc / static_cast<uint32_t>(n_local);
  const uint32_t n = pc - p * static_cast<uint32_t>(n_local);
  const int64_t col = (int64_t)src * n_local + n;
  y[(int64_t)(2 * p) * ldy + col] = __ushort_as_half(static_cast<unsigned short>(v.x & 0xffffu));
  if (2 * (int)p + 1 < M) y[(int64_t)(2 * p + 1) * ldy + col] = __ushort_as_half(static_cast<unsigned short>(v.x >> 16));
}
// Two received words of consecutive columns n, n + 1 (n even, same pair p)
// into y as two 4-byte stores (y's rows and columns are 4-byte aligned:
// ldy and the column are even).
RLA_DEVFN void peer_unpack_word2(uint2 a, uint2 b, __half* y, int64_t ldy, int M, int n_local, int src, uint32_t pc) {
  const uint32_t p = pc / static_cast<uint32_t>(n_local);
  const uint32_t n = pc - p * static_cast<uint32_t>(n_local);
  const int64_t col = (int64_t)src * n_local + n;
  *reinterpret_cast<uint32_t*>(y + (int64_t)(2 * p) * ldy + col) = (a.x & 0xffffu) | (b.x << 16);
  if (2 * (int)p + 1 < M)
    *reinterpret_cast<uint32_t*>(y + (int64_t)(2 * p + 1) * ldy + col) = (a.x >> 16) | (b.x & 0xffff0000u);
}

// Phase 2.  Called by the `nthreads` threads of a CTA that take part in named
// barrier `bar_id` (thread index tid), after their last phase-1 store; `slot`
// is a shared-memory int of the CTA.
//
// An exchange whose wait once gave up stays failed: the abort word of the
// sync area is never cleared, and every later call records
// RLA_DEVERR_PEER_POISONED and skips its waits at once (y incomplete) instead
// of waiting out its own limit.  The exchange must be closed and set up again
// by every rank.
RLA_DEVFN void peer_finish(const PeerOut& po, unsigned int s, __half* y, int64_t ldy, int M, int n_local, int tid,
                           int nthreads, int bar_id, int* slot) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  const unsigned int ctas = gridDim.x * gridDim.y;
  const unsigned int R = po.unpackers;
  // When the whole grid is resident at once (R == ctas) every CTA unpacks as
  // soon as its own phase 1 is done: no CTA of this launch can be kept from
  // running by the waiting ones, so the grid-wide arrival wait (and the
  // polling of one counter by every CTA, which slows the arrivals themselves)
  // is not needed; a CTA's share follows from its index.
  const bool resident_grid = R == ctas;
  if (tid == 0) {
    if (resident_grid) {
      *slot = static_cast<int>(blockIdx.y * gridDim.x + blockIdx.x);
    } else {
      const unsigned int ticket = atomicAdd(po.sync + kSyncArrive, 1u);
      *slot = ticket >= ctas - R ? static_cast<int>(ticket - (ctas - R)) : -1;
    }
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  const int u = *slot;
  if (u < 0) return;  // not an unpacker: this CTA is done
  const uint64_t t0 = rla_globaltimer();
  const bool poisoned = rla_ld_relaxed_gpu_u32(po.sync + kSyncAbort) != 0u;  // an earlier call gave up
  if (tid == 0) {
    if (poisoned) {
      rla_record_error(RLA_DEVERR_PEER_POISONED);
    } else if (!resident_grid) {
      // Wait until every CTA of the launch has finished phase 1.
      while (rla_ld_relaxed_gpu_u32(po.sync + kSyncArrive) < ctas) {
        if (rla_ld_relaxed_gpu_u32(po.sync + kSyncAbort) != 0u) break;
        if (rla_globaltimer() - t0 > po.wait_ns) {
          rla_record_error(RLA_DEVERR_TIMEOUT_GRID);
          atomicExch(po.sync + kSyncAbort, s);
          break;
        }
        __nanosleep(100);
      }
    }
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  const int pairs = (M + 1) / 2;
  const int64_t per_src = (int64_t)pairs * n_local;
  const int64_t total = per_src * (po.world - 1);
  // Units of two words (one 16-byte load) when every source slot starts on a
  // 16-byte boundary, else single words.  Each thread issues kBatch unit
  // loads before it looks at any flag; a word whose flag is not yet s is then
  // waited for on its own.
  const int wpu = (po.half_words % 2 == 0 && per_src % 2 == 0) ? 2 : 1;
  // Two words of one unit are columns n, n + 1 of one pair when n_local is
  // even (per_src even and every unit starts on an even word); they then go
  // to y as 4-byte stores when y's rows keep 4-byte alignment.
  const bool store2 = wpu == 2 && n_local % 2 == 0 && ldy % 2 == 0 && (reinterpret_cast<uintptr_t>(y) & 3u) == 0;
  // Index arithmetic in 32 bits: the host limits M to 32 and n_local to
  // 2^31, and total = pairs * n_local * (world - 1) < 2^32 for every
  // decode shard (16 * 28672 * 7 words at most in the 70B layers).
  const uint32_t units = static_cast<uint32_t>(total / wpu);
  const uint32_t per_src32 = static_cast<uint32_t>(per_src);
  const uint32_t stride = R * static_cast<uint32_t>(nthreads);
  constexpr int kBatch = 4;
  bool live = !poisoned;
  for (uint32_t base = static_cast<uint32_t>(u) * nthreads + tid; live && base < units; base += kBatch * stride) {
    uint2 v[kBatch][2];
    int src[kBatch];
    uint32_t pc[kBatch];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const uint32_t unit = base + b * stride;
      src[b] = -1;
      if (unit < units) {
        const uint32_t w = unit * wpu;
        const int si = static_cast<int>(w / per_src32);
        src[b] = si < po.rank ? si : si + 1;
        pc[b] = w - static_cast<uint32_t>(si) * per_src32;
        const uint2* a = peer_word(po, po.rank, s, src[b], pc[b]);
        if (wpu == 2) rla_ld_flagged2(a, v[b][0], v[b][1]);
        else v[b][0] = rla_ld_flagged(a);
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      if (src[b] < 0 || !live) continue;
      for (int j = 0; j < wpu; ++j) {
        if (v[b][j].y != s && !peer_wait_word(po, peer_word(po, po.rank, s, src[b], pc[b] + j), s, v[b][j], t0)) {
          live = false;
          break;
        }
      }
      if (!live) break;
      if (store2) {
        peer_unpack_word2(v[b][0], v[b][1], y, ldy, M, n_local, src[b], pc[b]);
      } else {
        for (int j = 0; j < wpu; ++j) peer_unpack_word(v[b][j], y, ldy, M, n_local, src[b], pc[b] + j);
      }
    }
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  if (tid == 0) {
    const unsigned int done = atomicAdd(po.sync + kSyncUnpacked, 1u);
    if (done == R - 1) {
      // Last unpacker: every CTA has taken its ticket and every unpacker has
      // stopped reading the counters; the next launch reads them only after
      // this one has completed.
      po.sync[kSyncArrive] = 0u;
      po.sync[kSyncUnpacked] = 0u;
      po.sync[kSyncSeq] = s;
    }
  }
}

// The same phase as an out-of-line call.  The decode kernel's forms with two
// or more token tiles use it: with the unpacking code kept out of the
// kernel body, the compiler's register choice for the GEMM part runs them
// faster (one GPU, world-1 exchange, M = 16: 8192 -> 14336 65-73 -> 46 us,
// 28672 -> 4096 48-51 -> 40 us, 8192 -> 3584 15.6-17.3 -> 14.0 us,
// 28672 -> 1024 16.0-16.5 -> 15.1 us), while the one-tile forms run slower
// that way (M = 1: 28.8 -> 41.9 us on 8192 -> 14336) and keep it inline.
__device__ __noinline__ void peer_finish_call(const PeerOut& po, unsigned int s, __half* y, int64_t ldy, int M,
                                              int n_local, int tid, int nthreads, int bar_id, int* slot) {
  peer_finish(po, s, y, ldy, M, n_local, tid, nthreads, bar_id, slot);
}

}  // namespace rla
