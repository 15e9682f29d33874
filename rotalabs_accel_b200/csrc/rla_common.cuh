// Shared device helpers for the sm_100a W8A16 kernels: int8 -> fp16
// conversion, bounded mbarrier waits, TMA and tcgen05 (TMEM / UMMA) wrappers.
//
// Every wait on another thread's progress is bounded by a wall-clock limit
// (%globaltimer).  On timeout the waiting thread records an error code in
// rla_device_error (read by the host through rla_get_device_error()) and the
// kernel unwinds instead of spinning forever.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define RLA_DEVFN __device__ __forceinline__

// Device-side error word: 0 = fine, otherwise the first error recorded.
// (The library is built as one translation unit, rla_lib.cu, so this is the
// only definition.)
__device__ unsigned int rla_device_error = 0;

enum : unsigned int {
  RLA_DEVERR_NONE = 0,
  RLA_DEVERR_TIMEOUT_TMA_FULL = 1,
  RLA_DEVERR_TIMEOUT_SLOT_EMPTY = 2,
  RLA_DEVERR_TIMEOUT_A_FULL = 3,
  RLA_DEVERR_TIMEOUT_A_EMPTY = 4,
  RLA_DEVERR_TIMEOUT_ACCUM = 5,
  RLA_DEVERR_TIMEOUT_SPLITK = 6,
  RLA_DEVERR_TIMEOUT_PEER_DATA = 7,  // a peer's slice of an exchange call did not arrive
  RLA_DEVERR_TIMEOUT_GRID = 8,       // CTAs of an exchange launch did not all finish their slice
  RLA_DEVERR_PEER_POISONED = 9,      // an exchange call on a sync area whose earlier wait gave up
};

// One second: far above any legitimate wait inside one launch.
#define RLA_WAIT_LIMIT_NS 1000000000ull

RLA_DEVFN uint64_t rla_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

RLA_DEVFN void rla_record_error(unsigned int code) { atomicCAS(&rla_device_error, 0u, code); }

// Before a <<<...>>> launch whose status is read with cudaGetLastError():
// drop a non-sticky error left by an earlier failed call (already returned to
// that call's caller), so the status read after the launch is this launch's.
static inline void rla_clear_stale_launch_error() { (void)cudaGetLastError(); }

// Split-K / stream-K arrival: one acquire-release atomic at gpu scope.  The
// release publishes every store the caller's CTA made before its barrier
// (cumulativity); the acquire makes the other CTAs' published stores visible
// to the caller and, through the next CTA barrier, to its whole CTA.
RLA_DEVFN unsigned int rla_arrive_acq_rel_gpu(unsigned int* counter) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  return old;
}

// ---------------------------------------------------------------------------
// int8 -> fp16, four values per 32-bit word.
//
// Published method ("magic number" conversion; Kim et al. 2022, "Who Says
// Elephants Can't Run: Bringing Large Scale MoE Models into Cloud Scale
// Production", as used in FasterTransformer): flip the sign bit so each byte
// holds b + 128 in [0, 255], splice each byte under the fp16 exponent byte
// 0x64 so the half reads 1024 + (b + 128) exactly, then subtract 1152.
// Two byte-permutes and two half2 subtractions per four values, all exact.
// ---------------------------------------------------------------------------
RLA_DEVFN void rla_i8x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a, b;
  // result bytes: [u.b0, 0x64, u.b1, 0x64] and [u.b2, 0x64, u.b3, 0x64]
  asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(b) : "r"(u), "r"(0x64646464u));
  const uint32_t bias = 0x64806480u;  // (1152, 1152) as half2
  asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(bias));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(bias));
}

// SwiGLU of one output: fp16(silu(g) * u), silu(g) = g * sigmoid(g) =
// g / (1 + e^-g), in fp32, from gate and up values already rounded to fp16
// (the rounding points of a gate GEMM, an up GEMM and a separate SwiGLU pass).
// Fast-math intrinsics: their few-ulp fp32 error is far below the fp16
// rounding that follows; for g <= -89, e^-g overflows to inf and the quotient
// is the correct limit -0.
RLA_DEVFN __half rla_swiglu(float gate, float up) {
  const float2 gu = __half22float2(__floats2half2_rn(gate, up));
  return __float2half_rn(__fdividef(gu.x, 1.0f + __expf(-gu.x)) * gu.y);
}

// ---------------------------------------------------------------------------
// Global loads
// ---------------------------------------------------------------------------
// Streaming 16-byte load of weights: read once, keep out of L1.
RLA_DEVFN uint4 rla_ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// 16-byte load of activations: shared by every warp of the CTA, keep in L1.
RLA_DEVFN uint4 rla_ldg_keep(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Legacy warp-level MMA m16n8k16, fp16 inputs, fp32 accumulate.  Used by the
// HBM-bound decode kernel, where tensor throughput is not the limit.
// ---------------------------------------------------------------------------
RLA_DEVFN void rla_mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start before its predecessor in the stream has finished;
// griddepcontrol.wait blocks until the predecessor has completed and its
// memory is visible, so every read of data a predecessor may write comes
// after it.  launch_dependents lets the next such kernel start launching.
// Both are no-ops for a kernel launched without the attribute.
// ---------------------------------------------------------------------------
RLA_DEVFN void rla_griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
RLA_DEVFN void rla_griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// Pull the cache line holding `p` into L2 (never stale: L2 is coherent).
RLA_DEVFN void rla_prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }
// Pull the cache line holding `p` into this SM's L1.  Only for data that no
// kernel running at the same time writes (here: after the dependency wait).
RLA_DEVFN void rla_prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

// ---------------------------------------------------------------------------
// Thread-block clusters: rank, barrier, distributed shared memory.
// ---------------------------------------------------------------------------
RLA_DEVFN uint32_t rla_cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
RLA_DEVFN uint32_t rla_cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster: stores before it are visible to
// the cluster's loads after it.
RLA_DEVFN void rla_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 16-byte load from CTA `rank`'s copy of the shared variable at `p`.
RLA_DEVFN float4 rla_ld_dsmem_f4(const void* p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// ---------------------------------------------------------------------------
// Shared memory / mbarrier
// ---------------------------------------------------------------------------
RLA_DEVFN uint32_t rla_smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

RLA_DEVFN void rla_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(rla_smem_u32(bar)), "r"(count));
}
RLA_DEVFN void rla_fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
RLA_DEVFN void rla_fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

RLA_DEVFN void rla_mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(rla_smem_u32(bar))
      : "memory");
}
RLA_DEVFN void rla_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(rla_smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
RLA_DEVFN bool rla_mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(rla_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Same, but the thread may be suspended in hardware for up to `hint_ns`
// while the phase is incomplete (no issue slots spent polling).
RLA_DEVFN bool rla_mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(rla_smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.  Returns
// false (after recording `err`) if it did not complete within the limit or
// if *abort_flag was raised by another warp of this CTA.
RLA_DEVFN bool rla_mbar_wait(uint64_t* bar, uint32_t parity, unsigned int err, volatile int* abort_flag) {
  if (rla_mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = rla_globaltimer();
  uint32_t spins = 0;
  while (true) {
    if (rla_mbar_try_wait_sleep(bar, parity, 1000u)) return true;
    if ((++spins & 15u) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (rla_globaltimer() - t0 > RLA_WAIT_LIMIT_NS) {
        rla_record_error(err);
        if (abort_flag) *abort_flag = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor copies, no multicast)
// ---------------------------------------------------------------------------
RLA_DEVFN void rla_tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(desc) : "memory");
}
RLA_DEVFN void rla_tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(rla_smem_u32(smem_dst)),
      "l"(desc), "r"(rla_smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: Tensor Memory and the 5th-generation tensor-core MMA
// ---------------------------------------------------------------------------
RLA_DEVFN void rla_tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   rla_smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
RLA_DEVFN void rla_tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
RLA_DEVFN void rla_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
RLA_DEVFN void rla_tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
RLA_DEVFN void rla_tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate).
RLA_DEVFN void rla_umma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
RLA_DEVFN void rla_umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   rla_smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i <-> lane (base + i).
RLA_DEVFN void rla_tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns.
RLA_DEVFN void rla_tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
RLA_DEVFN void rla_tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

RLA_DEVFN void rla_tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),
        "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
        "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
RLA_DEVFN void rla_tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format) for a K-major operand
// stored in the 128-byte-swizzled canonical layout: rows of 128 bytes, 8-row
// (1024-byte) swizzle atoms stacked along M/N.
//   bits  0-13 start address >> 4     bits 16-29 leading-dim byte offset >> 4
//   bits 32-45 stride-dim byte offset >> 4   bits 46-47 version (1)
//   bits 49-51 base offset (0: atoms 1024-byte aligned)   bits 61-63 layout (2 = 128B swizzle)
RLA_DEVFN uint64_t rla_smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // SBO: next 8-row group
  d |= static_cast<uint64_t>(1u) << 46;            // descriptor version for tcgen05
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, shape MxN.
__host__ __device__ constexpr uint32_t rla_idesc_f16_f32(int M, int N) {
  return (1u << 4)                                   // D format: f32
         | (0u << 7) | (0u << 10)                    // A, B format: f16
         | (0u << 15) | (0u << 16)                   // A, B K-major
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}
