// C ABI entry points and the per-shape kernel selector.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "rla_internal.h"

namespace rla {
cudaError_t launch_quantize(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int8_t* q, int64_t ldq,
                            float* scale, cudaStream_t s);
cudaError_t launch_gather(const void* staging, int64_t world, int64_t M, int64_t nl, void* y, int64_t ldy,
                          cudaStream_t s);

static std::atomic<uint64_t> g_launches{0};
static thread_local char g_err[512] = "";

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

static constexpr int kNumSMs = 148;  // B200; refined from the device at run time

#ifdef RLA_EXPERIMENTS
// Experiment builds only (never the shipped library): plan overrides from the
// environment, for A/B timing of plan rules.
static int exp_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}
#endif

int device_sm_count() {
  static std::atomic<int> cache[64];  // per device; 0 = not read yet
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kNumSMs;
  if (dev >= 0 && dev < 64 && (n = cache[dev].load(std::memory_order_relaxed)) > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return kNumSMs;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// ---------------------------------------------------------------------------
// The selector.  Static rules keyed on (M, N, K); no run-time autotuning.
//
// Skinny kernel (M <= 32): the weight stream is the whole cost, so the plan
// aims at enough independent 16-byte loads in flight on every SM
// (Little's law: ~6.5 TB/s x ~1 us => several MB in flight machine-wide).
// A CTA is 8 warps; rows per CTA and k-slicing are picked by K, and split-K
// across CTAs is added only while the whole grid stays resident (one wave).
//
// tcgen05 kernel (M > 32): tile 128 weight rows x BM tokens; BM = 256 for
// long prefills, smaller for mid-size M so that the grid covers the SMs.
// ---------------------------------------------------------------------------
static void skinny_shape(Plan& p, int64_t M, int64_t N, int64_t K, bool have_ws, int sms, bool gated = false,
                         bool peer = false) {
  p.kernel = RLA_KERNEL_SKINNY;
  p.nt = M <= 8 ? 1 : M <= 16 ? 2 : 4;
  const int64_t chunks = (K + 63) / 64;
  // Prefer more rows per CTA when K is short (fewer chunks to spread over warps).
  if (chunks >= 64) {
    p.wn = 1; p.wk = 8;
  } else if (chunks >= 16) {
    p.wn = 2; p.wk = 4;
  } else {
    p.wn = 4; p.wk = 2;
  }
  const int rows = 16 * p.wn;
  p.grid_x = static_cast<int>((N + rows - 1) / rows);
  // A grid of more 256-thread CTAs than fit on the GPU at once runs a last,
  // mostly empty wave; 128-thread CTAs (four k-warps) fit about twice as many
  // per SM and shorten or remove it.  Measured on B200: 4096 -> 11008 at
  // M = 1, 688 CTAs, 15.7 -> 11.1 us; 4096 -> 14336 at M = 1, 896 CTAs,
  // 16.4 -> 12.1 us; the gated 4096 -> 2 x 11008 at M = 16, 1376 CTAs (more
  // than one wave either way), 34.8 -> 28.3 us.
  if (p.wn == 1 && p.wk == 8 && p.grid_x > (int64_t)skinny_ctas_per_sm(p.nt, 1, 8, gated, false, peer) * sms)
    p.wk = 4;
  // Long K at M <= 8: 128-thread CTAs with twice the K slices.  Measured on
  // B200 at M = 1: 28672 -> 8192 49.8 -> 39.0 us, 28672 -> 1024 9.8 -> 8.5 us,
  // 8192 -> 3584 9.1 -> 8.2 us; not at 11008 -> 4096 (12.0 -> 12.6 us).  The
  // exchange form takes it for narrow shards only (one GPU, world-1
  // exchange, M = 1: 28672 -> 1024 11.5 -> 10.6 us, 8192 -> 3584 10.8 ->
  // 10.5 us; 28672 -> 4096 28.6 -> 29.6 us, so not there).
  if (!gated && p.nt == 1 && p.wn == 1 && p.wk == 8 && ((K >= 16384 && !peer) || (K >= 8192 && N < 4096)))
    p.wk = 4;
  // M <= 8 on layers of at most two row blocks per SM (but more than one):
  // one 512-thread CTA of 16 k-warps per row block (two resident per SM),
  // each warp's K share in fewer batches of loads, no split of K across CTAs
  // (in place of two 256-thread CTAs in a cluster).  Measured on B200 at
  // M = 1 (CUDA graphs): 4096 -> 4096 6.2 -> 5.1 us, 11008 -> 4096
  // 12.0 -> 10.1 us; not in place of the long-K 128-thread plans above
  // (8192 -> 3584: 8.2 -> 8.4 us).
  if (!gated && !peer && p.nt == 1 && p.wn == 1 && p.wk == 8 && chunks >= 64) {
    const int64_t r16 = skinny_resident_ctas(1, 1, 16, false, true, false, 1);
    if (p.grid_x <= r16 && 2 * p.grid_x > r16) p.wk = 16;
  }
  // M = 9..16 in 128-thread CTAs: loading each chunk's activations just
  // before its MMAs costs registers (fewer CTAs fit per SM) but streams
  // faster; used while the grid still fits in one wave.  Measured on B200,
  // 4096 -> 11008 at M = 16: 18.1 -> 15.2 us; 4096 -> 14336 (896 CTAs, one
  // more than fit) would need a second wave: 26.2 us against 18.6 without.
  p.xjit = 0;
  if (p.nt == 2 && p.wn == 1 && p.wk == 4 && !gated &&
      p.grid_x <= (int64_t)skinny_ctas_per_sm(p.nt, 1, 4, false, true, peer) * sms)
    p.xjit = 1;
#ifdef RLA_EXPERIMENTS
  {
    const int ewk = exp_int("RLA_EXP_WK", 0);
    if (p.wn == 1 && (ewk == 4 || ewk == 8)) {
      p.wk = ewk;
      if (ewk == 8) p.xjit = 0;
    }
  }
#endif
  p.splits = 1;
  p.cluster = 0;
  // Split K only as far as the whole grid stays resident at once (one wave):
  // measured on B200, a second wave costs more than the extra parallelism
  // gains (e.g. 4096 x 4096 at M = 16: 7.7 us unsplit vs 10.9 us with two
  // slices at two resident CTAs per SM; at M = 1, four per SM, two slices win).
  const int64_t resident = skinny_resident_ctas(p.nt, p.wn, p.wk, gated, p.xjit != 0, peer, 1);
  if (p.grid_x < resident) {
    // Each CTA slice should still give every k-warp a few chunks.
    const int64_t max_splits = chunks / (2 * p.wk);
    int64_t s = resident / p.grid_x;
    if (s > max_splits) s = max_splits;
    if (s > 32) s = 32;
#ifdef RLA_EXPERIMENTS
    {
      const int ems = exp_int("RLA_EXP_MAXSPLIT", 0);
      if (ems > 0 && s > ems) s = ems;
    }
#endif
    if (s > 1) {
      if (s <= kMaxClusterSplits || !have_ws || p.grid_x > kMaxSplitRowBlocks) {
        // the slices of a row block are one thread-block cluster and add up
        // through distributed shared memory: no workspace, no global round trip
        s = s < kMaxClusterSplits ? s : kMaxClusterSplits;
        // The whole grid must still fit at once counted in whole clusters
        // (all CTAs of a cluster sit in one GPC), which can be fewer CTAs
        // than the per-SM count suggests.
        while (s > 1 && p.grid_x * s > (int64_t)skinny_resident_ctas(p.nt, p.wn, p.wk, gated, p.xjit != 0, peer,
                                                                     static_cast<int>(s)))
          --s;
        if (s > 1) {
          p.splits = static_cast<int>(s);
          p.cluster = 1;
        }
      } else {
        p.splits = static_cast<int>(s);  // fp32 partial sums in the workspace
      }
    }
  }
  p.grid_y = p.splits;
  p.threads = 32 * p.wn * p.wk;
  p.smem = 0;
  if (p.splits > 1 && !p.cluster) p.workspace = kSplitCounterBytes + (size_t)p.splits * (size_t)M * (size_t)N * 4;
}

static std::atomic<int> g_decode_kernel{RLA_KERNEL_NONE};

// Persistent stream-K decode kernel: one CTA per SM (fewer if the problem has
// fewer 128-row x 128-k units), each streaming an equal share of the weight
// bytes.  Needs the workspace for the pieces of row blocks split between CTAs.
static void stream_shape(Plan& p, int64_t M, int64_t N, int64_t K, int sms) {
  p.kernel = RLA_KERNEL_STREAM;
  p.nt = M <= 8 ? 1 : M <= 16 ? 2 : 4;
  const int64_t units = ((N + 127) / 128) * ((K + 127) / 128);
  p.grid_x = static_cast<int>(units < sms ? units : sms);
  p.grid_y = 1;
  p.splits = 1;
  p.threads = 288;
  p.smem = stream_smem_bytes(p.nt);
  p.workspace = stream_workspace_bytes(M, p.grid_x);
}

static Plan make_plan_uncached(int64_t M, int64_t N, int64_t K, bool aligned, bool have_workspace, bool peer);

// The plan depends only on the shape, the flags, the device (its SM count and
// occupancy) and the forced decode kernel.  A model calls a few shapes over
// and over, each twice in a row (workspace size, then the launch), so each
// host thread keeps its recent plans in a small direct-mapped cache.
Plan make_plan(int64_t M, int64_t N, int64_t K, bool aligned, bool have_workspace, bool peer) {
  struct Entry {
    int64_t M = -1, N = -1, K = -1;
    int dev = -1, flags = -1, choice = -1;
    Plan plan;
  };
  constexpr int kEntries = 32;
  thread_local Entry cache[kEntries];
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  const int flags = (aligned ? 1 : 0) | (have_workspace ? 2 : 0) | (peer ? 4 : 0);
  const int choice = g_decode_kernel.load(std::memory_order_relaxed);
  const uint64_t h = (static_cast<uint64_t>(M) * 0x9E3779B97F4A7C15ull) ^ (static_cast<uint64_t>(N) * 0xC2B2AE3D27D4EB4Full) ^
                     (static_cast<uint64_t>(K) * 0x165667B19E3779F9ull) ^ static_cast<uint64_t>(flags * 7 + dev * 131);
  Entry& e = cache[(h >> 32) % kEntries];
#ifndef RLA_EXPERIMENTS  // (experiment builds read plan overrides from the environment on every call)
  if (dev >= 0 && e.M == M && e.N == N && e.K == K && e.dev == dev && e.flags == flags && e.choice == choice)
    return e.plan;
#endif
  const Plan p = make_plan_uncached(M, N, K, aligned, have_workspace, peer);
  if (dev >= 0) {
    e.M = M;
    e.N = N;
    e.K = K;
    e.dev = dev;
    e.flags = flags;
    e.choice = choice;
    e.plan = p;
  }
  return p;
}

static Plan make_plan_uncached(int64_t M, int64_t N, int64_t K, bool aligned, bool have_workspace, bool peer) {
  Plan p;
  if (M == 0 || N == 0) return p;
  if (K == 0) {
    p.kernel = RLA_KERNEL_FILL;
    return p;
  }
  const int sms = device_sm_count();
  if (aligned && K % 16 == 0 && M <= 32) {
    const int choice = g_decode_kernel.load(std::memory_order_relaxed);
    Plan sk;
    skinny_shape(sk, M, N, K, have_workspace, sms, false, peer);
    // Measured on B200 (CUDA graphs of back-to-back launches): from M = 9 on,
    // the persistent stream-K kernel wins on weights of 120 MB or more, and on
    // weights of 40 MB or more when the skinny grid needs more than one wave
    // of resident CTAs.  The skinny kernel wins on smaller layers, on narrow
    // column shards (lower fixed cost per launch) and, for M <= 8, on large
    // layers too.
    const double wbytes = static_cast<double>(N) * static_cast<double>(K);
    const bool multi_wave =
        sk.grid_x > (int64_t)skinny_ctas_per_sm(sk.nt, sk.wn, sk.wk, false, sk.xjit != 0, peer) * sms;
    // With the fused peer exchange the skinny kernel's exchange form holds
    // many more registers and loses more (one GPU, world-1 exchange, M = 16:
    // 8192 -> 14336 skinny 75.9 us vs stream 36.4; 28672 -> 4096 60.8 vs 37.8;
    // 8192 -> 3584 18.8 vs 18.5; M = 1: 8192 -> 14336 38.2 vs 30.5,
    // 28672 -> 4096 29.4 vs 31.4), while the stream kernel's exchange costs
    // about 2 us over its plain launch.
    // For M <= 8 the skinny kernel now wins on large layers too (M = 1:
    // 8192 -> 28672 skinny 40.9 us vs stream 45.2; 28672 -> 8192 39.0 vs
    // 45.3); at M = 16 the stream kernel keeps them (55.9 vs 64.9 us).
    // Its exchange form (56-64 registers at M <= 8 since the unpacking uses
    // 32-bit index arithmetic) also wins there: two ranks, the config-4
    // shards of 117 MB, M = 1: 30.2 vs 31.5 us (8192 -> 14336) and 31.2 vs
    // 33.0 us (28672 -> 4096); M = 8: 31.3 vs 32.4 and 31.8 vs 33.5 us.
    // At M = 9..16 the skinny exchange form (no grid-wide wait when its grid
    // is resident) wins on shards that fit one wave up to ~100 MB (one GPU,
    // world-1 exchange, M = 16: 8192 -> 3584 skinny 15.6 us vs stream 18.5;
    // 28672 -> 1024 16.1 vs 25.6), the stream form from 100 MB (two ranks,
    // M = 16: 28672 -> 4096 50.4 vs 39.6 us; 8192 -> 14336 68.2 vs 39.1).
    const bool stream_wins =
        M <= 16 && M > 8 &&
        (peer ? (wbytes >= 100e6 || (wbytes >= 40e6 && multi_wave))
              : ((wbytes >= 40e6 && multi_wave) || wbytes >= 120e6));
    const bool want_stream = choice == RLA_KERNEL_STREAM || (choice == RLA_KERNEL_NONE && stream_wins);
    // The stream kernel keeps one arrival counter per CTA in the counter region.
    if (have_workspace && want_stream && sms <= kMaxSplitRowBlocks) {
      stream_shape(p, M, N, K, sms);
      return p;
    }
    return sk;
  }
  if (aligned && M > 32) {
    p.kernel = RLA_KERNEL_TCGEN05;
    const int64_t ntiles = (N + 127) / 128;
    // Tile height by whole waves of tiles (one CTA per SM): 256-row tiles
    // unless 128-row tiles finish in less time.  A 128-row tile does half the
    // work of a 256-row one but takes 0.85-1.15 of its time (B200, measured
    // over the Llama-70B shards at M = 512-4096: e.g. 28672 -> 1024 one wave
    // of 128-row tiles 187 us, of 256-row tiles 207 us; 8192 -> 14336 at
    // M = 768 five waves of 128-row tiles 282 us, while M = 1024 in four
    // waves of 256-row tiles took 247 us), so 128 pays only with fewer waves.
    auto wave_cost = [&](int64_t bm, double rel) {
      const int64_t tiles = ntiles * ((M + bm - 1) / bm);
      return static_cast<double>((tiles + sms - 1) / sms) * static_cast<double>(bm) * rel;
    };
    if (M > 128 && wave_cost(256, 1.0) <= wave_cost(128, 1.9)) {
      p.bm = 256; p.stages = 4;
    } else if (M > 64) {
      p.bm = 128; p.stages = 6;
    } else {
      p.bm = 64; p.stages = 8;
    }
    p.grid_x = static_cast<int>(ntiles);
    p.grid_y = static_cast<int>((M + p.bm - 1) / p.bm);
    p.threads = 320;
    p.smem = tcgen05_smem_bytes(p.bm, p.stages);
    return p;
  }
  p.kernel = RLA_KERNEL_GENERIC;
  return p;
}

// The gated (SwiGLU) GEMM: gate and up of N outputs are 2N weight rows.
// Decode: one skinny kernel with the SwiGLU epilogue (its shape for 2N rows;
// never the stream kernel).  Prefill: two tcgen05 GEMMs write fp16 gate and
// up into the workspace and a streaming pass applies SwiGLU -- measured
// faster than a SwiGLU epilogue in the tcgen05 kernel, whose four epilogue
// warps cannot hide the exp / reciprocal latency.  Ragged shapes: generic.
size_t gated_prefill_half_bytes(int64_t M, int64_t N) { return ((size_t)M * (size_t)N * 2 + 255) & ~size_t(255); }

Plan make_plan_gated(int64_t M, int64_t N, int64_t K, bool aligned, bool have_workspace) {
  Plan p;
  if (M == 0 || N == 0) return p;
  if (K == 0 || !aligned || K % 16 != 0) {
    p.kernel = RLA_KERNEL_GENERIC;
    return p;
  }
  if (M <= 32) {
    skinny_shape(p, M, 2 * N, K, have_workspace, device_sm_count(), /*gated=*/true);
    return p;
  }
  p = make_plan(M, N, K, aligned, false);  // the tcgen05 plan of one projection
  // The split-K counter region stays first (other calls on the same
  // workspace rely on it being zero); gate and up follow it.
  p.workspace = kSplitCounterBytes + 2 * gated_prefill_half_bytes(M, N);
  return p;
}

}  // namespace rla

using namespace rla;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int fail(int code, const char* msg) {
  set_error("%s", msg);
  return code;
}

extern "C" {

int rla_version(void) { return 1 * 10000 + 0 * 100 + 0; }

int rla_set_decode_kernel(int kernel) {
  if (kernel != RLA_KERNEL_NONE && kernel != RLA_KERNEL_SKINNY && kernel != RLA_KERNEL_STREAM)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_set_decode_kernel: expected NONE, SKINNY or STREAM");
  g_decode_kernel.store(kernel, std::memory_order_relaxed);
  return RLA_OK;
}

const char* rla_last_error(void) { return g_err; }

uint64_t rla_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int rla_get_device_error(unsigned int* code) {
  if (!code) return fail(RLA_ERR_INVALID_ARGUMENT, "code is NULL");
  unsigned int zero = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(code, rla_device_error, sizeof(unsigned int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(rla_device_error, &zero, sizeof(unsigned int));
  if (e != cudaSuccess) {
    set_error("rla_get_device_error: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  return RLA_OK;
}

size_t rla_w8a16_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return 0;
  return make_plan(M, N, K, true, true).workspace;
}

int rla_w8a16_plan(int64_t M, int64_t N, int64_t K, int aligned, int have_workspace, int64_t* params) {
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_plan: sizes must be in [0, 2^31)");
  const Plan p = make_plan(M, N, K, aligned != 0, have_workspace != 0);
  if (params) {
    params[0] = p.kernel;
    params[1] = p.grid_x;
    params[2] = p.grid_y;
    params[3] = p.threads;
    params[4] = p.splits;
    params[5] = p.kernel == RLA_KERNEL_SKINNY ? 16 * p.wn
                : (p.kernel == RLA_KERNEL_STREAM || p.kernel == RLA_KERNEL_TCGEN05) ? 128 : 0;
    params[6] = (p.kernel == RLA_KERNEL_SKINNY || p.kernel == RLA_KERNEL_STREAM) ? 8 * p.nt : p.bm;
    params[7] = static_cast<int64_t>(p.smem);
  }
  return RLA_OK;
}

int rla_w8a16_gemm(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale, int scale_dtype,
                   const void* bias, int bias_dtype, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                   void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm: M, N, K must be in [0, 2^31)");
  if (M == 0 || N == 0) return RLA_OK;
  if (scale_dtype != RLA_DTYPE_F16 && scale_dtype != RLA_DTYPE_F32)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm: scale_dtype must be F16 or F32");
  if (bias_dtype != RLA_DTYPE_NONE && bias_dtype != RLA_DTYPE_F16 && bias_dtype != RLA_DTYPE_F32)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm: bias_dtype must be NONE, F16 or F32");
  if (bias_dtype != RLA_DTYPE_NONE && !bias)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm: bias is NULL but bias_dtype is set");
  if (!y || !scale || (K > 0 && (!x || !w)))
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm: null x, w, scale or y");
  if (ldy < N || (K > 0 && (ldx < K || ldw < K)))
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm: leading dimensions must be >= the row length");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(RLA_ERR_WORKSPACE, "rla_w8a16_gemm: workspace must be 256-byte aligned");

  GemmArgs a{x, ldx, w, ldw, scale, scale_dtype == RLA_DTYPE_F32 ? 1 : 0, bias,
             bias_dtype == RLA_DTYPE_NONE ? 0 : bias_dtype == RLA_DTYPE_F16 ? 1 : 2,
             y, ldy, (int)M, (int)N, (int)K};
  const bool aligned = aligned16(x) && aligned16(w) && (ldx % 8 == 0) && (ldw % 16 == 0);
  Plan p = make_plan(M, N, K, aligned, workspace != nullptr && workspace_bytes > 0);
  if (p.workspace > workspace_bytes) p = make_plan(M, N, K, aligned, false);  // too small: no split-K

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  switch (p.kernel) {
    case RLA_KERNEL_SKINNY: e = launch_skinny(a, p, workspace, s); break;
    case RLA_KERNEL_STREAM: e = launch_stream(a, p, workspace, s); break;
    case RLA_KERNEL_TCGEN05: e = launch_tcgen05(a, p, s); break;
    case RLA_KERNEL_GENERIC: e = launch_generic(a, s); break;
    case RLA_KERNEL_FILL: e = launch_fill(a, s); break;
    default: return RLA_OK;
  }
  if (e != cudaSuccess) {
    set_error("rla_w8a16_gemm: launch of kernel family %d failed: %s", p.kernel, cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

int rla_quantize_per_channel(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int8_t* q,
                             int64_t ldq, float* scale, void* stream) {
  if (N < 0 || K < 0 || N > INT32_MAX || K > INT32_MAX)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_quantize_per_channel: sizes must be in [0, 2^31)");
  if (N == 0) return RLA_OK;
  if (!w || !q || !scale) return fail(RLA_ERR_INVALID_ARGUMENT, "rla_quantize_per_channel: null pointer");
  if (w_dtype != RLA_DTYPE_F32 && w_dtype != RLA_DTYPE_F16 && w_dtype != RLA_DTYPE_BF16)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_quantize_per_channel: w_dtype must be F32, F16 or BF16");
  if (ldw < K || ldq < K) return fail(RLA_ERR_INVALID_ARGUMENT, "rla_quantize_per_channel: bad leading dimension");
  cudaError_t e = launch_quantize(w, w_dtype, ldw, N, K, q, ldq, scale, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("rla_quantize_per_channel: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

size_t rla_w8a16_swiglu_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M < 0 || N < 0 || K < 0) return 0;
  return make_plan_gated(M, N, K, true, true).workspace;
}

int rla_w8a16_gemm_swiglu(const void* x, int64_t ldx, const int8_t* w_gate, const int8_t* w_up, int64_t ldw,
                          const void* scale_gate, const void* scale_up, int scale_dtype, const void* bias_gate,
                          const void* bias_up, int bias_dtype, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm_swiglu: M, N, K must be in [0, 2^31)");
  if (M == 0 || N == 0) return RLA_OK;
  if (scale_dtype != RLA_DTYPE_F16 && scale_dtype != RLA_DTYPE_F32)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm_swiglu: scale_dtype must be F16 or F32");
  if (bias_dtype != RLA_DTYPE_NONE && bias_dtype != RLA_DTYPE_F16 && bias_dtype != RLA_DTYPE_F32)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm_swiglu: bias_dtype must be NONE, F16 or F32");
  if (bias_dtype != RLA_DTYPE_NONE && (!bias_gate || !bias_up))
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm_swiglu: bias_dtype set but a bias is NULL");
  if (!y || !scale_gate || !scale_up || (K > 0 && (!x || !w_gate || !w_up)))
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm_swiglu: null x, weight, scale or y");
  if (ldy < N || (K > 0 && (ldx < K || ldw < K)))
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_w8a16_gemm_swiglu: leading dimensions must be >= the row length");
  if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return fail(RLA_ERR_WORKSPACE, "rla_w8a16_gemm_swiglu: workspace must be 256-byte aligned");
  GemmArgs a{x, ldx, w_gate, ldw, scale_gate, scale_dtype == RLA_DTYPE_F32 ? 1 : 0, bias_gate,
             bias_dtype == RLA_DTYPE_NONE ? 0 : bias_dtype == RLA_DTYPE_F16 ? 1 : 2,
             y, ldy, (int)M, (int)N, (int)K};
  a.w_up = w_up;
  a.scale_up = scale_up;
  a.bias_up = bias_up;
  const bool aligned = aligned16(x) && aligned16(w_gate) && aligned16(w_up) && (ldx % 8 == 0) && (ldw % 16 == 0);
  Plan p = make_plan_gated(M, N, K, aligned, workspace != nullptr && workspace_bytes > 0);
  if (p.kernel == RLA_KERNEL_SKINNY && p.workspace > workspace_bytes)
    p = make_plan_gated(M, N, K, aligned, false);
  if (p.kernel == RLA_KERNEL_TCGEN05 && p.workspace > workspace_bytes) {
    set_error("rla_w8a16_gemm_swiglu: M = %lld needs %zu bytes of workspace for the gate and up outputs "
              "(rla_w8a16_swiglu_workspace_size), got %zu", (long long)M, p.workspace, workspace_bytes);
    return RLA_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  switch (p.kernel) {
    case RLA_KERNEL_SKINNY: e = launch_skinny(a, p, workspace, s); break;
    case RLA_KERNEL_TCGEN05: {
      // gate and up (fp16 [M, N]) after the counter region, then SwiGLU.
      __half* gbuf = reinterpret_cast<__half*>(static_cast<char*>(workspace) + kSplitCounterBytes);
      __half* ubuf = reinterpret_cast<__half*>(static_cast<char*>(workspace) + kSplitCounterBytes +
                                               gated_prefill_half_bytes(M, N));
      GemmArgs g{x, ldx, w_gate, ldw, scale_gate, a.scale_f32, bias_gate, a.bias_kind, gbuf, N, (int)M, (int)N,
                 (int)K};
      GemmArgs u{x, ldx, w_up, ldw, scale_up, a.scale_f32, bias_up, a.bias_kind, ubuf, N, (int)M, (int)N, (int)K};
      e = launch_tcgen05(g, p, s);
      if (e == cudaSuccess) e = launch_tcgen05(u, p, s);
      if (e == cudaSuccess) e = launch_swiglu(gbuf, ubuf, N, y, ldy, (int)M, (int)N, s);
      if (e == cudaSuccess) {
        note_launch();
        note_launch();
      }
      break;
    }
    case RLA_KERNEL_GENERIC: e = launch_generic(a, s); break;
    default: return fail(RLA_ERR_UNSUPPORTED, "rla_w8a16_gemm_swiglu: no kernel for this shape");
  }
  if (e != cudaSuccess) {
    set_error("rla_w8a16_gemm_swiglu: launch of kernel family %d failed: %s", p.kernel, cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

int rla_rmsnorm(const void* x, int64_t ldx, const void* weight, int weight_dtype, float eps, void* y, int64_t ldy,
                int64_t M, int64_t K, void* stream) {
  if (M < 0 || K < 0 || M > INT32_MAX || K > INT32_MAX)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_rmsnorm: M, K must be in [0, 2^31)");
  if (M == 0 || K == 0) return RLA_OK;
  if (!x || !weight || !y) return fail(RLA_ERR_INVALID_ARGUMENT, "rla_rmsnorm: null pointer");
  if (weight_dtype != RLA_DTYPE_F32 && weight_dtype != RLA_DTYPE_F16 && weight_dtype != RLA_DTYPE_BF16)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_rmsnorm: weight_dtype must be F32, F16 or BF16");
  if (ldx < K || ldy < K) return fail(RLA_ERR_INVALID_ARGUMENT, "rla_rmsnorm: leading dimensions must be >= K");
  if (!(eps >= 0.f)) return fail(RLA_ERR_INVALID_ARGUMENT, "rla_rmsnorm: eps must be >= 0");
  const cudaError_t e = launch_rmsnorm(x, ldx, weight, weight_dtype, eps, y, ldy, (int)M, (int)K,
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("rla_rmsnorm: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

int rla_gather_columns(const void* staging, int64_t world, int64_t M, int64_t n_local, void* y, int64_t ldy,
                       void* stream) {
  if (world < 1 || M < 0 || n_local < 0 || ldy < world * n_local)
    return fail(RLA_ERR_INVALID_ARGUMENT, "rla_gather_columns: bad sizes");
  if (M == 0 || n_local == 0) return RLA_OK;
  if (!staging || !y) return fail(RLA_ERR_INVALID_ARGUMENT, "rla_gather_columns: null pointer");
  cudaError_t e = launch_gather(staging, world, M, n_local, y, ldy, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error("rla_gather_columns: %s", cudaGetErrorString(e));
    return RLA_ERR_CUDA;
  }
  note_launch();
  return RLA_OK;
}

}  // extern "C"
