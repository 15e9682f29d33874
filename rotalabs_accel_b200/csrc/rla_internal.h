// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/rla_w8a16.h"

namespace rla {

// Direct peer-to-peer output exchange of the column-parallel layer (one
// process per GPU, every rank's receive buffer IPC-mapped into every other
// rank; protocol in rla_peer.cuh).  world == 0: no exchange.
constexpr int kMaxPeers = 8;
// Sync area of one rank (local, never mapped by peers): 32-bit words.
constexpr int kSyncSeq = 0;        // exchange calls this rank has completed
constexpr int kSyncArrive = 32;    // CTAs of the running call that finished phase 1
constexpr int kSyncUnpacked = 64;  // unpacking CTAs of the running call that are done
constexpr int kSyncAbort = 96;     // call number whose wait gave up (stops the other waits; never cleared)
constexpr size_t kSyncBytes = 512;
static_assert(kSyncAbort == RLA_PEER_SYNC_ABORT_WORD && kSyncBytes == RLA_PEER_SYNC_BYTES, "sync area layout");

struct PeerOut {
  uint2* recv[kMaxPeers];       // rank d's receive buffer: 2 halves (call parity) of flagged words
  unsigned int* sync;           // this rank's sync area
  int64_t half_words;           // flagged words per parity half
  int64_t slot_words;           // words of one source rank's slice in this call: ceil(M/2) * n_local
  unsigned long long wait_ns;   // limit of every wait
  unsigned int unpackers;       // R: CTAs that unpack peer slices (1 <= R <= CTAs of the launch)
  int world;
  int rank;
};

// Arguments common to every W8A16 GEMM kernel.
struct GemmArgs {
  const void* x;
  int64_t ldx;
  const int8_t* w;
  int64_t ldw;
  const void* scale;
  int scale_f32;  // 1: fp32 scale, 0: fp16 scale
  const void* bias;
  int bias_kind;  // 0 none, 1 fp16, 2 fp32
  void* y;
  int64_t ldy;
  int M, N, K;
  // world == 0 unless the call is rla_w8a16_gemm_allgather; then y is the
  // full [M, world * n_local] output and N = n_local.
  PeerOut peer{};
  // Gated (SwiGLU) GEMM, rla_w8a16_gemm_swiglu, decode and generic kernels:
  // w / scale / bias are the gate projection, these the up projection (same
  // layout), and y = fp16(silu(gate) * up) with gate and up rounded to fp16
  // first.
  const int8_t* w_up = nullptr;
  const void* scale_up = nullptr;
  const void* bias_up = nullptr;
};

// A launch plan chosen by the per-shape selector.
struct Plan {
  int kernel = RLA_KERNEL_NONE;
  // skinny kernel
  int nt = 0;      // 8-row tiles of x per MMA column block (M <= 8 * nt)
  int wn = 0;      // 16-row groups of w per CTA
  int wk = 0;      // k-slicing warps per CTA
  int splits = 1;  // CTAs along K (split-K across CTAs when > 1)
  int cluster = 0; // split-K inside a thread-block cluster of `splits` CTAs (no workspace)
  int xjit = 0;    // NT = 2, (1, 4): activation loads just before the MMAs
  // tcgen05 kernel
  int bm = 0;      // rows of x per tile (MMA N)
  int stages = 0;  // TMA pipeline depth
  // common
  int grid_x = 0, grid_y = 0, threads = 0;
  size_t smem = 0;
  size_t workspace = 0;
};

// Split-K workspace layout (fixed, so calls with different shapes can share
// one workspace): [0, kSplitCounterBytes) arrival counters, one per row
// block, zero between calls; then the fp32 partial sums [splits][M][N].
constexpr size_t kSplitCounterBytes = 4096;
constexpr int kMaxSplitRowBlocks = static_cast<int>(kSplitCounterBytes / sizeof(unsigned int));
// Largest split-K done inside one thread-block cluster (the portable cluster size).
constexpr int kMaxClusterSplits = 8;

// peer: plan for the launch with the fused peer exchange (its own occupancy)
Plan make_plan(int64_t M, int64_t N, int64_t K, bool aligned, bool have_workspace, bool peer = false);

void note_launch();
int device_sm_count();  // SMs of the current device (148 if it cannot be read)
void set_error(const char* fmt, ...);

cudaError_t launch_skinny(const GemmArgs& a, const Plan& p, void* workspace, cudaStream_t s);
// Resident CTAs per SM of the skinny kernel instance (plain or gated form);
// 2 when the device cannot be queried.
int skinny_ctas_per_sm(int nt, int wn, int wk, bool gated, bool xjit = false, bool peer = false);
// CTAs of the skinny kernel instance that fit on the device at once, with the
// K slices of a row block in clusters of `cluster` CTAs (whole clusters
// counted); 2 per SM when the device cannot be queried.
int skinny_resident_ctas(int nt, int wn, int wk, bool gated, bool xjit, bool peer, int cluster);
cudaError_t launch_stream(const GemmArgs& a, const Plan& p, void* workspace, cudaStream_t s);
size_t stream_workspace_bytes(int64_t M, int ctas);
size_t stream_smem_bytes(int nt);
cudaError_t launch_tcgen05(const GemmArgs& a, const Plan& p, cudaStream_t s);
cudaError_t launch_generic(const GemmArgs& a, cudaStream_t s);  // also the gated form (a.w_up set)
cudaError_t launch_swiglu(const void* gate, const void* up, int64_t ld, void* y, int64_t ldy, int M, int N,
                          cudaStream_t s);
cudaError_t launch_rmsnorm(const void* x, int64_t ldx, const void* weight, int weight_dtype, float eps, void* y,
                           int64_t ldy, int M, int K, cudaStream_t s);
cudaError_t launch_fill(const GemmArgs& a, cudaStream_t s);

size_t tcgen05_smem_bytes(int bm, int stages);
int tcgen05_tmem_cols(int bm);

}  // namespace rla
