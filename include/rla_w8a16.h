/*
 * rla_w8a16.h -- C ABI of the B200 (sm_100a) W8A16 GEMM library.
 *
 * W8A16: fp16 activations x int8 weights with one symmetric scale per output
 * channel, fp32 accumulation, fp16 output:
 *
 *     y[m, n] = fp16( scale[n] * sum_k x[m, k] * w[n, k]  (+ bias[n]) )
 *
 * Plain pointers and sizes only (no framework types).  Device pointers are
 * CUDA device addresses on the current device; `stream` is a cudaStream_t
 * (NULL = legacy default stream).  Every entry point returns an rla_status;
 * nothing throws across this boundary.  rla_last_error() gives a message for
 * the last failure on the calling thread.
 *
 * Each entry point names the rotalabs-accel interface it replaces
 * (paths inside the rotalabs-accel project).
 */
#ifndef RLA_W8A16_H
#define RLA_W8A16_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RLA_API __attribute__((visibility("default")))
#else
#define RLA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum rla_status {
  RLA_OK = 0,
  RLA_ERR_INVALID_ARGUMENT = 1, /* bad size, stride, dtype or null pointer      */
  RLA_ERR_UNSUPPORTED = 2,      /* valid request this build cannot run          */
  RLA_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed         */
  RLA_ERR_WORKSPACE = 4,        /* workspace missing, too small or misaligned   */
  RLA_ERR_DEVICE = 5            /* no device, or not an sm_100 device           */
} rla_status;

typedef enum rla_dtype {
  RLA_DTYPE_NONE = 0, /* "no tensor" (e.g. no bias) */
  RLA_DTYPE_F16 = 1,
  RLA_DTYPE_F32 = 2,
  RLA_DTYPE_BF16 = 3
} rla_dtype;

/* Kernel families the per-shape selector can pick. */
typedef enum rla_kernel {
  RLA_KERNEL_NONE = 0,     /* nothing to compute (M == 0 or N == 0)              */
  RLA_KERNEL_SKINNY = 1,   /* HBM-streaming split-K kernel, M <= 32 (decode)     */
  RLA_KERNEL_TCGEN05 = 2,  /* TMA + int8->fp16 into TMEM + tcgen05.mma (prefill) */
  RLA_KERNEL_GENERIC = 3,  /* any alignment / any K (ragged shapes)              */
  RLA_KERNEL_FILL = 4,     /* K == 0: y = bias (or 0)                            */
  RLA_KERNEL_STREAM = 5    /* persistent stream-K TMA decode kernel, M <= 32     */
} rla_kernel;

/*
 * Process-wide choice of the decode (M <= 32) kernel family:
 * RLA_KERNEL_NONE (0, the default) lets the selector choose; RLA_KERNEL_SKINNY
 * or RLA_KERNEL_STREAM force that kernel where it applies.  For A/B
 * measurements and tests; not synchronised with GEMM calls running
 * concurrently on other threads.  Part of the per-shape selector that
 * replaces the Triton autotuner (src/rotalabs_accel/kernels/gemm.py:53-65).
 */
RLA_API int rla_set_decode_kernel(int kernel);

/*
 * W8A16 GEMM on device buffers.
 *
 * Replaces rotalabs-accel's GPU launch of the Triton kernel
 * (src/rotalabs_accel/kernels/gemm.py:140-186, `_int8_gemm_triton` ->
 * `_int8_gemm_kernel[grid](...)` at :169-178, with the separate bias add at
 * :180-182) behind the dispatcher `int8_gemm` (gemm.py:189-238).
 *
 *   x      fp16 [M, K], row stride ldx elements (ldx >= K)
 *   w      int8 [N, K], row stride ldw bytes    (ldw >= K), K contiguous
 *          (the reference's `weight_int8` layout; no transposed copy is used)
 *   scale  [N], scale_dtype RLA_DTYPE_F32 (Int8Linear) or RLA_DTYPE_F16
 *   bias   [N] or NULL; bias_dtype RLA_DTYPE_NONE / F16 / F32
 *   y      fp16 [M, N], row stride ldy elements (ldy >= N)
 *   workspace / workspace_bytes: caller-owned device scratch for split-K /
 *          stream-K partial sums, at least rla_w8a16_workspace_size(M, N, K) bytes,
 *          256-byte aligned.  Layout: the first 4096 bytes hold arrival
 *          counters that must be zero before the first call (the library
 *          leaves them at zero after every call, so one workspace serves
 *          calls of any shape); fp32 partial sums follow.  May be NULL / 0:
 *          the selector then plans split-K only inside thread-block
 *          clusters (up to 8 slices, added through distributed shared
 *          memory, which needs no workspace).  Calls that share a workspace
 *          must be stream-ordered.
 *   stream cudaStream_t to launch on.
 *
 * Returns RLA_OK, or an error with nothing launched.
 */
RLA_API int rla_w8a16_gemm(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                   int scale_dtype, const void* bias, int bias_dtype, void* y, int64_t ldy, int64_t M,
                   int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace the selector's plan for (M, N, K) can use (0 if none:
 * no split-K, or split-K inside thread-block clusters).
 * Part of the same replacement as rla_w8a16_gemm (gemm.py:140-186). */
RLA_API size_t rla_w8a16_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * The per-shape kernel selector (replaces the Triton autotuner keyed on
 * (M, N, K), src/rotalabs_accel/kernels/gemm.py:53-65).  Describes the plan
 * rla_w8a16_gemm would run for this call without launching anything:
 * kernel family (rla_kernel) and its launch parameters.  `aligned` = 1 when
 * x, w are 16-byte aligned, ldx % 8 == 0 and ldw % 16 == 0.  `params`
 * (may be NULL) receives up to 8 integers: [0] kernel, [1] grid.x,
 * [2] grid.y, [3] threads per CTA, [4] split-K slices, [5] tile rows of w,
 * [6] tile rows of x, [7] dynamic shared memory bytes.
 */
RLA_API int rla_w8a16_plan(int64_t M, int64_t N, int64_t K, int aligned, int have_workspace, int64_t* params);

/*
 * Per-output-channel symmetric int8 quantization on the device.
 *
 * Replaces quantize_weight_per_channel
 * (src/rotalabs_accel/quantization/symmetric.py:126-151 ->
 * quantize_symmetric(dim=1), :24-82), bit-identical to it: per row,
 * scale = max|w| / 127 computed in the input dtype, 0 -> 1, then
 * q = round_half_even(w / scale) (quotient rounded to the input dtype first,
 * as torch does) clamped to [-128, 127]; scale is returned as fp32.
 *
 *   w      [N, K] of w_dtype (F32, F16 or BF16), row stride ldw elements
 *   q      int8 [N, K], row stride ldq bytes
 *   scale  fp32 [N]
 */
RLA_API int rla_quantize_per_channel(const void* w, int w_dtype, int64_t ldw, int64_t N, int64_t K, int8_t* q,
                             int64_t ldq, float* scale, void* stream);

/*
 * Column-parallel assembly: the all-gathered staging buffer
 * staging[world][M][n_local] (fp16, contiguous; what ncclAllGather of each
 * rank's [M, n_local] output slice produces) is rearranged into
 * y[M][world * n_local] (row stride ldy).  No counterpart in rotalabs-accel,
 * which has no distributed code; it is the output step of the column-parallel
 * sharded Int8Linear (each rank holds rows [r*n_local, (r+1)*n_local) of
 * weight_int8 / scale, src/rotalabs_accel/kernels/gemm.py:268-279).
 */
RLA_API int rla_gather_columns(const void* staging, int64_t world, int64_t M, int64_t n_local, void* y, int64_t ldy,
                       void* stream);

/*
 * Allocation-free W8A16 GEMM for the decode regime.  No counterpart in
 * rotalabs-accel: it exists for callers that cannot allocate GPU memory
 * where the GEMM runs -- a serving loop that must not let cudaMalloc
 * synchronise the device between decode steps, a process whose memory is
 * reserved up front (KV cache, custom pool), or a plugin/enqueue callback
 * that gets no workspace.  Same arguments and result as rla_w8a16_gemm
 * without the workspace: the split-K scratch is a file-scope device array of
 * 1 MiB per GPU (held by every GPU that loads the library until exit).
 * Limits: 1 <= M <= 32, K % 16 == 0, 16-byte aligned x and w, ldx % 8 == 0,
 * ldw % 16 == 0 (else RLA_ERR_UNSUPPORTED); a shape whose split-K plan needs
 * more than 1 MiB is rejected with RLA_ERR_WORKSPACE.  Nothing is launched
 * on an error.  The first call on a device sets that device up (looks up the
 * array's address, zeroes its counters on `stream`): make it before any
 * stream capture.  All calls share the array: calls that overlap on the GPU
 * race and must be ordered by the caller.  Never calls cudaMalloc/cudaFree.
 */
RLA_API int rla_w8a16_gemm_noalloc(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                                   int scale_dtype, const void* bias, int bias_dtype, void* y, int64_t ldy,
                                   int64_t M, int64_t N, int64_t K, void* stream);

/*
 * Column-parallel W8A16 GEMM with a direct peer-to-peer all-gather epilogue
 * (one process per GPU on one node).  No counterpart in rotalabs-accel, which
 * has no distributed code: it is the fused form of the sharded Int8Linear's
 * "local GEMM + ncclAllGather + reorder" (rank r holds rows
 * [r * n_local, (r + 1) * n_local) of weight_int8 / scale / bias,
 * src/rotalabs_accel/kernels/gemm.py:268-279 split by output channel).
 *
 * Rank `rank` of `world` (1 <= world <= RLA_MAX_PEERS) computes its slice
 *     y[m, rank * n_local + j] = fp16( scale[j] * sum_k x[m, k] * w[j, k] (+ bias[j]) ),
 *     0 <= j < n_local,
 * into its own y and, as 8-byte flagged words {two fp16 values, call number},
 * into the receive buffer of every peer over NVLink; the last CTAs of the
 * launch then unpack every peer's slice from this rank's receive buffer into
 * y.  When the kernel has completed, y[M, world * n_local] (row stride ldy)
 * holds all slices: no gather, no reorder, no host synchronisation.
 *
 *   x, ldx, w (int8 [n_local, K], row stride ldw), scale, bias, workspace:
 *          as in rla_w8a16_gemm, with N = n_local; size the workspace with
 *          rla_w8a16_allgather_workspace_size (this launch is planned for
 *          the exchange kernel, which can differ from rla_w8a16_gemm's plan).
 *   y      this rank's fp16 output [M, ldy], ldy >= world * n_local (any
 *          device memory; not shared with the peers).
 *   recv_peers  HOST array of `world` device pointers, valid in this process,
 *          to every rank's receive buffer (recv_peers[rank] is this rank's;
 *          the peers' mapped with rla_ipc_open), each recv_bytes bytes from
 *          rla_peer_alloc (zeroed, 16-byte aligned).  Needs
 *          recv_bytes >= 16 * world * ceil(M / 2) * n_local, else
 *          RLA_ERR_WORKSPACE.
 *   sync   this rank's sync area, RLA_PEER_SYNC_BYTES of zeroed device memory
 *          (128-byte aligned), used by no other exchange.
 *
 * Every rank must make the same sequence of calls with the same shapes,
 * stream-ordered on each rank (as with the collectives of one communicator).
 * Decode shapes only (1 <= M <= 32, K % 16 == 0, 16-byte aligned x and w,
 * ldx % 8 == 0, ldw % 16 == 0): otherwise RLA_ERR_UNSUPPORTED with nothing
 * launched, and the caller uses its collective path.  Waits are bounded
 * (rla_set_peer_wait_limit); a wait that gives up records device error 7 (a
 * peer's slice did not arrive) or 8 (this launch's CTAs did not all finish)
 * and leaves y incomplete.  The sync area then stays marked: every later call
 * on it records device error 9 and returns at once with y incomplete (no
 * second wait of the full limit).  After device error 7, 8 or 9, every rank
 * frees and re-creates its buffers and sync area (receive buffers may still
 * hold words of the failed call).  Stores to peers are plain stores over
 * NVLink (no multicast).
 */
#define RLA_MAX_PEERS 8
#define RLA_PEER_SYNC_BYTES 512
/* Index (in 32-bit words) of the sync area's abort word: non-zero once a wait
 * of an exchange call on that sync area has given up (a host may read it). */
#define RLA_PEER_SYNC_ABORT_WORD 96
#define RLA_IPC_HANDLE_BYTES 64
RLA_API int rla_w8a16_gemm_allgather(const void* x, int64_t ldx, const int8_t* w, int64_t ldw, const void* scale,
                                     int scale_dtype, const void* bias, int bias_dtype, void* y, int64_t ldy,
                                     int64_t M, int64_t n_local, int64_t K, void* const* recv_peers,
                                     size_t recv_bytes, void* sync, int rank, int world, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* Bytes of workspace the plan of rla_w8a16_gemm_allgather for (M, n_local, K)
 * can use (0 if none).  Part of the same replacement as that entry point. */
RLA_API size_t rla_w8a16_allgather_workspace_size(int64_t M, int64_t n_local, int64_t K);

/* Limit of every wait inside rla_w8a16_gemm_allgather, in nanoseconds
 * (default 1 s; 1 ms .. 60 s).  Process-wide. */
RLA_API int rla_set_peer_wait_limit(uint64_t ns);

/*
 * Device memory for the peer exchange: rla_peer_alloc returns `bytes` of
 * zeroed device memory on the current device (its own cudaMalloc, so the IPC
 * handle covers exactly this buffer); rla_peer_free releases it.
 * rla_ipc_export writes the RLA_IPC_HANDLE_BYTES-byte IPC handle of such a
 * buffer into `handle` (host memory); another process on the same node opens
 * it with rla_ipc_open (peer access enabled lazily) and closes it with
 * rla_ipc_close.  These replace nothing in rotalabs-accel; they are the
 * set-up of rla_w8a16_gemm_allgather.
 */
RLA_API int rla_peer_alloc(size_t bytes, void** ptr);
RLA_API int rla_peer_free(void* ptr);
RLA_API int rla_ipc_export(const void* ptr, void* handle);
RLA_API int rla_ipc_open(const void* handle, void** ptr);
RLA_API int rla_ipc_close(void* ptr);

/*
 * Pull exchange of the column-parallel prefill: the output step of a sharded
 * Int8Linear (src/rotalabs_accel/kernels/gemm.py:241-336 with its output
 * channels split over the ranks; rotalabs-accel itself has no distributed
 * code) for long activation blocks, overlapped with the GEMM block by block.
 * Rank r owns output columns [r * n_local, (r + 1) * n_local).
 *
 * Per rank, set up once (collectively): an exchange buffer xb of
 * max_rows * ld_xb fp16 and a sync area of RLA_PX_SYNC_BYTES, both from
 * rla_peer_alloc (zeroed), both IPC-mapped into every other rank.  One call:
 *
 *   rla_prefill_exchange_begin(sync_peers, rank, world, stream)
 *       advances the call number and waits until every peer finished reading
 *       this rank's xb in the previous call (so the GEMMs may overwrite it);
 *   then for each block b = 0, 1, ... of rows [row0, row0 + rows):
 *     rla_w8a16_gemm(... , y = xb + row0 * ld_xb, ldy = ld_xb, M = rows,
 *                    N = n_local ...)               on the compute stream;
 *     rla_prefill_exchange_block(xb_peers, ld_xb, sync_peers, rank, world,
 *                    b, last = (b is the final block), row0, rows, n_local,
 *                    y, ldy, comm_stream)           ordered after that GEMM
 *       marks block b ready in every rank's sync area, waits for every
 *       rank's mark of block b, and copies every rank's slice of those rows
 *       from its xb (over NVLink) into y[row0:row0+rows, src * n_local ...].
 *       On the last block it then tells every peer that this rank's reads of
 *       the call are over.
 *
 * xb_peers / sync_peers are HOST arrays of `world` device pointers valid in
 * this process (entry `rank` is this rank's own).  Needs n_local, ld_xb and
 * ldy multiples of 8, ld_xb >= n_local, ldy >= world * n_local, 16-byte
 * aligned xb and y, 128-byte aligned sync areas, block < RLA_PX_MAX_BLOCKS,
 * rows < 2^31 (else RLA_ERR_INVALID_ARGUMENT, nothing launched).
 * Every rank makes the same calls with the same blocks in the same order.
 * Waits are bounded (rla_set_peer_wait_limit); a wait that gives up records
 * device error 7 and marks the sync area (word RLA_PX_SYNC_ABORT_WORD); later
 * calls on it record device error 9 and return at once, y incomplete.  The
 * GEMMs themselves do not read the mark: after a failure every rank frees
 * and re-creates its buffers.  Plain loads and stores over NVLink, no
 * multicast, no copy engine.
 */
#define RLA_PX_SYNC_BYTES 1024
#define RLA_PX_MAX_BLOCKS 16
#define RLA_PX_SYNC_ABORT_WORD 1
RLA_API int rla_prefill_exchange_begin(void* const* sync_peers, int rank, int world, void* stream);
RLA_API int rla_prefill_exchange_block(const void* const* xb_peers, int64_t ld_xb, void* const* sync_peers, int rank,
                                       int world, int block, int last, int64_t row0, int64_t rows, int64_t n_local,
                                       void* y, int64_t ldy, void* stream);

/*
 * Gate and up projections of a SwiGLU MLP in one W8A16 GEMM, with the
 * activation in the epilogue:
 *
 *     y[m, n] = fp16( silu(g) * u ),  g = fp16(scale_gate[n] * sum_k x[m,k] w_gate[n,k] (+ bias_gate[n])),
 *                                     u = fp16(scale_up[n]   * sum_k x[m,k] w_up[n,k]   (+ bias_up[n])),
 *     silu(g) = g * sigmoid(g), computed in fp32.
 *
 * Replaces rotalabs-accel's `int8_gemm(x, gate) ; int8_gemm(x, up) ;
 * swiglu_fused(gate, up)` (src/rotalabs_accel/kernels/gemm.py:189-238 twice,
 * then kernels/activations.py:109-137 -> the Triton kernel at :55-80, which
 * computes silu(gate) * up in fp32 from the two fp16 outputs) with one
 * launch and no [M, N] intermediates.  w_gate and w_up are int8 [N, K] with
 * the same row stride ldw; scales [N] share scale_dtype, biases [N] share
 * bias_dtype (both NULL with RLA_DTYPE_NONE).  Workspace sized by
 * rla_w8a16_swiglu_workspace_size (same counter rules as rla_w8a16_gemm).
 * Decode (M <= 32): one launch, the skinny kernel with gate and up rows in
 * one MMA tile and the SwiGLU in its epilogue.  Prefill (M > 32): two
 * tcgen05 GEMMs write fp16 gate and up into the workspace after its
 * 4096-byte counter region (4096 + 4 * M * N bytes, rounded up; required:
 * RLA_ERR_WORKSPACE otherwise), then one SwiGLU pass.
 */
RLA_API int rla_w8a16_gemm_swiglu(const void* x, int64_t ldx, const int8_t* w_gate, const int8_t* w_up, int64_t ldw,
                                  const void* scale_gate, const void* scale_up, int scale_dtype, const void* bias_gate,
                                  const void* bias_up, int bias_dtype, void* y, int64_t ldy, int64_t M, int64_t N,
                                  int64_t K, void* workspace, size_t workspace_bytes, void* stream);
RLA_API size_t rla_w8a16_swiglu_workspace_size(int64_t M, int64_t N, int64_t K);

/*
 * RMSNorm of M fp16 rows of length K: y = fp16(x * rsqrt(mean(x^2) + eps) * w),
 * the mean and product in fp32.  Replaces rotalabs-accel's CUDA RMSNorm
 * (src/rotalabs_accel/kernels/normalization.py:186-213 -> the Triton kernel
 * at :66-101); weight [K] is F32, F16 or BF16.  The normalisation in front of
 * the gate/up GEMM of the MLP block.
 */
RLA_API int rla_rmsnorm(const void* x, int64_t ldx, const void* weight, int weight_dtype, float eps, void* y,
                        int64_t ldy, int64_t M, int64_t K, void* stream);

/* Number of kernels this library has launched in this process (all devices). */
RLA_API uint64_t rla_launch_count(void);

/* Reads and clears the device-side error word of the current device (0 = no
 * error; otherwise a bounded wait inside a kernel gave up: 1 TMA tile,
 * 2 free slot, 3 converted operand, 4 operand slot, 5 accumulator,
 * 6 split-K partner, 7 a peer's slice of an exchange call did not arrive,
 * 8 an exchange launch's CTAs did not all finish).  Synchronises the device. */
RLA_API int rla_get_device_error(unsigned int* code);

/* Message for the last non-OK status returned on this thread ("" if none). */
RLA_API const char* rla_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
RLA_API int rla_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RLA_W8A16_H */
