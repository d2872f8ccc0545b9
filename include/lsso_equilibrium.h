/*
 * lsso_equilibrium.h -- C ABI of the B200 (sm_100a) LSSO mixer library
 * (lsso_equilibrium_sm100.so).
 *
 * The library implements the strict native operator of Yang916-yy/LSSO: the
 * complete DYNAMIC + Rank-Rotary mixer (forward and analytic first-order
 * backward) on BF16 packed coordinates.  Each entry point replaces one
 * operator of the reference's TORCH_LIBRARY(lsso_equilibrium) extension
 * (csrc/ball/binding.cpp:79-107 in the LSSO project); the argument meaning,
 * shapes and dtypes follow csrc/ball/common.cuh:194-269.
 *
 * Conventions
 *  - All pointers are device pointers on the current CUDA device, except
 *    where noted.  BF16 tensors are passed as void*.
 *  - The caller allocates every output and the workspace; the library
 *    allocates no device memory except the IPC-shareable exchange region of
 *    lsso_peer_region_create.  Sizes come from the *_workspace_size queries.
 *    (lsso_backward_with_wgrad creates one stream and two events of its own
 *    per device, on its first call there.)
 *  - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL is the
 *    legacy default stream).  Entry points do not synchronize.
 *  - Return value 0 means success.  Non-zero codes are LSSO_ERR_*; the text
 *    of the last error of the calling thread is lsso_last_error().  Entry
 *    points never abort the process.
 */
#ifndef LSSO_EQUILIBRIUM_H_
#define LSSO_EQUILIBRIUM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LSSO_CONTRACT_VERSION 8

#if defined(__GNUC__)
#define LSSO_API __attribute__((visibility("default")))
#else
#define LSSO_API
#endif

enum {
  LSSO_OK = 0,
  LSSO_ERR_INVALID_ARGUMENT = 1,
  LSSO_ERR_UNSUPPORTED_DEVICE = 2,
  LSSO_ERR_CUDA = 3,
  LSSO_ERR_WORKSPACE = 4
};

/* Native contract version (8).  Replaces lsso_equilibrium::contract_version
 * (csrc/ball/binding.cpp:73-75,80-83). */
LSSO_API int lsso_contract_version(void);

/* Compute capability the library was compiled for, as major*10+minor (100). */
LSSO_API int lsso_compiled_sm(void);

/* Check that CUDA device `device` is the compiled SM; 0 on success, else
 * LSSO_ERR_UNSUPPORTED_DEVICE with the reference's mismatch message
 * (csrc/ball/common.cuh:271-301). */
LSSO_API int lsso_check_device(int device);

/* Text of the calling thread's last error ("" if none). */
LSSO_API const char* lsso_last_error(void);

/* Read the kernel status word of the current device (0 = no kernel reported a
 * failure, 1 = a bounded tensor-core wait ran out, 2 = a peer rank did not reach
 * a gradient exchange in time).  Synchronizes the device.
 * reset != 0 clears it afterwards. */
LSSO_API int lsso_device_status(int reset);

/* Test hook (no counterpart in the reference): time limit, in nanoseconds,
 * of the pipeline waits of the current device's tensor-core kernels (default
 * and limit_ns == 0: one second).  A test sets a tiny limit so that those
 * waits run out: the kernels then take their abort path (each role stops,
 * in-flight TMA loads, tensor-core operations and bulk stores are awaited,
 * TMEM is freed), the status word reads 1 and the outputs are undefined; it
 * restores the default afterwards.  Synchronous; not for use while kernels of
 * the library run. */
LSSO_API int lsso_set_wait_limit_ns(unsigned long long limit_ns);

/* Floats per (sample, head) row of the training tape:
 * N*R + 3*R*R + 2*R*(D/H) + 1 (pinned by the reference's tape-size test,
 * tests/cuda/test_fast_path.py:1508-1509). */
LSSO_API int64_t lsso_tape_stride(int64_t N, int64_t H, int64_t D, int64_t R);

/* Workspace bytes for lsso_forward with these sizes (train != 0: a tape is
 * produced).  positions_batched != 0 when centered positions are [B, N]. */
LSSO_API size_t lsso_forward_workspace_size(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                                   int positions_batched, int train);

/* Forward mixer.  Replaces lsso_equilibrium::forward_inference (tape == NULL,
 * pivots == NULL) and lsso_equilibrium::forward_train
 * (csrc/ball/binding.cpp:84-90, forward.cu:1505-1556).
 *   projected          BF16 [B, N, H*R + D], contiguous; masked rows zero
 *   core_base_raw      FP32 [H, R, R]
 *   core_drive_weight  FP32 [H, D/H, R]
 *   eta_raw            FP32 [H]
 *   centered_positions FP32 [N] or [B, N] (positions_batched), or NULL for t-(N-1)/2
 *   valid_counts       FP32 [B] (max(n_valid, 1)) or NULL for N
 *   mixed              BF16 [B, N, D] output
 *   tape               FP32 [B*H, lsso_tape_stride(...)] output or NULL
 *   pivots             INT32 [B*H, R] output (one-based) or NULL
 * R must be 16, 32, 48 or 64; D must be a positive multiple of H. */
LSSO_API int lsso_forward(const void* projected, const float* core_base_raw, const float* core_drive_weight,
                 const float* eta_raw, const float* centered_positions, int positions_batched,
                 const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                 void* mixed, float* tape, int32_t* pivots, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Workspace bytes for lsso_backward. */
LSSO_API size_t lsso_backward_workspace_size(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                                    int positions_batched);

/* Analytic first-order backward.  Replaces lsso_equilibrium::backward
 * (csrc/ball/binding.cpp:91-96, backward.cu:1634-1667).
 *   grad_output            BF16 [B, N, D] (masked rows zero)
 *   projected, core_*, eta_raw, centered_positions, valid_counts as in lsso_forward
 *   tape, pivots           outputs of the training forward
 *   grad_projected         BF16 [B, N, H*R + D] output
 *   grad_core_base_raw     FP32 [H, R, R] output
 *   grad_core_drive_weight FP32 [H, D/H, R] output
 *   grad_eta_raw           FP32 [H] output
 * Parameter gradients are reduced deterministically (no atomics). */
LSSO_API int lsso_backward(const void* grad_output, const void* projected, const float* core_base_raw,
                  const float* core_drive_weight, const float* eta_raw, const float* tape,
                  const int32_t* pivots, const float* centered_positions, int positions_batched,
                  const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                  void* grad_projected, float* grad_core_base_raw, float* grad_core_drive_weight,
                  float* grad_eta_raw, void* workspace, size_t workspace_bytes, void* stream);

/* lsso_backward plus one projection weight gradient, the output
 * projection's dW_o = bf16(dY)^T bf16(mixed) in the LSSO layer (the
 * reference computes it in _TensorCoreLinear.backward,
 * lsso/ball/reference.py:229-234, before the mixer's backward of
 * csrc/ball/binding.cpp:91-96 runs; the two are independent).  The first 21
 * arguments are lsso_backward's, the wg_* ones lsso_linear_wgrad's (wg_dw,
 * wg_workspace of lsso_linear_wgrad_workspace_size(wg_T, wg_Nout, wg_K)).
 * With `concurrent` nonzero, the backward's per-(sample, head) solves, which
 * are latency-bound and fill less than one wave, run as a persistent grid on
 * a stream of the library's own (forked from and joined back into `stream`
 * with events, so the call still behaves as stream-ordered on `stream` and
 * can be captured in a CUDA graph), while the weight gradient runs on
 * `stream`, one of its CTAs beside two solve CTAs on every SM.  The library
 * creates that stream and its two events on the first such call on a device
 * (make the first call before any stream capture).  Calls from several
 * host threads share it.  When the kernels cannot share an SM (ranks above
 * 32, a per-head kernel path) or `concurrent` is 0, the same kernels run
 * one after the other on `stream`.  All outputs are bit-identical to
 * lsso_backward followed by lsso_linear_wgrad. */
LSSO_API int lsso_backward_with_wgrad(const void* grad_output, const void* projected, const float* core_base_raw,
                                      const float* core_drive_weight, const float* eta_raw, const float* tape,
                                      const int32_t* pivots, const float* centered_positions,
                                      int positions_batched, const float* valid_counts, int64_t B, int64_t N,
                                      int64_t H, int64_t D, int64_t R, void* grad_projected,
                                      float* grad_core_base_raw, float* grad_core_drive_weight, float* grad_eta_raw,
                                      void* workspace, size_t workspace_bytes, const void* wg_g, int wg_g_dtype,
                                      const void* wg_x, int wg_x_dtype, const uint8_t* wg_row_mask, int64_t wg_T,
                                      int64_t wg_Nout, int64_t wg_K, float* wg_dw, void* wg_workspace,
                                      size_t wg_workspace_bytes, int concurrent, void* stream);

/* Workspace bytes of lsso_linear (the BF16 copy of the weight in tensor-core
 * layout) for an [M, K] x [Nout, K]^T product; 0 if the shape is unsupported
 * (K must be a positive multiple of 8, at most 1024). */
LSSO_API size_t lsso_linear_workspace_size(int64_t M, int64_t K, int64_t Nout);

/* Projection GEMM of the LSSO layer.  Replaces the reference's
 * tensor_core_linear products (lsso/ball/reference.py:58-97,170-247,347-408;
 * cuBLAS / Triton there):
 *   out[t, n] = sum_k bf16(a[t, k]) * bf16(w[n, k]) (+ bias[n]),
 * FP32 accumulation and bias, one final rounding to out_dtype; rows with
 * row_mask[t] == 0 are written as zero.
 *   a            [M, K] row-major, a_dtype 0 = BF16, 1 = FP16 (rounded to BF16)
 *   weight       FP32 [Nout, K] row-major, or [K, Nout] if weight_transposed
 *   bias         FP32 [Nout] or NULL;  row_mask  uint8/bool [M] or NULL
 *   out          [M, ldo] of out_dtype 0 = BF16, 1 = FP16, 2 = FP32
 * `a` must be 16-byte aligned.  Runs on tcgen05 tensor cores fed by TMA. */
LSSO_API int lsso_linear(const void* a, int a_dtype, int64_t M, int64_t K, const float* weight,
                         int weight_transposed, int64_t Nout, const float* bias, const uint8_t* row_mask,
                         void* out, int out_dtype, int64_t ldo, void* workspace, size_t workspace_bytes,
                         void* stream);

/* The same GEMM with the weight conversion split off, so that one launch
 * prepares every weight image a layer step needs (the input and output
 * projections' weights, each in the forward and the transposed orientation)
 * instead of one conversion kernel per product.  Replaces the BF16 weight
 * copy the reference's _TensorCoreLinear makes in its forward and keeps for
 * its backward (lsso/ball/reference.py:181-183,204-205).
 *
 * lsso_linear_image_size: bytes of one image for a [.., K] x [Nout, K]^T
 *   product (depends on K and Nout only); 0 if unsupported.
 * lsso_linear_prepare: converts count (1..4) FP32 weights, weights[i] being
 *   [Nout[i], K[i]] (or [K[i], Nout[i]] if weight_transposed[i]), into
 *   images[i] (lsso_linear_image_size(K[i], Nout[i]) bytes, 16-byte aligned),
 *   in one kernel launch on `stream`.
 * lsso_linear_prepared: lsso_linear reading the weight from an image made by
 *   lsso_linear_prepare for the same K, Nout and orientation; no conversion
 *   kernel, no workspace.  Bit-identical to lsso_linear.  flags:
 *   LSSO_LINEAR_REVERSE walks the 128-row tiles of `a` from the last to the
 *   first (same result), so that a product can start with the rows the
 *   kernel before it wrote or read last, which are still in L2. */
#define LSSO_LINEAR_REVERSE 1
LSSO_API size_t lsso_linear_image_size(int64_t K, int64_t Nout);
LSSO_API int lsso_linear_prepare(int count, const float* const* weights, const int* weight_transposed,
                                 const int64_t* K, const int64_t* Nout, void* const* images, void* stream);
LSSO_API int lsso_linear_prepared(const void* a, int a_dtype, int64_t M, int64_t K, const void* image,
                                  int64_t Nout, const float* bias, const uint8_t* row_mask, void* out,
                                  int out_dtype, int64_t ldo, int flags, void* stream);

/* Workspace bytes of lsso_linear_wgrad for T tokens, Nout outputs, K inputs
 * (per-split FP32 partial tiles, enough for either operand orientation the
 * kernel picks from the dtypes); 0 if unsupported (Nout and K must be
 * positive multiples of 8). */
LSSO_API size_t lsso_linear_wgrad_workspace_size(int64_t T, int64_t Nout, int64_t K);

/* Weight gradient of a projection.  Replaces the weight VJP of the
 * reference's tensor_core_linear (lsso/ball/reference.py:229-234; cuBLAS there):
 *   dw[n, k] = sum_t bf16(g[t, n]) * bf16(x[t, k])  over tokens with row_mask[t] != 0,
 * FP32 accumulation, deterministic (fixed-order reduction of per-split
 * partials, no atomics).  g [T, Nout] and x [T, K] row-major, dtype 0 = BF16,
 * 1 = FP16 (rounded to BF16); dw FP32 [Nout, K]; g, x, dw and the workspace
 * 16-byte aligned.  The workspace size does not depend on the dtypes. */
LSSO_API int lsso_linear_wgrad(const void* g, int g_dtype, const void* x, int x_dtype, const uint8_t* row_mask,
                               int64_t T, int64_t Nout, int64_t K, float* dw, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Size of the fixed scratch area of lsso_forward_inference_noalloc (32 MiB). */
#define LSSO_NOALLOC_SCRATCH_BYTES (32u << 20)

/* Inference forward that allocates nothing -- no counterpart in the
 * reference (its operators always allocate through PyTorch).
 *
 * For callers that cannot call cudaMalloc where they run the mixer: a host
 * that owns all device memory through its own arena and forbids allocation
 * inside plugin calls, or a serving loop whose memory is fixed up front so
 * that no call can fail for lack of memory or stall in the allocator.  The
 * caller still passes every input and the output (`mixed`, BF16 [B, N, D]);
 * arguments mean what they mean for lsso_forward without a tape.  The kernels'
 * scratch (phase table, moment partials, compact state, readout operand) lives
 * in one static device array of LSSO_NOALLOC_SCRATCH_BYTES inside the
 * library, which every GPU that loads the library holds until the process
 * exits.  Shapes whose scratch would exceed it are rejected with
 * LSSO_ERR_WORKSPACE and a message naming the size (use lsso_forward then).
 * The first call on a device resolves the array's device address with
 * cudaGetSymbolAddress while that device is current; make that first call
 * before any stream capture.  The address is kept per device number for the
 * device's primary context (the one the CUDA runtime and PyTorch use): a
 * caller that runs the library in a context of its own, or that resets the
 * device (cudaDeviceReset) between calls, must load the library anew.  All calls share the array and every call
 * overwrites the parts it reads, so nothing needs clearing; calls whose
 * kernels overlap on the same GPU (e.g. on two streams) race on it. */
LSSO_API int lsso_forward_inference_noalloc(const void* projected, const float* core_base_raw,
                                            const float* core_drive_weight, const float* eta_raw,
                                            const float* centered_positions, int positions_batched,
                                            const float* valid_counts, int64_t B, int64_t N, int64_t H,
                                            int64_t D, int64_t R, void* mixed, void* stream);

/* ---- Sequence-parallel halves (no counterpart in the reference).
 *
 * One sample's tokens may be split over several GPUs ("ranks"): the mixer's
 * only cross-token quantities are the per-(sample, head) moment sums, so
 * each rank runs the moment pass over its own tokens, the caller sums the
 * moment buffers over the ranks (one all-reduce), and every rank then runs
 * the solves and its own tokens' readout / gradient pass.  Every rank passes
 * its own N (tokens it holds), the centered positions of those tokens taken
 * from the whole sequence (required), and, to the finish calls, the counts of
 * valid tokens over the whole sequence (required).  The workspace is the one
 * of lsso_forward / lsso_backward for the rank's sizes.
 *
 * Elements (FP32) of the moment buffer: B*H*ndt*2R*(R + dt) forward,
 * B*H*ndt*2R*dt backward (ndt, dt from the content width; independent of N,
 * so equal on every rank holding the same samples). */
LSSO_API size_t lsso_moment_elements(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, int backward);

/* Phase table and forward moment pass of this rank's tokens; writes the
 * rank's moment sums to `moments` (16-byte aligned). */
LSSO_API int lsso_forward_moments(const void* projected, const float* centered_positions, int positions_batched,
                                  int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, float* moments,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* Solves from the moment sums of all ranks and the readout of this rank's
 * tokens; arguments otherwise as in lsso_forward (tape and pivots optional,
 * together). */
LSSO_API int lsso_forward_finish(const void* projected, const float* core_base_raw,
                                 const float* core_drive_weight, const float* eta_raw,
                                 const float* centered_positions, int positions_batched, const float* valid_counts,
                                 int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, const float* moments,
                                 void* mixed, float* tape, int32_t* pivots, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Backward moment pass of this rank's tokens (A'^T dY sums into `moments`). */
LSSO_API int lsso_backward_moments(const void* grad_output, const void* projected, const float* centered_positions,
                                   int positions_batched, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                                   float* moments, void* workspace, size_t workspace_bytes, void* stream);

/* Backward solves from the moment sums of all ranks, this rank's gradient
 * pass and the parameter gradients.  The terms every rank computes
 * identically from the shared moments (the whole gradient of core_base_raw
 * and core_drive_weight, and the solve's part of eta_raw's) are multiplied by
 * `redundant`: pass 1 on one rank and 0 on the others, so that the sum of the
 * parameter gradients over the ranks counts them once.  Arguments otherwise
 * as in lsso_backward. */
LSSO_API int lsso_backward_finish(const void* grad_output, const void* projected, const float* core_drive_weight,
                                  const float* eta_raw, const float* tape, const float* centered_positions,
                                  int positions_batched, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                                  const float* moments, float redundant, void* grad_projected,
                                  float* grad_core_base_raw, float* grad_core_drive_weight, float* grad_eta_raw,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* ---- Peer-memory gradient exchange (replaces the NCCL all-reduce that DDP
 * or the reference's training loop runs over the parameter gradients after
 * the backward; no counterpart in the reference's own code).
 *
 * One process per GPU, all ranks on one node with peer access (NVLink /
 * NVSwitch).  Each rank creates one exchange region: a 512-byte header of
 * flags (LSSO_PEER_DATA_OFFSET) followed by `count` FP32 values, the flat
 * gradient buffer its backward writes.  The regions are shared with CUDA IPC:
 * every rank sends its 64-byte handle to the others (any host channel, e.g.
 * torch.distributed.all_gather_object) and opens theirs.  Then each
 * lsso_peer_allreduce call, made by every rank in the same order, writes
 * out[i] = scale * (sum over ranks r = 0..world-1, in that order, of region
 * r's value i) on every rank: bit-identical results on all ranks.  The call
 * returns at once; its kernel waits for the other ranks' kernels of the same
 * exchange (flags in the regions, each wait bounded by wait_limit_ns, 0 = 30
 * s).  When a peer does not come in time the status word
 * (lsso_device_status) reads 2 and `out` is undefined.  A region's values
 * may be rewritten once that rank's call has completed on its stream.  The
 * call can be captured in a CUDA graph (exchanges are numbered on the
 * device).  Regions persist across calls; counts must match on all ranks. */
#define LSSO_PEER_HANDLE_BYTES 64
#define LSSO_PEER_DATA_OFFSET 512
#define LSSO_PEER_MAX_RANKS 8
#define LSSO_PEER_DEFAULT_WAIT_NS 30000000000ull

/* Bytes of one exchange region holding `count` FP32 values (header included). */
LSSO_API size_t lsso_peer_region_bytes(int64_t count);
/* Allocate and zero this rank's region on the current device (cudaMalloc,
 * synchronous); `handle` receives LSSO_PEER_HANDLE_BYTES bytes to send to the
 * peers.  The values start at (char*)*region + LSSO_PEER_DATA_OFFSET. */
LSSO_API int lsso_peer_region_create(int64_t count, void** region, void* handle);
/* Map another process's region from its handle (not one of this process). */
LSSO_API int lsso_peer_region_open(const void* handle, void** region);
/* Unmap a region opened with lsso_peer_region_open. */
LSSO_API int lsso_peer_region_close(void* region);
/* Free this rank's region (after every peer has closed it or stopped using it). */
LSSO_API int lsso_peer_region_destroy(void* region);
/* One exchange: `regions` (host array of `world` pointers) holds every
 * rank's region as mapped in this process, this rank's own at [rank]; the
 * values [first, first + count) of every region are summed (first a multiple
 * of 4, so that several exchanges can each take one part of the buffer, in
 * the same order on every rank) into `out`, a local 16-byte aligned [count]
 * FP32 buffer. */
LSSO_API int lsso_peer_allreduce(void* const* regions, int world, int rank, int64_t first, int64_t count,
                                 float scale, float* out, unsigned long long wait_limit_ns, void* stream);

/* Per-kernel timing (no counterpart in the reference; instrumentation only).
 * lsso_profile_start() makes every subsequent kernel launch of the library
 * record a CUDA event pair on its launch stream; lsso_profile_stop()
 * synchronizes those events, stops recording and reports, per kernel name,
 * the summed device time in milliseconds and the launch count.  `names`
 * receives `capacity` slots of 32 bytes each (NUL-terminated).  Returns the
 * number of distinct kernels (or -1 on a CUDA error).  Intended for one
 * thread at a time. */
LSSO_API int lsso_profile_start(void);
LSSO_API int lsso_profile_stop(int capacity, char* names, float* total_ms, int* launches);

#ifdef __cplusplus
}
#endif

#endif /* LSSO_EQUILIBRIUM_H_ */
