// Argument blocks and launchers of the mixer kernels (internal to the library).
#pragma once

#include <initializer_list>

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "linear.h"

namespace lsso {

struct Plan;
using bf16 = __nv_bfloat16;

struct MomentArgs {
  const bf16* proj;      // [B, N, W] packed (relation | content)
  const bf16* vsrc;      // second operand source (content: proj; backward: grad_output)
  const float2* phase;   // [pos_rows, N, R/2] (cos, sin)
  float* partial;        // [B*H][nchunks][ndt][2R][NC]
  int* status;
  int64_t N, W, v_stride, v_col0;
  int H, d, dt, ndt, nchunks, chunk_len, pos_batched, vec;
};

struct SolveFwdArgs {
  const float* partial;
  const float* base;
  const float* drive;
  const float* eta_raw;
  const float* counts;
  float* zbuf;  // [B*H][R][d] when no tape
  bf16* rmat;   // [B*H][d_pad x R] readout operand (K-major canonical)
  float* tape;  // nullable
  int* pivots;  // nullable
  int64_t N, tape_stride;
  int H, d, d_pad, dt, ndt, nchunks;
};

struct ReadoutArgs {
  const bf16* proj;
  const float2* phase;
  const bf16* rmat;
  const float* eta_raw;
  bf16* out;
  int* status;
  int64_t N, W, out_stride;
  int H, d, d_pad, nb, njd, ntiles, pos_batched, vec;
};

struct SolveBwdArgs {
  const float* partial;
  const float* tape;
  const float* drive;
  const float* eta_raw;
  float* dbuf;  // [B*H][R][d]
  float* lbuf;  // [B*H][R][d]
  bf16* b1y;    // [B*H][R x d_pad]
  bf16* b1c;    // [B*H][R x d_pad]
  bf16* b1a;    // [B*H][R x R]
  bf16* b2;     // [B*H][d_pad x R]
  float* gbase;   // [B*H][R][R]
  float* gdrive;  // [B*H][d][R]
  float* etadot;  // [B*H]
  int64_t N, tape_stride;
  int H, d, d_pad, dt, ndt, nchunks;
};

struct GradArgs {
  const bf16* gout;
  const bf16* proj;
  const float2* phase;
  const bf16* b1y;
  const bf16* b1c;
  const bf16* b1a;
  const bf16* b2;
  const float* eta_raw;
  bf16* gproj;
  float* etastat;  // [B*H][ntiles]
  int* status;
  int64_t N, W, D;
  int H, d, d_pad, nb, njd, ntiles, pos_batched, vec;
};

struct ParamReduceArgs {
  const float* gbase;
  const float* gdrive;
  const float* etastat;
  const float* etadot;
  const float* eta_raw;
  float* grad_base;
  float* grad_drive;
  float* grad_eta;
  int64_t B, H, R, d, ntiles;
};

struct ForwardBuffers {
  const bf16* projected;
  const float* base;
  const float* drive;
  const float* eta_raw;
  const float* positions;  // nullable
  int positions_batched;
  const float* counts;     // nullable
  bf16* mixed;
  float* tape;             // nullable (inference)
  int* pivots;             // nullable (inference)
  float2* phase;
  __half2* phase16;        // the same phases as FP16 pairs (staged per tile by the tile kernels)
  float* partial;
  float* zbuf;
  bf16* rmat;
  int* status;
  int vec;
};

struct BackwardBuffers {
  const bf16* grad_output;
  const bf16* projected;
  const float* drive;
  const float* eta_raw;
  const float* tape;
  const float* positions;
  bf16* grad_projected;
  float* grad_base;
  float* grad_drive;
  float* grad_eta;
  float2* phase;
  __half2* phase16;  // the same phases as FP16 pairs (staged by the gradient tile kernel)
  float* partial;
  float* dbuf;
  float* lbuf;
  bf16* b1y;
  bf16* b1c;
  bf16* b1a;
  bf16* b2;
  float* gbase;
  float* gdrive;
  float* etastat;
  float* etadot;
  int* status;
  int vec;
};

// Optional per-kernel timing: when set, called around every kernel launch
// (on the launching thread, with the launch stream).  Used by the profiling
// entry points of the C ABI; null in normal operation.
// Raise a kernel's dynamic shared-memory limit to `bytes` on the current
// device; the attribute is set once per (device, kernel, size) so that launches
// inside a CUDA graph capture issue no attribute calls.
cudaError_t allow_smem(const void* fn, size_t bytes);

using LaunchHook = void (*)(const char* kernel, cudaStream_t stream);
extern LaunchHook g_before_launch;
extern LaunchHook g_after_launch;

// Bracket one kernel launch with the timing hooks (no-ops unless profiling).
struct LaunchScope {
  const char* name;
  cudaStream_t stream;
  LaunchScope(const char* n, cudaStream_t s) : name(n), stream(s) {
    if (g_before_launch != nullptr) g_before_launch(name, stream);
  }
  ~LaunchScope() {
    if (g_after_launch != nullptr) g_after_launch(name, stream);
  }
};

// Head-group tile kernels of the token passes (tokens.cu).  tiled_usable()
// says whether the plan chose them and every pointer meets the TMA alignment.
bool tiled_usable(const Plan& p, std::initializer_list<const void*> ptrs);
cudaError_t launch_moments_tiled(const Plan& p, bool bwd, const bf16* proj, const bf16* gout, const __half2* phase16,
                                 float* partial, int* status, int sm_count, cudaStream_t stream);
cudaError_t launch_readout_tiled(const Plan& p, const bf16* proj, const __half2* phase16, const bf16* rmat,
                                 const float* eta_raw, bf16* out, int* status, int sm_count, cudaStream_t stream);
cudaError_t launch_grad_tiled(const Plan& p, const bf16* gout, const bf16* proj, const __half2* phase16, const bf16* b1y,
                              const bf16* b1c, const bf16* b1a, const float* eta_raw, bf16* gproj,
                              float* etastat, int* status, int sm_count, cudaStream_t stream);

// Register-resident warp solves for R <= 32 (solve.cu).
bool warp_solves_usable(const Plan& p);
cudaError_t launch_solve_forward_warp(const Plan& p, const SolveFwdArgs& s, cudaStream_t stream);
cudaError_t launch_solve_backward_warp(const Plan& p, const SolveBwdArgs& s, cudaStream_t stream);
// The backward warp solve as a persistent grid of `grid` CTAs (each takes
// systems blockIdx.x, + grid, ...), and what one of its CTAs holds on an SM.
cudaError_t launch_solve_backward_persistent(const Plan& p, const SolveBwdArgs& s, int grid, cudaStream_t stream);
CtaFootprint solve_backward_footprint(const Plan& p);

cudaError_t launch_forward(const Plan& p, const ForwardBuffers& fb, cudaStream_t stream);
cudaError_t launch_backward(const Plan& p, const BackwardBuffers& bb, cudaStream_t stream);

// The backward with one projection weight gradient beside it.  The weight
// gradient does not depend on the mixer's backward, and the backward solves
// (latency-bound, less than one wave) leave most of each SM idle: after the
// moment pass, the solves run as a persistent grid on `side` (forked from and
// joined back into `stream` with the two events) while the weight gradient
// runs on `stream`, its CTA and `solve_ctas` solve CTAs on every SM at once;
// then the gradient pass and the parameter reduction.  solve_ctas = 0 runs
// the same kernels one after the other on `stream`.  Results are identical
// either way.
struct SideStream {
  cudaStream_t stream;
  cudaEvent_t fork, join;
};
cudaError_t launch_backward_with_wgrad(const Plan& p, const BackwardBuffers& bb, const WgradPlan& wp,
                                       const WgradCall& wc, int solve_ctas, const SideStream& side,
                                       cudaStream_t stream);
// Solve CTAs per SM that fit beside one CTA of the weight gradient (0: none).
int solve_ctas_beside(const Plan& p, const WgradPlan& wp, int device);

// Sequence-parallel halves.  The moment halves run the phase table and the
// token moment pass over this rank's tokens and sum the chunk partials into
// `moments` ([B*H][ndt][2R][R + dt] forward, [B*H][ndt][2R][dt] backward,
// moment_elements); the caller sums `moments` over the ranks holding the
// other tokens, then the finish halves recompute the phase table and run the
// solves and the readout (forward) or the gradient pass and the parameter
// reduction (backward), with the solve-computed parameter terms weighted by
// `redundant` (1 on one rank, 0 on the others, so that summing the
// parameter gradients over the ranks counts them once).
int64_t moment_elements(const Plan& p, bool bwd);
cudaError_t launch_forward_moments(const Plan& p, const ForwardBuffers& fb, float* moments, cudaStream_t stream);
cudaError_t launch_forward_finish(const Plan& p, const ForwardBuffers& fb, const float* moments, cudaStream_t stream);
cudaError_t launch_backward_moments(const Plan& p, const BackwardBuffers& bb, float* moments, cudaStream_t stream);
cudaError_t launch_backward_finish(const Plan& p, const BackwardBuffers& bb, const float* moments, float redundant,
                                   cudaStream_t stream);

}  // namespace lsso
