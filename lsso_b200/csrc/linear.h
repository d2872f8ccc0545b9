// Projection GEMM launch plan and entry (internal to the library).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace lsso {

struct LinearPlan {
  int64_t M, K, Nout, K_pad;
  int BN, NT, grid;
  int b_stream;          // weight k-blocks streamed with the activation stages
  int stages;
  uint32_t stage_bytes;
  size_t smem, prep_bytes;
};

struct LinearCall {
  const void* a;            // activations [M, K] row-major, BF16 or FP16
  int a_fp16;
  const float* weight;      // FP32 [Nout, K], or [K, Nout] when weight_transposed
  int weight_transposed;
  const float* bias;        // nullable FP32 [Nout]
  const uint8_t* row_mask;  // nullable [M]
  void* out;                // [M, ldo] of out_dtype
  int64_t ldo;
  int out_dtype;            // 0 BF16, 1 FP16, 2 FP32
  uint8_t* prep;            // workspace for the prepared weight (plan.prep_bytes, 16-byte aligned)
  int prepared;             // 1: `prep` already holds this weight's image (launch_prepare_images); no prep kernel
  int reverse;              // 1: M tiles from the last to the first
  int* status;
};

// One weight to convert into the GEMM's BF16 image (the layout launch_linear's
// prep kernel writes into its workspace; it depends on K, Nout and the
// orientation only, not on M).
struct WeightImage {
  const float* weight;  // FP32 [Nout, K], or [K, Nout] when transposed
  int64_t K, Nout;
  int transposed;
  uint8_t* image;       // image_bytes(K, Nout) bytes, 16-byte aligned
};
constexpr int kMaxImages = 4;

struct WgradPlan {
  int64_t T, Nout, K;
  int64_t Mdim, Ndim;  // GEMM M (A-side features) and N (B-side features)
  int swapped;         // A = X and B = G (the kernel computes dW^T)
  int BNW, mtiles, ntilesw, splits, tokens_per_split, stages, grid;
  size_t smem, partial_bytes;
};

struct WgradCall {
  const void* g;            // [T, Nout] BF16 or FP16
  int g_fp16;
  const void* x;            // [T, K] BF16 or FP16
  int x_fp16;
  const uint8_t* row_mask;  // nullable [T]
  float* dw;                // FP32 [Nout, K]
  float* partial;           // workspace (plan.partial_bytes)
  int* status;
};

// What one CTA of a kernel holds on its SM (for kernels meant to share SMs).
struct CtaFootprint {
  int threads = 0;
  int regs = 0;     // per thread, as compiled
  size_t smem = 0;  // dynamic + static bytes (the per-CTA reservation not included)
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (null if unavailable).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// max_stages (<= 4): fewer pipeline stages leave shared memory for a kernel
// that runs beside this one (the split over tokens, hence the partials and
// the result, do not depend on it).
WgradPlan make_wgrad_plan(int64_t T, int64_t Nout, int64_t K, int sm_count, int g_fp16, int x_fp16,
                          int max_stages = 4);
cudaError_t launch_wgrad(const WgradPlan& plan, const WgradCall& call, cudaStream_t stream);
CtaFootprint wgrad_footprint(const WgradPlan& plan);

LinearPlan make_linear_plan(int64_t M, int64_t K, int64_t Nout, int sm_count);
bool linear_shape_supported(int64_t K);
cudaError_t launch_linear(const LinearPlan& plan, const LinearCall& call, cudaStream_t stream);

// Bytes of one prepared weight image.
size_t image_bytes(int64_t K, int64_t Nout, int sm_count);
// Converts up to kMaxImages weights in one launch.
cudaError_t launch_prepare_images(const WeightImage* images, int count, int sm_count, cudaStream_t stream);

}  // namespace lsso
