// C ABI of lsso_equilibrium_sm100.so: argument validation, workspace layout
// and the kernel sequences of the mixer.  See include/lsso_equilibrium.h.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/lsso_equilibrium.h"
#include "linear.h"
#include "mixer.h"
#include "mixer_common.cuh"
#include "peer.h"

// Fixed device scratch of lsso_forward_inference_noalloc (see below).  Host
// code must never pass `g_noalloc_scratch` itself to a kernel: on the host it
// names a stand-in, not device memory.  Its device address is resolved once
// per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LSSO_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(LSSO_ERR_CUDA, "CUDA error in %s: %s", where, cudaGetErrorString(e));
}

// Per-device status word and pipeline-wait limit (lsso::DeviceControl); the
// kernels receive the address of its first member as their `int* status`.
__device__ lsso::DeviceControl g_control = {0, 0, lsso::kWaitLimitNs};

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
int* g_status_ptr[kMaxDevices];
std::mutex g_device_mutex;

int current_device(int* device) {
  cudaError_t e = cudaGetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*device < 0 || *device >= kMaxDevices) return fail(LSSO_ERR_UNSUPPORTED_DEVICE, "device index out of range");
  return LSSO_OK;
}

int check_sm(int device) {
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (major != 10 || minor != 0) {
    return fail(LSSO_ERR_UNSUPPORTED_DEVICE,
                "the loaded LSSO CUDA extension targets SM100 but received SM%d.%d; load the matching strict "
                "artifact",
                major, minor);
  }
  return LSSO_OK;
}

// Per-device facts resolved once: SM count and the status word's address.
int device_info(int* device, int* sm_count, int** status) {
  int rc = current_device(device);
  if (rc != LSSO_OK) return rc;
  std::lock_guard<std::mutex> lock(g_device_mutex);
  if (g_status_ptr[*device] == nullptr) {
    rc = check_sm(*device);
    if (rc != LSSO_OK) return rc;
    int count = 0;
    cudaError_t e = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, *device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_control);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    g_sm_count[*device] = count;
    g_status_ptr[*device] = static_cast<int*>(ptr);
  }
  *sm_count = g_sm_count[*device];
  *status = g_status_ptr[*device];
  return LSSO_OK;
}

int validate_sizes(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R) {
  if (B <= 0 || N <= 0 || H <= 0) return fail(LSSO_ERR_INVALID_ARGUMENT, "B, N, and H must be positive");
  if (R != 16 && R != 32 && R != 48 && R != 64) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "the CUDA fast path supports rank in {16, 32, 48, 64}, got %lld",
                static_cast<long long>(R));
  }
  if (D <= 0) return fail(LSSO_ERR_INVALID_ARGUMENT, "projected width must exceed H*R for a nonempty content channel");
  if (D % H != 0) return fail(LSSO_ERR_INVALID_ARGUMENT, "projected content width D must be divisible by H");
  // Grid sizes stay below 2^31 and chunk lengths in int range.
  if (N > (int64_t(1) << 30) || B * H > (int64_t(1) << 24) || D / H > (int64_t(1) << 16)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "shape exceeds the supported launch range");
  }
  return LSSO_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct ForwardLayout {
  size_t phase, phase16, partial, zbuf, rmat, total;
};
ForwardLayout forward_layout(const lsso::Plan& p, bool train) {
  ForwardLayout l{};
  size_t off = 0;
  l.phase = off;
  off = align256(off + sizeof(float2) * p.pos_rows * p.N * (p.R / 2));
  l.phase16 = off;
  off = align256(off + sizeof(__half2) * p.pos_rows * p.N * (p.R / 2));
  l.partial = off;
  off = align256(off + sizeof(float) * p.BH * p.nchunks * p.ndt * 2 * p.R * (p.R + p.dt));
  l.zbuf = off;
  if (!train) off = align256(off + sizeof(float) * p.BH * p.R * p.d);
  l.rmat = off;
  off = align256(off + sizeof(uint16_t) * p.BH * p.d_pad * p.R);
  l.total = off;
  return l;
}


struct BackwardLayout {
  size_t phase, phase16, partial, dbuf, lbuf, b1y, b1c, b1a, b2, gbase, gdrive, etastat, etadot, total;
};
BackwardLayout backward_layout(const lsso::Plan& p) {
  BackwardLayout l{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align256(off + bytes);
    return at;
  };
  l.phase = take(sizeof(float2) * p.pos_rows * p.N * (p.R / 2));
  l.phase16 = take(sizeof(__half2) * p.pos_rows * p.N * (p.R / 2));
  l.partial = take(sizeof(float) * p.BH * p.nchunks * p.ndt * 2 * p.R * p.dt);
  l.dbuf = take(sizeof(float) * p.BH * p.R * p.d);
  l.lbuf = take(sizeof(float) * p.BH * p.R * p.d);
  l.b1y = take(sizeof(uint16_t) * p.BH * p.R * p.d_pad);
  l.b1c = take(sizeof(uint16_t) * p.BH * p.R * p.d_pad);
  l.b1a = take(sizeof(uint16_t) * p.BH * p.R * p.R);
  l.b2 = take(sizeof(uint16_t) * p.BH * p.d_pad * p.R);
  l.gbase = take(sizeof(float) * p.BH * p.R * p.R);
  l.gdrive = take(sizeof(float) * p.BH * p.d * p.R);
  l.etastat = take(sizeof(float) * p.BH * p.ntiles);
  l.etadot = take(sizeof(float) * p.BH);
  l.total = off;
  return l;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int plan_for(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, int positions_batched, lsso::Plan* plan) {
  int rc = validate_sizes(B, N, H, D, R);
  if (rc != LSSO_OK) return rc;
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  *plan = lsso::make_plan(B, N, H, D, R, positions_batched != 0, sms);
  return LSSO_OK;
}

// ---------------------------------------------------------------- allocation-free inference
// Scratch of lsso_forward_inference_noalloc: a fixed area inside the library
// image, so that callers which must not allocate device memory can still run
// the mixer.  Every device that loads the library holds it until the process
// exits.  All calls share it: the forward overwrites every byte it later
// reads (phase table, moment partials, compact state, readout operand), so
// nothing needs clearing between calls; two calls whose kernels overlap on
// the same GPU (for example on two streams) race on it.
constexpr size_t kNoallocScratchBytes = size_t(LSSO_NOALLOC_SCRATCH_BYTES);
void* g_noalloc_scratch_addr[kMaxDevices];

// ---------------------------------------------------------------- profiling
struct ProfileRecord {
  const char* name;
  cudaEvent_t start;
  cudaEvent_t stop;
};
std::vector<ProfileRecord> g_records;
std::vector<cudaEvent_t> g_event_pool;
size_t g_events_used = 0;

cudaEvent_t take_event() {
  if (g_events_used == g_event_pool.size()) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    g_event_pool.push_back(e);
  }
  return g_event_pool[g_events_used++];
}

void profile_before(const char* name, cudaStream_t stream) {
  ProfileRecord r{name, take_event(), nullptr};
  if (r.start != nullptr) cudaEventRecord(r.start, stream);
  g_records.push_back(r);
}

void profile_after(const char* name, cudaStream_t stream) {
  (void)name;
  if (g_records.empty()) return;
  cudaEvent_t e = take_event();
  if (e != nullptr) cudaEventRecord(e, stream);
  g_records.back().stop = e;
}

}  // namespace

extern "C" {

size_t lsso_linear_workspace_size(int64_t M, int64_t K, int64_t Nout) {
  g_last_error.clear();
  if (M <= 0 || Nout <= 0 || !lsso::linear_shape_supported(K)) {
    fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: K must be a positive multiple of 8 (at most 1024), M and Nout "
                                    "positive");
    return 0;
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  if (device_info(&device, &sms, &status) != LSSO_OK) return 0;
  return lsso::make_linear_plan(M, K, Nout, sms).prep_bytes;
}

int lsso_linear(const void* a, int a_dtype, int64_t M, int64_t K, const float* weight, int weight_transposed,
                int64_t Nout, const float* bias, const uint8_t* row_mask, void* out, int out_dtype, int64_t ldo,
                void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (a == nullptr || weight == nullptr || out == nullptr || workspace == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: a required pointer is NULL");
  }
  if (M <= 0 || Nout <= 0 || !lsso::linear_shape_supported(K)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT,
                "lsso_linear: K must be a positive multiple of 8 (at most 1024), M and Nout positive");
  }
  if (M > (int64_t(1) << 31) - 1 || Nout > (int64_t(1) << 20)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: shape exceeds the supported launch range");
  }
  if (a_dtype != 0 && a_dtype != 1) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: a_dtype must be 0 or 1");
  if (out_dtype < 0 || out_dtype > 2) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: out_dtype must be 0..2");
  if (ldo < Nout) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: ldo must be at least Nout");
  if (!aligned16(a) || !aligned16(workspace)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear: a and workspace must be 16-byte aligned");
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  const lsso::LinearPlan plan = lsso::make_linear_plan(M, K, Nout, sms);
  if (workspace_bytes < plan.prep_bytes) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_linear: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, plan.prep_bytes);
  }
  lsso::LinearCall c{};
  c.a = a;
  c.a_fp16 = a_dtype;
  c.weight = weight;
  c.weight_transposed = weight_transposed;
  c.bias = bias;
  c.row_mask = row_mask;
  c.out = out;
  c.ldo = ldo;
  c.out_dtype = out_dtype;
  c.prep = static_cast<uint8_t*>(workspace);
  c.status = status;
  const cudaError_t e = lsso::launch_linear(plan, c, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_linear");
  return LSSO_OK;
}

size_t lsso_linear_image_size(int64_t K, int64_t Nout) {
  g_last_error.clear();
  if (Nout <= 0 || !lsso::linear_shape_supported(K)) {
    fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_image_size: K must be a positive multiple of 8 (at most 1024), "
                                    "Nout positive");
    return 0;
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  if (device_info(&device, &sms, &status) != LSSO_OK) return 0;
  return lsso::image_bytes(K, Nout, sms);
}

int lsso_linear_prepare(int count, const float* const* weights, const int* weight_transposed, const int64_t* K,
                        const int64_t* Nout, void* const* images, void* stream) {
  g_last_error.clear();
  if (count < 1 || count > lsso::kMaxImages) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepare: count must be 1..%d", lsso::kMaxImages);
  }
  if (weights == nullptr || weight_transposed == nullptr || K == nullptr || Nout == nullptr || images == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepare: a required pointer is NULL");
  }
  lsso::WeightImage list[lsso::kMaxImages];
  for (int i = 0; i < count; ++i) {
    if (weights[i] == nullptr || images[i] == nullptr) {
      return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepare: weight or image %d is NULL", i);
    }
    if (Nout[i] <= 0 || Nout[i] > (int64_t(1) << 20) || !lsso::linear_shape_supported(K[i])) {
      return fail(LSSO_ERR_INVALID_ARGUMENT,
                  "lsso_linear_prepare: image %d: K must be a positive multiple of 8 (at most 1024), Nout positive", i);
    }
    if (!aligned16(images[i])) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepare: image %d is not 16-byte "
                                                                      "aligned", i);
    list[i] = lsso::WeightImage{weights[i], K[i], Nout[i], weight_transposed[i] != 0 ? 1 : 0,
                                static_cast<uint8_t*>(images[i])};
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  const int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  const cudaError_t e = lsso::launch_prepare_images(list, count, sms, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_linear_prepare");
  return LSSO_OK;
}

int lsso_linear_prepared(const void* a, int a_dtype, int64_t M, int64_t K, const void* image, int64_t Nout,
                         const float* bias, const uint8_t* row_mask, void* out, int out_dtype, int64_t ldo, int flags,
                         void* stream) {
  g_last_error.clear();
  if (a == nullptr || image == nullptr || out == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepared: a required pointer is NULL");
  }
  if (M <= 0 || Nout <= 0 || !lsso::linear_shape_supported(K)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT,
                "lsso_linear_prepared: K must be a positive multiple of 8 (at most 1024), M and Nout positive");
  }
  if (M > (int64_t(1) << 31) - 1 || Nout > (int64_t(1) << 20)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepared: shape exceeds the supported launch range");
  }
  if (a_dtype != 0 && a_dtype != 1) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepared: a_dtype must be 0 or 1");
  if (out_dtype < 0 || out_dtype > 2) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepared: out_dtype must be 0..2");
  }
  if (ldo < Nout) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepared: ldo must be at least Nout");
  if (!aligned16(a) || !aligned16(image)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_prepared: a and image must be 16-byte aligned");
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  const lsso::LinearPlan plan = lsso::make_linear_plan(M, K, Nout, sms);
  lsso::LinearCall c{};
  c.a = a;
  c.a_fp16 = a_dtype;
  c.weight = nullptr;
  c.bias = bias;
  c.row_mask = row_mask;
  c.out = out;
  c.ldo = ldo;
  c.out_dtype = out_dtype;
  c.prep = static_cast<uint8_t*>(const_cast<void*>(image));
  c.prepared = 1;
  c.reverse = (flags & LSSO_LINEAR_REVERSE) != 0 ? 1 : 0;
  c.status = status;
  const cudaError_t e = lsso::launch_linear(plan, c, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_linear_prepared");
  return LSSO_OK;
}

size_t lsso_linear_wgrad_workspace_size(int64_t T, int64_t Nout, int64_t K) {
  g_last_error.clear();
  if (T <= 0 || Nout <= 0 || K <= 0 || Nout % 8 != 0 || K % 8 != 0) {
    fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_linear_wgrad: T positive, Nout and K positive multiples of 8");
    return 0;
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  if (device_info(&device, &sms, &status) != LSSO_OK) return 0;
  // The operand orientation depends on the dtypes: cover both.
  const size_t plain = lsso::make_wgrad_plan(T, Nout, K, sms, 0, 0).partial_bytes;
  const size_t swapped = lsso::make_wgrad_plan(T, Nout, K, sms, 0, 1).partial_bytes;
  return plain > swapped ? plain : swapped;
}

// Validation and plan of one weight gradient (lsso_linear_wgrad and
// lsso_backward_with_wgrad; `who` names the entry point in the messages).
static int prepare_wgrad(const void* g, int g_dtype, const void* x, int x_dtype, const uint8_t* row_mask, int64_t T,
                         int64_t Nout, int64_t K, float* dw, void* workspace, size_t workspace_bytes, const char* who,
                         lsso::WgradPlan* plan, lsso::WgradCall* call) {
  if (g == nullptr || x == nullptr || dw == nullptr || workspace == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "%s: a required pointer is NULL", who);
  }
  if (T <= 0 || Nout <= 0 || K <= 0 || Nout % 8 != 0 || K % 8 != 0) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "%s: T positive, Nout and K positive multiples of 8", who);
  }
  if (T > (int64_t(1) << 31) - 1 || Nout > (int64_t(1) << 16) || K > (int64_t(1) << 16)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "%s: shape exceeds the supported launch range", who);
  }
  if ((g_dtype != 0 && g_dtype != 1) || (x_dtype != 0 && x_dtype != 1)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "%s: dtypes must be 0 (BF16) or 1 (FP16)", who);
  }
  if (!aligned16(g) || !aligned16(x) || !aligned16(dw) || !aligned16(workspace)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "%s: g, x, dw and workspace must be 16-byte aligned", who);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  *plan = lsso::make_wgrad_plan(T, Nout, K, sms, g_dtype, x_dtype);
  if (workspace_bytes < plan->partial_bytes) {
    return fail(LSSO_ERR_WORKSPACE, "%s: workspace of %zu bytes is smaller than the required %zu", who,
                workspace_bytes, plan->partial_bytes);
  }
  lsso::WgradCall c{};
  c.g = g;
  c.g_fp16 = g_dtype;
  c.x = x;
  c.x_fp16 = x_dtype;
  c.row_mask = row_mask;
  c.dw = dw;
  c.partial = static_cast<float*>(workspace);
  c.status = status;
  *call = c;
  return LSSO_OK;
}

int lsso_linear_wgrad(const void* g, int g_dtype, const void* x, int x_dtype, const uint8_t* row_mask, int64_t T,
                      int64_t Nout, int64_t K, float* dw, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  lsso::WgradPlan plan{};
  lsso::WgradCall c{};
  const int rc = prepare_wgrad(g, g_dtype, x, x_dtype, row_mask, T, Nout, K, dw, workspace, workspace_bytes,
                               "lsso_linear_wgrad", &plan, &c);
  if (rc != LSSO_OK) return rc;
  const cudaError_t e = lsso::launch_wgrad(plan, c, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_linear_wgrad");
  return LSSO_OK;
}

int lsso_forward_inference_noalloc(const void* projected, const float* core_base_raw,
                                   const float* core_drive_weight, const float* eta_raw,
                                   const float* centered_positions, int positions_batched,
                                   const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D,
                                   int64_t R, void* mixed, void* stream) {
  g_last_error.clear();
  if (projected == nullptr || core_base_raw == nullptr || core_drive_weight == nullptr || eta_raw == nullptr ||
      mixed == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward_inference_noalloc: a required pointer is NULL");
  }
  const bool batched = centered_positions != nullptr && positions_batched != 0;
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, batched ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const ForwardLayout l = forward_layout(p, false);
  if (l.total > kNoallocScratchBytes) {
    return fail(LSSO_ERR_WORKSPACE,
                "lsso_forward_inference_noalloc: this shape needs %zu bytes of scratch, more than the library's "
                "fixed %zu-byte area; use lsso_forward with a caller-allocated workspace",
                l.total, kNoallocScratchBytes);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  void* scratch = nullptr;
  {
    // First call on this device (which is current): resolve the array's device address.
    std::lock_guard<std::mutex> lock(g_device_mutex);
    if (g_noalloc_scratch_addr[device] == nullptr) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
      g_noalloc_scratch_addr[device] = ptr;
    }
    scratch = g_noalloc_scratch_addr[device];
  }
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  lsso::ForwardBuffers fb{};
  fb.projected = static_cast<const lsso::bf16*>(projected);
  fb.base = core_base_raw;
  fb.drive = core_drive_weight;
  fb.eta_raw = eta_raw;
  fb.positions = centered_positions;
  fb.positions_batched = batched ? 1 : 0;
  fb.counts = valid_counts;
  fb.mixed = static_cast<lsso::bf16*>(mixed);
  fb.tape = nullptr;
  fb.pivots = nullptr;
  fb.phase = reinterpret_cast<float2*>(ws + l.phase);
  fb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  fb.partial = reinterpret_cast<float*>(ws + l.partial);
  fb.zbuf = reinterpret_cast<float*>(ws + l.zbuf);
  fb.rmat = reinterpret_cast<lsso::bf16*>(ws + l.rmat);
  fb.status = status;
  fb.vec = p.vec && aligned16(projected) && aligned16(mixed);
  const cudaError_t e = lsso::launch_forward(p, fb, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_forward_inference_noalloc");
  return LSSO_OK;
}

// ---------------------------------------------------------------- peer-memory gradient exchange
static_assert(sizeof(cudaIpcMemHandle_t) == LSSO_PEER_HANDLE_BYTES, "IPC handle size");
static_assert(lsso::kPeerDataOffset == LSSO_PEER_DATA_OFFSET, "exchange region layout");
static_assert(lsso::kPeerMaxRanks == LSSO_PEER_MAX_RANKS, "exchange rank limit");

size_t lsso_peer_region_bytes(int64_t count) {
  if (count < 0) return 0;
  return lsso::kPeerDataOffset + align256(sizeof(float) * static_cast<size_t>(count));
}

int lsso_peer_region_create(int64_t count, void** region, void* handle) {
  g_last_error.clear();
  if (count < 0 || region == nullptr || handle == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_peer_region_create needs count >= 0 and region / handle outputs");
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  const size_t bytes = lsso_peer_region_bytes(count);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (exchange region)");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "lsso_peer_region_create");
  }
  std::memcpy(handle, &h, sizeof(h));
  *region = p;
  return LSSO_OK;
}

int lsso_peer_region_open(const void* handle, void** region) {
  g_last_error.clear();
  if (handle == nullptr || region == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_peer_region_open needs a handle and a region output");
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle (peer exchange region)");
  *region = p;
  return LSSO_OK;
}

int lsso_peer_region_close(void* region) {
  g_last_error.clear();
  if (region == nullptr) return LSSO_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(region);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return LSSO_OK;
}

int lsso_peer_region_destroy(void* region) {
  g_last_error.clear();
  if (region == nullptr) return LSSO_OK;
  const cudaError_t e = cudaFree(region);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree (exchange region)");
  return LSSO_OK;
}

int lsso_peer_allreduce(void* const* regions, int world, int rank, int64_t first, int64_t count, float scale,
                        float* out, unsigned long long wait_limit_ns, void* stream) {
  g_last_error.clear();
  if (world < 1 || world > LSSO_PEER_MAX_RANKS) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "the peer exchange supports 1 to %d ranks, got %d", LSSO_PEER_MAX_RANKS,
                world);
  }
  if (rank < 0 || rank >= world) return fail(LSSO_ERR_INVALID_ARGUMENT, "rank %d outside [0, %d)", rank, world);
  if (count < 0) return fail(LSSO_ERR_INVALID_ARGUMENT, "count must be non-negative");
  if (first < 0 || first % 4 != 0) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "first must be a non-negative multiple of 4, got %lld",
                static_cast<long long>(first));
  }
  if (regions == nullptr) return fail(LSSO_ERR_INVALID_ARGUMENT, "regions must not be NULL");
  if (count > 0 && (out == nullptr || (reinterpret_cast<uintptr_t>(out) & 15) != 0)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "out must be a 16-byte aligned device buffer");
  }
  lsso::PeerArgs a{};
  for (int r = 0; r < world; ++r) {
    if (regions[r] == nullptr || (reinterpret_cast<uintptr_t>(regions[r]) & 255) != 0) {
      return fail(LSSO_ERR_INVALID_ARGUMENT, "region %d is NULL or not an exchange region", r);
    }
    a.region[r] = static_cast<char*>(regions[r]);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  a.world = world;
  a.rank = rank;
  a.first = first;
  a.count = count;
  a.scale = scale;
  a.out = out;
  a.status = status;
  a.limit_ns = wait_limit_ns == 0 ? LSSO_PEER_DEFAULT_WAIT_NS : wait_limit_ns;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  lsso::LaunchScope scope("peer_allreduce", s);
  const cudaError_t e = lsso::launch_peer_allreduce(a, sms, s);
  if (e != cudaSuccess) return cuda_fail(e, "peer_allreduce_kernel");
  return LSSO_OK;
}

int lsso_profile_start(void) {
  g_records.clear();
  g_events_used = 0;
  lsso::g_before_launch = profile_before;
  lsso::g_after_launch = profile_after;
  return LSSO_OK;
}

int lsso_profile_stop(int capacity, char* names, float* total_ms, int* launches) {
  lsso::g_before_launch = nullptr;
  lsso::g_after_launch = nullptr;
  std::vector<std::string> keys;
  std::vector<float> totals;
  std::vector<int> counts;
  for (const ProfileRecord& r : g_records) {
    if (r.start == nullptr || r.stop == nullptr) return -1;
    if (cudaEventSynchronize(r.stop) != cudaSuccess) return -1;
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) return -1;
    size_t k = 0;
    while (k < keys.size() && keys[k] != r.name) ++k;
    if (k == keys.size()) {
      keys.emplace_back(r.name);
      totals.push_back(0.0f);
      counts.push_back(0);
    }
    totals[k] += ms;
    counts[k] += 1;
  }
  g_records.clear();
  g_events_used = 0;
  const int n = static_cast<int>(keys.size());
  for (int k = 0; k < n && k < capacity; ++k) {
    if (names != nullptr) {
      std::memset(names + 32 * k, 0, 32);
      std::strncpy(names + 32 * k, keys[k].c_str(), 31);
    }
    if (total_ms != nullptr) total_ms[k] = totals[k];
    if (launches != nullptr) launches[k] = counts[k];
  }
  return n;
}

int lsso_contract_version(void) { return LSSO_CONTRACT_VERSION; }

int lsso_compiled_sm(void) { return 100; }

int lsso_check_device(int device) {
  g_last_error.clear();
  return check_sm(device);
}

const char* lsso_last_error(void) { return g_last_error.c_str(); }

int lsso_device_status(int reset) {
  int device = 0, sms = 0;
  int* status = nullptr;
  if (device_info(&device, &sms, &status) != LSSO_OK) return -1;
  int value = 0;
  if (cudaMemcpy(&value, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (reset != 0) {
    const int zero = 0;
    if (cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return -1;
  }
  return value;
}

int lsso_set_wait_limit_ns(unsigned long long limit_ns) {
  g_last_error.clear();
  int device = 0, sms = 0;
  int* status = nullptr;
  const int rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  const unsigned long long value = limit_ns == 0 ? lsso::kWaitLimitNs : limit_ns;
  auto* control = reinterpret_cast<lsso::DeviceControl*>(status);
  const cudaError_t e = cudaMemcpy(&control->wait_limit_ns, &value, sizeof(value), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "lsso_set_wait_limit_ns");
  return LSSO_OK;
}

int64_t lsso_tape_stride(int64_t N, int64_t H, int64_t D, int64_t R) {
  if (H <= 0) return 0;
  return N * R + 3 * R * R + 2 * R * (D / H) + 1;
}

size_t lsso_forward_workspace_size(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, int positions_batched,
                                   int train) {
  lsso::Plan p{};
  if (plan_for(B, N, H, D, R, positions_batched, &p) != LSSO_OK) return 0;
  return forward_layout(p, train != 0).total;
}

size_t lsso_backward_workspace_size(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, int positions_batched) {
  lsso::Plan p{};
  if (plan_for(B, N, H, D, R, positions_batched, &p) != LSSO_OK) return 0;
  return backward_layout(p).total;
}

int lsso_forward(const void* projected, const float* core_base_raw, const float* core_drive_weight,
                 const float* eta_raw, const float* centered_positions, int positions_batched,
                 const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, void* mixed,
                 float* tape, int32_t* pivots, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (projected == nullptr || core_base_raw == nullptr || core_drive_weight == nullptr || eta_raw == nullptr ||
      mixed == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward: a required pointer is NULL");
  }
  if ((tape == nullptr) != (pivots == nullptr)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward: tape and pivots must be given together");
  }
  const bool batched = centered_positions != nullptr && positions_batched != 0;
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, batched ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const bool train = tape != nullptr;
  const ForwardLayout l = forward_layout(p, train);
  if (workspace_bytes < l.total || (l.total > 0 && workspace == nullptr)) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_forward: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, l.total);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  lsso::ForwardBuffers fb{};
  fb.projected = static_cast<const lsso::bf16*>(projected);
  fb.base = core_base_raw;
  fb.drive = core_drive_weight;
  fb.eta_raw = eta_raw;
  fb.positions = centered_positions;
  fb.positions_batched = batched ? 1 : 0;
  fb.counts = valid_counts;
  fb.mixed = static_cast<lsso::bf16*>(mixed);
  fb.tape = tape;
  fb.pivots = pivots;
  fb.phase = reinterpret_cast<float2*>(ws + l.phase);
  fb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  fb.partial = reinterpret_cast<float*>(ws + l.partial);
  fb.zbuf = train ? nullptr : reinterpret_cast<float*>(ws + l.zbuf);
  fb.rmat = reinterpret_cast<lsso::bf16*>(ws + l.rmat);
  fb.status = status;
  fb.vec = p.vec && aligned16(projected) && aligned16(mixed);
  const cudaError_t e = lsso::launch_forward(p, fb, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_forward");
  return LSSO_OK;
}

// Validation, plan and buffers of the mixer backward (lsso_backward and
// lsso_backward_with_wgrad).
static int prepare_backward(const void* grad_output, const void* projected, const float* core_base_raw,
                            const float* core_drive_weight, const float* eta_raw, const float* tape,
                            const int32_t* pivots, const float* centered_positions, int positions_batched,
                            const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                            void* grad_projected, float* grad_core_base_raw, float* grad_core_drive_weight,
                            float* grad_eta_raw, void* workspace, size_t workspace_bytes, lsso::Plan* plan,
                            lsso::BackwardBuffers* buffers) {
  (void)core_base_raw;  // Theta (and with it the base) is read from the tape
  (void)pivots;         // the LU factors carry no row exchanges (one-based identity)
  (void)valid_counts;   // the tape records each sample's count
  if (grad_output == nullptr || projected == nullptr || core_drive_weight == nullptr || eta_raw == nullptr ||
      tape == nullptr || grad_projected == nullptr || grad_core_base_raw == nullptr ||
      grad_core_drive_weight == nullptr || grad_eta_raw == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_backward: a required pointer is NULL");
  }
  const bool batched = centered_positions != nullptr && positions_batched != 0;
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, batched ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const BackwardLayout l = backward_layout(p);
  if (workspace_bytes < l.total || workspace == nullptr) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_backward: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, l.total);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  lsso::BackwardBuffers bb{};
  bb.grad_output = static_cast<const lsso::bf16*>(grad_output);
  bb.projected = static_cast<const lsso::bf16*>(projected);
  bb.drive = core_drive_weight;
  bb.eta_raw = eta_raw;
  bb.tape = tape;
  bb.positions = centered_positions;
  bb.grad_projected = static_cast<lsso::bf16*>(grad_projected);
  bb.grad_base = grad_core_base_raw;
  bb.grad_drive = grad_core_drive_weight;
  bb.grad_eta = grad_eta_raw;
  bb.phase = reinterpret_cast<float2*>(ws + l.phase);
  bb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  bb.partial = reinterpret_cast<float*>(ws + l.partial);
  bb.dbuf = reinterpret_cast<float*>(ws + l.dbuf);
  bb.lbuf = reinterpret_cast<float*>(ws + l.lbuf);
  bb.b1y = reinterpret_cast<lsso::bf16*>(ws + l.b1y);
  bb.b1c = reinterpret_cast<lsso::bf16*>(ws + l.b1c);
  bb.b1a = reinterpret_cast<lsso::bf16*>(ws + l.b1a);
  bb.b2 = reinterpret_cast<lsso::bf16*>(ws + l.b2);
  bb.gbase = reinterpret_cast<float*>(ws + l.gbase);
  bb.gdrive = reinterpret_cast<float*>(ws + l.gdrive);
  bb.etastat = reinterpret_cast<float*>(ws + l.etastat);
  bb.etadot = reinterpret_cast<float*>(ws + l.etadot);
  bb.status = status;
  bb.vec = p.vec && aligned16(projected) && aligned16(grad_output) && aligned16(grad_projected);
  *plan = p;
  *buffers = bb;
  return LSSO_OK;
}

int lsso_backward(const void* grad_output, const void* projected, const float* core_base_raw,
                  const float* core_drive_weight, const float* eta_raw, const float* tape, const int32_t* pivots,
                  const float* centered_positions, int positions_batched, const float* valid_counts, int64_t B,
                  int64_t N, int64_t H, int64_t D, int64_t R, void* grad_projected, float* grad_core_base_raw,
                  float* grad_core_drive_weight, float* grad_eta_raw, void* workspace, size_t workspace_bytes,
                  void* stream) {
  g_last_error.clear();
  lsso::Plan p{};
  lsso::BackwardBuffers bb{};
  const int rc = prepare_backward(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots,
                                  centered_positions, positions_batched, valid_counts, B, N, H, D, R,
                                  grad_projected, grad_core_base_raw, grad_core_drive_weight, grad_eta_raw,
                                  workspace, workspace_bytes, &p, &bb);
  if (rc != LSSO_OK) return rc;
  const cudaError_t e = lsso::launch_backward(p, bb, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_backward");
  return LSSO_OK;
}

// The library's own side stream per device (with its fork / join events),
// created on the first lsso_backward_with_wgrad call on that device.
static lsso::SideStream g_side[kMaxDevices];

static int side_stream(int device, lsso::SideStream* out) {
  std::lock_guard<std::mutex> lock(g_device_mutex);
  lsso::SideStream& s = g_side[device];
  if (s.stream == nullptr) {
    lsso::SideStream n{};
    cudaError_t e = cudaStreamCreateWithFlags(&n.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&n.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&n.join, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "creating the library's side stream");
    s = n;
  }
  *out = s;
  return LSSO_OK;
}

int lsso_backward_with_wgrad(const void* grad_output, const void* projected, const float* core_base_raw,
                             const float* core_drive_weight, const float* eta_raw, const float* tape,
                             const int32_t* pivots, const float* centered_positions, int positions_batched,
                             const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                             void* grad_projected, float* grad_core_base_raw, float* grad_core_drive_weight,
                             float* grad_eta_raw, void* workspace, size_t workspace_bytes, const void* wg_g,
                             int wg_g_dtype, const void* wg_x, int wg_x_dtype, const uint8_t* wg_row_mask,
                             int64_t wg_T, int64_t wg_Nout, int64_t wg_K, float* wg_dw, void* wg_workspace,
                             size_t wg_workspace_bytes, int concurrent, void* stream) {
  g_last_error.clear();
  lsso::Plan p{};
  lsso::BackwardBuffers bb{};
  int rc = prepare_backward(grad_output, projected, core_base_raw, core_drive_weight, eta_raw, tape, pivots,
                            centered_positions, positions_batched, valid_counts, B, N, H, D, R, grad_projected,
                            grad_core_base_raw, grad_core_drive_weight, grad_eta_raw, workspace, workspace_bytes,
                            &p, &bb);
  if (rc != LSSO_OK) return rc;
  lsso::WgradPlan wp{};
  lsso::WgradCall wc{};
  rc = prepare_wgrad(wg_g, wg_g_dtype, wg_x, wg_x_dtype, wg_row_mask, wg_T, wg_Nout, wg_K, wg_dw, wg_workspace,
                     wg_workspace_bytes, "lsso_backward_with_wgrad", &wp, &wc);
  if (rc != LSSO_OK) return rc;
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  int solve_ctas = 0;
  lsso::SideStream side{};
  if (concurrent) {
    // three pipeline stages leave the shared memory for solve CTAs beside each weight-gradient CTA
    const lsso::WgradPlan shared = lsso::make_wgrad_plan(wg_T, wg_Nout, wg_K, sms, wg_g_dtype, wg_x_dtype, 3);
    solve_ctas = lsso::solve_ctas_beside(p, shared, device);
    if (solve_ctas > 0) {
      wp = shared;
      rc = side_stream(device, &side);
      if (rc != LSSO_OK) return rc;
    }
  }
  const cudaError_t e =
      lsso::launch_backward_with_wgrad(p, bb, wp, wc, solve_ctas, side, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_backward_with_wgrad");
  return LSSO_OK;
}

size_t lsso_moment_elements(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, int backward) {
  g_last_error.clear();
  lsso::Plan p{};
  if (plan_for(B, N, H, D, R, 0, &p) != LSSO_OK) return 0;
  return static_cast<size_t>(lsso::moment_elements(p, backward != 0));
}

int lsso_forward_moments(const void* projected, const float* centered_positions, int positions_batched, int64_t B,
                         int64_t N, int64_t H, int64_t D, int64_t R, float* moments, void* workspace,
                         size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (projected == nullptr || centered_positions == nullptr || moments == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT,
                "lsso_forward_moments: projected, centered_positions and moments are required");
  }
  if (!aligned16(moments)) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward_moments: moments must be 16-byte aligned");
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, positions_batched != 0 ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const ForwardLayout l = forward_layout(p, true);
  if (workspace_bytes < l.total || workspace == nullptr) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_forward_moments: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, l.total);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  lsso::ForwardBuffers fb{};
  fb.projected = static_cast<const lsso::bf16*>(projected);
  fb.positions = centered_positions;
  fb.positions_batched = positions_batched != 0 ? 1 : 0;
  fb.phase = reinterpret_cast<float2*>(ws + l.phase);
  fb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  fb.partial = reinterpret_cast<float*>(ws + l.partial);
  fb.status = status;
  fb.vec = p.vec && aligned16(projected);
  const cudaError_t e = lsso::launch_forward_moments(p, fb, moments, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_forward_moments");
  return LSSO_OK;
}

int lsso_forward_finish(const void* projected, const float* core_base_raw, const float* core_drive_weight,
                        const float* eta_raw, const float* centered_positions, int positions_batched,
                        const float* valid_counts, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                        const float* moments, void* mixed, float* tape, int32_t* pivots, void* workspace,
                        size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (projected == nullptr || core_base_raw == nullptr || core_drive_weight == nullptr || eta_raw == nullptr ||
      centered_positions == nullptr || valid_counts == nullptr || moments == nullptr || mixed == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward_finish: a required pointer is NULL (centered_positions and "
                                           "valid_counts are required)");
  }
  if ((tape == nullptr) != (pivots == nullptr)) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward_finish: tape and pivots must be given together");
  }
  if (!aligned16(moments)) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_forward_finish: moments must be 16-byte aligned");
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, positions_batched != 0 ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const bool train = tape != nullptr;
  const ForwardLayout l = forward_layout(p, train);
  if (workspace_bytes < l.total || workspace == nullptr) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_forward_finish: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, l.total);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  lsso::ForwardBuffers fb{};
  fb.projected = static_cast<const lsso::bf16*>(projected);
  fb.base = core_base_raw;
  fb.drive = core_drive_weight;
  fb.eta_raw = eta_raw;
  fb.positions = centered_positions;
  fb.positions_batched = positions_batched != 0 ? 1 : 0;
  fb.counts = valid_counts;
  fb.mixed = static_cast<lsso::bf16*>(mixed);
  fb.tape = tape;
  fb.pivots = pivots;
  fb.phase = reinterpret_cast<float2*>(ws + l.phase);
  fb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  fb.partial = reinterpret_cast<float*>(ws + l.partial);
  fb.zbuf = train ? nullptr : reinterpret_cast<float*>(ws + l.zbuf);
  fb.rmat = reinterpret_cast<lsso::bf16*>(ws + l.rmat);
  fb.status = status;
  fb.vec = p.vec && aligned16(projected) && aligned16(mixed);
  const cudaError_t e = lsso::launch_forward_finish(p, fb, moments, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_forward_finish");
  return LSSO_OK;
}

int lsso_backward_moments(const void* grad_output, const void* projected, const float* centered_positions,
                          int positions_batched, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, float* moments,
                          void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (grad_output == nullptr || projected == nullptr || centered_positions == nullptr || moments == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT,
                "lsso_backward_moments: grad_output, projected, centered_positions and moments are required");
  }
  if (!aligned16(moments)) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_backward_moments: moments must be 16-byte aligned");
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, positions_batched != 0 ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const BackwardLayout l = backward_layout(p);
  if (workspace_bytes < l.total || workspace == nullptr) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_backward_moments: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, l.total);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  lsso::BackwardBuffers bb{};
  bb.grad_output = static_cast<const lsso::bf16*>(grad_output);
  bb.projected = static_cast<const lsso::bf16*>(projected);
  bb.positions = centered_positions;
  bb.phase = reinterpret_cast<float2*>(ws + l.phase);
  bb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  bb.partial = reinterpret_cast<float*>(ws + l.partial);
  bb.status = status;
  bb.vec = p.vec && aligned16(projected) && aligned16(grad_output);
  const cudaError_t e = lsso::launch_backward_moments(p, bb, moments, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_backward_moments");
  return LSSO_OK;
}

int lsso_backward_finish(const void* grad_output, const void* projected, const float* core_drive_weight,
                         const float* eta_raw, const float* tape, const float* centered_positions,
                         int positions_batched, int64_t B, int64_t N, int64_t H, int64_t D, int64_t R,
                         const float* moments, float redundant, void* grad_projected, float* grad_core_base_raw,
                         float* grad_core_drive_weight, float* grad_eta_raw, void* workspace,
                         size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (grad_output == nullptr || projected == nullptr || core_drive_weight == nullptr || eta_raw == nullptr ||
      tape == nullptr || centered_positions == nullptr || moments == nullptr || grad_projected == nullptr ||
      grad_core_base_raw == nullptr || grad_core_drive_weight == nullptr || grad_eta_raw == nullptr) {
    return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_backward_finish: a required pointer is NULL");
  }
  if (!aligned16(moments)) return fail(LSSO_ERR_INVALID_ARGUMENT, "lsso_backward_finish: moments must be 16-byte aligned");
  lsso::Plan p{};
  int rc = plan_for(B, N, H, D, R, positions_batched != 0 ? 1 : 0, &p);
  if (rc != LSSO_OK) return rc;
  const BackwardLayout l = backward_layout(p);
  if (workspace_bytes < l.total || workspace == nullptr) {
    return fail(LSSO_ERR_WORKSPACE, "lsso_backward_finish: workspace of %zu bytes is smaller than the required %zu",
                workspace_bytes, l.total);
  }
  int device = 0, sms = 0;
  int* status = nullptr;
  rc = device_info(&device, &sms, &status);
  if (rc != LSSO_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  lsso::BackwardBuffers bb{};
  bb.grad_output = static_cast<const lsso::bf16*>(grad_output);
  bb.projected = static_cast<const lsso::bf16*>(projected);
  bb.drive = core_drive_weight;
  bb.eta_raw = eta_raw;
  bb.tape = tape;
  bb.positions = centered_positions;
  bb.grad_projected = static_cast<lsso::bf16*>(grad_projected);
  bb.grad_base = grad_core_base_raw;
  bb.grad_drive = grad_core_drive_weight;
  bb.grad_eta = grad_eta_raw;
  bb.phase = reinterpret_cast<float2*>(ws + l.phase);
  bb.phase16 = reinterpret_cast<__half2*>(ws + l.phase16);
  bb.partial = reinterpret_cast<float*>(ws + l.partial);
  bb.dbuf = reinterpret_cast<float*>(ws + l.dbuf);
  bb.lbuf = reinterpret_cast<float*>(ws + l.lbuf);
  bb.b1y = reinterpret_cast<lsso::bf16*>(ws + l.b1y);
  bb.b1c = reinterpret_cast<lsso::bf16*>(ws + l.b1c);
  bb.b1a = reinterpret_cast<lsso::bf16*>(ws + l.b1a);
  bb.b2 = reinterpret_cast<lsso::bf16*>(ws + l.b2);
  bb.gbase = reinterpret_cast<float*>(ws + l.gbase);
  bb.gdrive = reinterpret_cast<float*>(ws + l.gdrive);
  bb.etastat = reinterpret_cast<float*>(ws + l.etastat);
  bb.etadot = reinterpret_cast<float*>(ws + l.etadot);
  bb.status = status;
  bb.vec = p.vec && aligned16(projected) && aligned16(grad_output) && aligned16(grad_projected);
  const cudaError_t e =
      lsso::launch_backward_finish(p, bb, moments, redundant, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lsso_backward_finish");
  return LSSO_OK;
}

}  // extern "C"
