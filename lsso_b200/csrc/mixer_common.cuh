// Shared definitions of the LSSO mixer kernels: launch plan, argument blocks,
// and the per-token device helpers (Rank-Rotary rotation, the bounded
// complement, canonical operand layouts).
//
// Reference algorithm (file:line inside the LSSO project):
//   rank_rotary        lsso/ball/reference.py:691-724
//   qr_soft_frame      lsso/ball/reference.py:411-447  (used as P = A L^{-T})
//   bounded_complement lsso/ball/reference.py:450-471
//   accretive_generator / equilibrium   reference.py:474-572
//   dynamic coordinates model.py:245-268
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tc.cuh"

namespace lsso {

using bf16 = __nv_bfloat16;

constexpr int kMomentTile = 64;     // tokens per moment-pass tile (MMA K = 64)
constexpr int kTokenTile = 128;     // tokens per readout / gradient tile (MMA M = 128)
constexpr int kMaxMomentCols = 128; // widest content tile of the moment pass
constexpr int kReadoutBlock = 128;  // widest output-column block of readout / dC
constexpr int kGradChunk = 32;      // dY/C feature columns staged per gradient K-chunk
constexpr float kSoftplusOneOffset = 0.54132485461291810f;  // log(e - 1)

// ----------------------------------------------------------------------------
// Launch plan: every size derived from (B, N, H, D, R) in one place, shared by
// the workspace-size queries and the launches.
// ----------------------------------------------------------------------------
struct Plan {
  int64_t B, N, H, D, R, W, d;   // W = H*R + D, d = D / H
  int64_t BH;
  int64_t d_pad;                 // d rounded up to 16 (MMA N granularity)
  int64_t dt, ndt;               // moment-pass content tile width and count
  int64_t chunk_len, nchunks;    // tokens per moment CTA and chunks per (b, h)
  int64_t ntiles;                // 128-token tiles per sample
  int64_t nb, njd;               // readout / dC column block width and count
  int64_t pos_rows;              // phase-table rows (B when positions are per sample)
  int64_t tape_stride;           // floats per (b, h) training tape row
  int m_pad;                     // moment-pass MMA M (2R rounded up to 64/128)
  bool vec;                      // 16-byte vector path usable (d % 8 == 0)
  // Head-group tiling of the token passes (tokens.cu): a work item is one
  // 128-token tile of `hg` heads whose relation and content features fill
  // whole 64-feature boxes (nrel / nval boxes); the moment pass sums `ct`
  // tiles per chunk.
  bool tiled;
  bool tiled_grad;               // the gradient pass too (its slot is the largest)
  int hg, groups, nrel, nval, ct;
  int sms;                       // SM count the plan was made for
};

constexpr int kTileTokens = 128;
constexpr int64_t kTileBox = kTileTokens * 128;       // one 64-feature x 128-token BF16 box
constexpr int64_t kTileSmemBudget = 230400;           // dynamic shared memory per tile CTA
constexpr int kTileMaxSlots = 6;

// Bytes of one pipeline slot of each tile kernel (a multiple of 1024):
// kind 0 moments forward, 1 moments backward, 2 readout, 3 gradient.  Every
// slot holds the item's boxes, operand matrices and the tile's FP16 phase rows
// (128 tokens x R/2 pairs).
inline int64_t tile_slot_bytes(int kind, int64_t R, int64_t d, int64_t hg) {
  const int64_t nrel = (hg * R + 63) / 64, nval = hg * d / 64;  // relation boxes: hg*R features from hg*R*g
  const int64_t phase = kTileTokens * R * 2;
  int64_t bytes = 0;
  if (kind <= 1) {
    // one relation box per item (64 / R heads) + the value boxes of those heads, and one box
    // for the lo ring (two lo boxes below the slots, shared by all of them)
    const int64_t hm = 64 / R;
    bytes = (2 + (hm * d + 63) / 64) * kTileBox + phase;
  } else if (kind == 2) {
    bytes = (nrel + nval) * kTileBox + phase + hg * d * R * 2;
  } else {
    // the gradient kernel stages the tile's FP16 phase rows for its epilogue and
    // the per-head B1y, B1c (also read transposed, as B2) and B1a matrices
    bytes = (nrel + 2 * nval) * kTileBox + kTileTokens * R * 2 + hg * (2 * R * d + R * R) * 2;
  }
  return (bytes + 1023) / 1024 * 1024;
}
inline int tile_slots(int64_t slot_bytes) {
  const int64_t n = (kTileSmemBudget - 1024) / slot_bytes;
  return static_cast<int>(n > kTileMaxSlots ? kTileMaxSlots : n);
}

// Choose the head group and the moment-pass chunking of the tiled token
// kernels; leaves p.tiled false for shapes they do not cover (those use the
// per-head kernels of mixer.cu).
inline void plan_tiles(Plan& p, int sm_count) {
  p.tiled = false;
  p.tiled_grad = false;
  const bool r_ok = p.R == 16 || p.R == 32 || p.R == 48 || p.R == 64;
  const bool d_ok = p.d == 32 || p.d == 64;
  if (!r_ok || !d_ok || (p.W % 8) != 0 || p.D != p.H * p.d) return;
  const int hg = static_cast<int>(64 / (p.R < p.d ? p.R : p.d));
  if (p.H % hg != 0) return;
  // the moment pass's fused MMA has N = 64 + the value boxes of 64 / R heads (at most 256)
  if (64 + 64 * (((64 / p.R) * p.d + 63) / 64) > 256) return;
  for (int kind = 0; kind < 3; ++kind)
    if (tile_slots(tile_slot_bytes(kind, p.R, p.d, hg)) < 2) return;
  p.tiled_grad = tile_slots(tile_slot_bytes(3, p.R, p.d, hg)) >= 2;
  p.hg = hg;
  p.groups = static_cast<int>(p.H / hg);
  p.nrel = static_cast<int>((hg * p.R + 63) / 64);
  p.nval = static_cast<int>(hg * p.d / 64);
  const int64_t ntiles = (p.N + kTileTokens - 1) / kTileTokens;
  // the moment pass's items hold one relation box: 64 / R heads (one head at R = 48, 64)
  const int64_t hm = p.R <= 64 && 64 / p.R > 0 ? 64 / p.R : 1;
  const int64_t pairs = p.B * (p.H / hm);
  const int64_t sms = sm_count > 0 ? sm_count : 148;
  // Largest chunk (fewest partials) whose item count still balances over the SMs.
  int best = 1;
  double best_eff = -1.0;
  for (int ct = 16; ct >= 1; ct /= 2) {
    if (ct > ntiles && ct > 1) continue;
    const int64_t items = pairs * ((ntiles + ct - 1) / ct);
    const int64_t waves = (items + sms - 1) / sms;
    const double eff = static_cast<double>(items) / static_cast<double>(waves * sms);
    if (eff >= 0.9) {
      best = ct;
      break;
    }
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = ct;
    }
  }
  p.ct = best;
  p.tiled = true;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

inline Plan make_plan(int64_t B, int64_t N, int64_t H, int64_t D, int64_t R, bool pos_batched,
                      int sm_count) {
  Plan p{};
  p.B = B; p.N = N; p.H = H; p.D = D; p.R = R;
  p.sms = sm_count > 0 ? sm_count : 148;
  p.W = H * R + D;
  p.d = D / H;
  p.BH = B * H;
  p.d_pad = round_up(p.d, 16);
  p.dt = p.d_pad < kMaxMomentCols ? p.d_pad : kMaxMomentCols;
  p.ndt = ceil_div(p.d_pad, p.dt);
  // Enough moment CTAs to fill the GPU several times over, but never chunks
  // shorter than 256 tokens (each chunk writes one partial per (b, h)).
  const int64_t target = 8 * static_cast<int64_t>(sm_count > 0 ? sm_count : 148);
  int64_t want = ceil_div(target, p.BH * p.ndt);
  int64_t most = ceil_div(N, 256);
  if (want > most) want = most;
  if (want < 1) want = 1;
  p.chunk_len = round_up(ceil_div(N, want), kMomentTile);
  p.nchunks = ceil_div(N, p.chunk_len);
  p.ntiles = ceil_div(N, kTokenTile);
  p.nb = p.d_pad < kReadoutBlock ? p.d_pad : kReadoutBlock;
  p.njd = ceil_div(p.d_pad, p.nb);
  p.pos_rows = pos_batched ? B : 1;
  p.tape_stride = N * R + 3 * R * R + 2 * R * p.d + 1;
  p.m_pad = (2 * R <= 64) ? 64 : 128;
  p.vec = (p.d % 8) == 0;
  plan_tiles(p, sm_count);
  if (p.tiled) {
    p.chunk_len = static_cast<int64_t>(p.ct) * kTileTokens;
    p.nchunks = ceil_div(N, p.chunk_len);
    p.dt = p.d_pad;
    p.ndt = 1;
  }
  return p;
}

// Offsets (floats) of the per-system training tape row
// [unused N*R | L (R*R) | Z (R*d) | Theta (R*R) | LU (R*R) | U (R*d) | n (1)].
struct TapeLayout {
  int64_t L, Z, Theta, LU, U, n;
};
__host__ __device__ inline TapeLayout tape_layout(int64_t N, int64_t R, int64_t d) {
  TapeLayout t{};
  t.L = N * R;
  t.Z = t.L + R * R;
  t.Theta = t.Z + R * d;
  t.LU = t.Theta + R * R;
  t.U = t.LU + R * R;
  t.n = t.U + R * d;
  return t;
}

// ----------------------------------------------------------------------------
// Device helpers
// ----------------------------------------------------------------------------

// (1 - eps_fp32) * tanh(raw) through the stable logistic form (reference.py:450-471).
__device__ __forceinline__ float bounded_complement(float raw) {
  const float p = expf(-2.0f * fabsf(raw));
  const float t = (1.0f - p) / (1.0f + p);
  return (1.0f - 1.1920928955078125e-07f) * (raw >= 0.0f ? t : -t);
}
// Its derivative (1 - eps) * 4p / (1 + p)^2, finite in the FP32 tanh tail.
__device__ __forceinline__ float bounded_complement_derivative(float raw) {
  const float p = expf(-2.0f * fabsf(raw));
  const float q = 1.0f + p;
  return (1.0f - 1.1920928955078125e-07f) * 4.0f * p / (q * q);
}
// torch softplus (beta 1, threshold 20) and its derivative.
__device__ __forceinline__ float softplus20(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus20_derivative(float x) {
  return x > 20.0f ? 1.0f : 1.0f / (1.0f + expf(-x));
}

// Phase table entries: (cos, sin) of pos * 10000^(-k/(R/2)), computed in FP32,
// rounded to FP16 like the reference and stored as FP32 pairs, so applying
// them needs no conversion.  Phase4 holds 4 consecutive pairs (32 bytes).
struct Phase4 {
  float4 a, b;  // (cos0, sin0, cos1, sin1), (cos2, sin2, cos3, sin3)
};
__device__ __forceinline__ Phase4 phase_identity() {
  return Phase4{make_float4(1.0f, 0.0f, 1.0f, 0.0f), make_float4(1.0f, 0.0f, 1.0f, 0.0f)};
}
// 4 pairs starting at p (32-byte aligned), read-only path.
__device__ __forceinline__ Phase4 load_phase4(const float2* p) {
  const float4* q = reinterpret_cast<const float4*>(p);
  return Phase4{__ldg(q), __ldg(q + 1)};
}

// Rotate 8 relation coordinates (4 even/odd pairs) by their phases.
// rel holds 8 BF16 values.
__device__ __forceinline__ void rotate8(const uint4 rel, const Phase4& ph, float (&a)[8]) {
  const uint32_t rv[4] = {rel.x, rel.y, rel.z, rel.w};
  const float c[4] = {ph.a.x, ph.a.z, ph.b.x, ph.b.z};
  const float s[4] = {ph.a.y, ph.a.w, ph.b.y, ph.b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 eo = unpack_bf16(rv[i]);
    a[2 * i] = eo.x * c[i] - eo.y * s[i];
    a[2 * i + 1] = eo.x * s[i] + eo.y * c[i];
  }
}
// Adjoint of rotate8 for FP32 gradients: returns 8 values.
__device__ __forceinline__ void rotate8_transpose(const float (&g)[8], const Phase4& ph, float (&out)[8]) {
  const float c[4] = {ph.a.x, ph.a.z, ph.b.x, ph.b.z};
  const float s[4] = {ph.a.y, ph.a.w, ph.b.y, ph.b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    out[2 * i] = g[2 * i] * c[i] + g[2 * i + 1] * s[i];
    out[2 * i + 1] = -g[2 * i] * s[i] + g[2 * i + 1] * c[i];
  }
}

__device__ __forceinline__ uint4 pack8_bf16(const float (&a)[8]) {
  return make_uint4(pack_bf16(a[0], a[1]), pack_bf16(a[2], a[3]), pack_bf16(a[4], a[5]),
                    pack_bf16(a[6], a[7]));
}

// Load 8 consecutive BF16 values; 16-byte vector when vec, else element-wise
// (any alignment).  Elements at or beyond `count` read as zero.
__device__ __forceinline__ uint4 load8_bf16(const bf16* src, int count, bool vec) {
  if (vec && count >= 8) return __ldg(reinterpret_cast<const uint4*>(src));
  uint16_t e[8];
  const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = i < count ? __ldg(s + i) : uint16_t(0);
  return make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16), e[4] | (uint32_t(e[5]) << 16),
                    e[6] | (uint32_t(e[7]) << 16));
}
// Store 8 BF16 values; 16-byte vector when vec, else element-wise (first count).
__device__ __forceinline__ void store8_bf16(bf16* dst, const float (&a)[8], int count, bool vec) {
  if (vec && count >= 8) {
    *reinterpret_cast<uint4*>(dst) = pack8_bf16(a);
    return;
  }
  for (int i = 0; i < 8 && i < count; ++i) dst[i] = __float2bfloat16_rn(a[i]);
}

// Byte offset of element (mn, k) in a no-swizzle canonical operand whose core
// matrices are K-adjacent at 128 bytes and M/N-adjacent at sbo bytes.
__host__ __device__ __forceinline__ uint32_t kmajor_offset(uint32_t mn, uint32_t k, uint32_t sbo) {
  return (mn >> 3) * sbo + (k >> 3) * 128u + (mn & 7u) * 16u + (k & 7u) * 2u;
}

// Block-wide sum for 128-thread CTAs, deterministic order.
__device__ __forceinline__ float block_sum_128(float v, float* scratch4) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) scratch4[w] = v;
  __syncthreads();
  float s = 0.0f;
  if (threadIdx.x == 0) s = (scratch4[0] + scratch4[1]) + (scratch4[2] + scratch4[3]);
  return s;
}

}  // namespace lsso
