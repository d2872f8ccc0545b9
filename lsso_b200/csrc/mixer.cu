// LSSO DYNAMIC + Rank-Rotary mixer for sm_100a: forward and analytic backward.
//
// Per sample b and head h (A' = rank_rotary(relation), n = valid count):
//   G = A'^T A' / n + I = L L^T,   S = A'^T C / sqrt(n),   Z = L^{-1} S
//   Theta = base + Z W_drive / sqrt(n),  K = F F^T + Omega,  U = (I+K)^{-1} Z
//   Y = eta C + A' [L^{-T} (2U - (1+eta) Z)] / sqrt(n)
// which is the reference operator (lsso/ball/reference.py:411-572,
// lsso/ball/model.py:245-268) with its QR soft frame written as P = A L^{-T}.
//
// Kernels (token passes run on the tensor cores through tcgen05/TMEM):
//   phase_kernel          FP16 Rank-Rotary phase table        (reference.py:691-724)
//   moments_kernel<R,0>   G and S partials per token chunk      (HBM-bound pass 1)
//   solve_forward_kernel  Cholesky, Z, Theta, K, LU, U, readout matrix per (b, h)
//   readout_kernel        Y = eta C + A' R_d per 128-token tile (HBM-bound pass 2)
//   moments_kernel<R,1>   backward statistic A'^T dY partials
//   solve_backward_kernel adjoint solves, parameter-gradient partials, pass-2 operands
//   grad_kernel           d relation / d content per 128-token tile
//   param_reduce_kernel   deterministic sum of parameter gradients over samples
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <vector>

#include "mixer.h"
#include "mixer_common.cuh"

namespace lsso {

// ============================================================================
// Phase table: (cos, sin) of pos * 10000^(-k/(R/2)), FP32 angle, rounded to
// FP16 (reference.py:691-724) and stored as FP32 pairs.
// ============================================================================
struct InvFreq {
  float v[32];
};

// One thread per (token, frequency) of position rows blockIdx.y, + gridDim.y, ...; the
// frequency table stays in parameter space (__grid_constant__), so indexing it
// with the thread's frequency does not copy it to local memory.
__global__ void phase_kernel(const float* __restrict__ pos, int64_t rows, int N, int half,
                             const __grid_constant__ InvFreq f,
                             float2* __restrict__ out, __half2* __restrict__ out16) {
  pdl_wait();
  const int i = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;  // t * half + k within the row
  if (i >= N * half) return;
  const int t = i / half, k = i - t * half;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const float p = pos != nullptr ? pos[row * N + t] : static_cast<float>(t) - 0.5f * static_cast<float>(N - 1);
    float s, c;
    sincosf(p * f.v[k], &s, &c);
    const __half2 h = __floats2half2_rn(c, s);
    const int64_t o = row * N * half + i;
    out[o] = __half22float2(h);
    if (out16 != nullptr) out16[o] = h;
  }
}

// ============================================================================
// Moment pass (forward G/S and backward A'^T dY).
//
// One CTA per (b, h, token chunk, content tile).  Each 64-token tile:
//   cp.async the relation slice (row-major) and the content/dY slice (straight
//   into the MN-major operand layout), rotate the relation, split it into
//   BF16 hi + lo parts (A' = hi + lo to 2^-17) and store both MN-major;
//   one thread issues  D[:, 0:R)   += [hi | lo]^T hi       (forward only)
//                      D[:, R:..) += [hi | lo]^T V
//   with M = 2R (padded to 64/128) features, K = 64 tokens.  Rows [0, R) of D
//   hold hi-products and rows [R, 2R) lo-products; the solve kernel combines
//   G = hh + lh + lh^T and S = hV + lV.  Three load stages, two operand
//   buffers, MMA completion tracked by two mbarriers.
// ============================================================================
template <int R, bool BWD>
__global__ void __launch_bounds__(128) moments_kernel(const MomentArgs a) {
  pdl_wait();
  constexpr int M_PAD = (2 * R <= 64) ? 64 : 128;
  constexpr int RQ = R / 8;
  constexpr int X_BYTES = M_PAD * kMomentTile * 2;
  constexpr int RAW_BYTES = kMomentTile * R * 2;
  constexpr uint32_t SBO = kMomentTile * 16;  // M/N-adjacent core matrices (MN-major)
  const int dt = a.dt;
  const int V_BYTES = dt * kMomentTile * 2;
  const int NC = (BWD ? 0 : R) + dt;
  const uint32_t tcols = tmem_cols_for(NC);

  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* xbuf = smem;
  uint8_t* rawbuf = xbuf + 2 * X_BYTES;
  uint8_t* vbuf = rawbuf + 3 * RAW_BYTES;
  __shared__ __align__(8) uint64_t bars[3];  // [2]: teardown drain of the MMA thread
  __shared__ uint32_t tmem_s;

  int64_t blk = blockIdx.x;
  const int j = static_cast<int>(blk % a.ndt);
  blk /= a.ndt;
  const int h = static_cast<int>(blk % a.H);
  blk /= a.H;
  const int c = static_cast<int>(blk % a.nchunks);
  const int64_t b = blk / a.nchunks;
  const int64_t t_begin = static_cast<int64_t>(c) * a.chunk_len;
  const int64_t t_end = min(a.N, t_begin + a.chunk_len);
  const int ntiles = static_cast<int>((t_end - t_begin + kMomentTile - 1) / kMomentTile);
  const int tid = threadIdx.x;
  const int64_t pb = a.pos_batched ? b : 0;
  const int col0 = j * dt;
  const bool vec = a.vec != 0;

  // Zero the padding feature groups of both operand buffers once.
  constexpr int PAD_GROUPS = M_PAD / 8 - 2 * RQ;
  if constexpr (PAD_GROUPS > 0) {
    for (int idx = tid; idx < 2 * PAD_GROUPS * kMomentTile; idx += 128) {
      const int buf = idx / (PAD_GROUPS * kMomentTile);
      const int rem = idx % (PAD_GROUPS * kMomentTile);
      uint8_t* p = xbuf + buf * X_BYTES + (2 * RQ + rem / kMomentTile) * (kMomentTile * 16) + (rem % kMomentTile) * 16;
      *reinterpret_cast<uint4*>(p) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if (tid == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    mbar_init(smem_u32(&bars[2]), 1);
    fence_mbar_init();
  }
  if (tid < 32) tmem_alloc(smem_u32(&tmem_s), tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;

  auto load_tile = [&](int i, int s) {
    const int64_t t0 = t_begin + static_cast<int64_t>(i) * kMomentTile;
    uint8_t* raw = rawbuf + s * RAW_BYTES;
    uint8_t* vb = vbuf + s * V_BYTES;
    for (int idx = tid; idx < kMomentTile * RQ; idx += 128) {
      const int t = idx / RQ, q = idx % RQ;
      const int64_t tok = t0 + t;
      const bool valid = tok < t_end;
      const bf16* src = a.proj + ((b * a.N + (valid ? tok : t_begin)) * a.W + static_cast<int64_t>(h) * R + 8 * q);
      uint8_t* dst = raw + t * (R * 2) + q * 16;
      if (vec) {
        cp_async_16(smem_u32(dst), src, valid ? 16u : 0u);
      } else {
        *reinterpret_cast<uint4*>(dst) = valid ? load8_bf16(src, 8, false) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    const int VQ = dt / 8;
    for (int idx = tid; idx < kMomentTile * VQ; idx += 128) {
      const int t = idx / VQ, g = idx % VQ;
      const int64_t tok = t0 + t;
      const int col = col0 + 8 * g;
      const int cnt = min(8, a.d - col);
      const bool valid = tok < t_end && cnt > 0;
      const bf16* src = a.vsrc + ((b * a.N + (valid ? tok : t_begin)) * a.v_stride + a.v_col0 +
                                  static_cast<int64_t>(h) * a.d + (valid ? col : 0));
      uint8_t* dst = vb + g * (kMomentTile * 16) + t * 16;
      if (vec) {
        cp_async_16(smem_u32(dst), src, valid ? 16u : 0u);
      } else {
        *reinterpret_cast<uint4*>(dst) = valid ? load8_bf16(src, cnt, false) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };

  auto transform = [&](int i, int s, int xb) {
    const int64_t t0 = t_begin + static_cast<int64_t>(i) * kMomentTile;
    const uint8_t* raw = rawbuf + s * RAW_BYTES;
    uint8_t* x = xbuf + xb * X_BYTES;
    for (int idx = tid; idx < kMomentTile * RQ; idx += 128) {
      const int t = idx / RQ, q = idx % RQ;
      const int64_t tok = t0 + t;
      const uint4 rv = *reinterpret_cast<const uint4*>(raw + t * (R * 2) + q * 16);
      Phase4 ph = phase_identity();
      if (tok < t_end) ph = load_phase4(a.phase + ((pb * a.N + tok) * (R / 2) + 4 * q));
      float v[8];
      rotate8(rv, ph, v);
      const uint4 hi = pack8_bf16(v);
      const float2 h0 = unpack_bf16(hi.x), h1 = unpack_bf16(hi.y), h2 = unpack_bf16(hi.z), h3 = unpack_bf16(hi.w);
      float lo[8] = {v[0] - h0.x, v[1] - h0.y, v[2] - h1.x, v[3] - h1.y,
                     v[4] - h2.x, v[5] - h2.y, v[6] - h3.x, v[7] - h3.y};
      *reinterpret_cast<uint4*>(x + q * (kMomentTile * 16) + t * 16) = hi;
      *reinterpret_cast<uint4*>(x + (RQ + q) * (kMomentTile * 16) + t * 16) = pack8_bf16(lo);
    }
  };

  const uint32_t idesc_a = make_idesc(M_PAD, R, true, true);
  const uint32_t idesc_v = make_idesc(M_PAD, dt, true, true);
  auto issue = [&](int i, int s, int xb) {
    const uint32_t xa = smem_u32(xbuf + xb * X_BYTES);
    const uint32_t va = smem_u32(vbuf + s * V_BYTES);
#pragma unroll
    for (int ks = 0; ks < kMomentTile / 16; ++ks) {
      const uint32_t acc = (i > 0 || ks > 0) ? 1u : 0u;
      const uint64_t ad = make_desc(xa + ks * 256, 128, SBO);
      if (!BWD) mma_bf16(tmem, ad, ad, idesc_a, acc);
      mma_bf16(tmem + (BWD ? 0 : R), ad, make_desc(va + ks * 256, 128, SBO), idesc_v, acc);
    }
    mma_commit(smem_u32(&bars[i & 1]));
  };

  load_tile(0, 0);
  cp_async_commit();
  if (ntiles > 1) load_tile(1, 1);
  cp_async_commit();
  bool ok = true;
  for (int i = 0; i < ntiles; ++i) {
    cp_async_wait<1>();
    ok = __syncthreads_and(ok);
    transform(i, i % 3, i & 1);
    fence_proxy_async();
    __syncthreads();
    if (tid == 0 && ok) issue(i, i % 3, i & 1);
    if (i >= 1 && ok) ok = mbar_wait(smem_u32(&bars[(i - 1) & 1]), ((i - 1) >> 1) & 1, a.status);
    if (i + 2 < ntiles) load_tile(i + 2, (i + 2) % 3);
    cp_async_commit();
  }
  cp_async_wait<0>();
  if (ok) ok = mbar_wait(smem_u32(&bars[(ntiles - 1) & 1]), ((ntiles - 1) >> 1) & 1, a.status);
  ok = __syncthreads_and(ok);
  tc_fence_after();

  if (ok) {
    const int w = tid >> 5, lane = tid & 31;
    int row;
    bool rvalid;
    if (M_PAD == 128) {
      row = 32 * w + lane;
      rvalid = row < 2 * R;
    } else {
      row = 16 * w + lane;
      rvalid = lane < 16 && row < 2 * R;
    }
    float* out = a.partial + (((b * a.H + h) * a.nchunks + c) * a.ndt + j) * static_cast<int64_t>(2 * R * NC);
    for (int c0 = 0; c0 < NC; c0 += 8) {
      float v[8];
      tmem_ld8(tmem + (static_cast<uint32_t>(32 * w) << 16) + c0, v);
      tmem_ld_wait();
      if (rvalid) {
        float4* o = reinterpret_cast<float4*>(out + static_cast<int64_t>(row) * NC + c0);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    }
  }
  if (tid == 0) mma_drain(smem_u32(&bars[2]), a.status);  // tid 0 issued the MMAs
  tc_fence_before();
  __syncthreads();
  if (tid < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

// ============================================================================
// Per-(b, h) forward solve: Cholesky of G, Z, Theta, accretive generator, LU
// without pivoting (I + K has a positive-definite symmetric part), U, and the
// BF16 readout operand R_d = L^{-T} (2U - (1+eta) Z) / sqrt(n).
// ============================================================================
constexpr int kSolveThreads = 256;
constexpr int kColChunk = 32;

template <int R>
struct SolveSmem {
  static constexpr int LD = R + 1;
  static constexpr int CLD = kColChunk + 1;
};

// Right-looking Cholesky of the lower triangle of L (in place), run by warp 0
// alone with warp-level synchronisation (the factorisation is a chain of R
// short steps; block-wide barriers per step would dominate its latency).
// Every thread of the block must call it; the upper triangle is zeroed.
template <int R>
__device__ __forceinline__ void cholesky_inplace(float* L) {
  constexpr int LD = R + 1;
  const int tid = threadIdx.x;
  __syncthreads();
  if (tid < 32) {
    for (int k = 0; k < R; ++k) {
      const float piv = sqrtf(L[k * LD + k]);
      __syncwarp();
      if (tid == 0) L[k * LD + k] = piv;
      for (int i = k + 1 + tid; i < R; i += 32) L[i * LD + k] /= piv;
      __syncwarp();
      for (int i = k + 1 + tid; i < R; i += 32) {
        const float lik = L[i * LD + k];
        for (int jj = k + 1; jj <= i; ++jj) L[i * LD + jj] -= lik * L[jj * LD + k];
      }
      __syncwarp();
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    if (jj > i) L[i * LD + jj] = 0.0f;
  }
  __syncthreads();
}

// Doolittle LU without pivoting (in place; unit lower factor below the
// diagonal), run by warp 0 with warp-level synchronisation.  I + K has a
// positive-definite symmetric part, so no pivoting is needed.
template <int R>
__device__ __forceinline__ void lu_inplace(float* M) {
  constexpr int LD = R + 1;
  const int tid = threadIdx.x;
  __syncthreads();
  if (tid < 32) {
    for (int k = 0; k < R; ++k) {
      const float piv = M[k * LD + k];
      for (int i = k + 1 + tid; i < R; i += 32) M[i * LD + k] /= piv;
      __syncwarp();
      for (int i = k + 1 + tid; i < R; i += 32) {
        const float lik = M[i * LD + k];
        for (int jj = k + 1; jj < R; ++jj) M[i * LD + jj] -= lik * M[k * LD + jj];
      }
      __syncwarp();
    }
  }
  __syncthreads();
}

// Column-wise triangular solves on a [R][CLD] column chunk (one thread per column).
template <int R>
__device__ __forceinline__ void forward_subst(const float* L, float* X, int cc) {  // X <- L^{-1} X
  constexpr int LD = R + 1, CLD = kColChunk + 1;
  for (int i = 0; i < R; ++i) {
    float z = X[i * CLD + cc];
    for (int k = 0; k < i; ++k) z -= L[i * LD + k] * X[k * CLD + cc];
    X[i * CLD + cc] = z / L[i * LD + i];
  }
}
template <int R>
__device__ __forceinline__ void backward_subst_transposed(const float* L, float* X, int cc) {  // X <- L^{-T} X
  constexpr int LD = R + 1, CLD = kColChunk + 1;
  for (int i = R - 1; i >= 0; --i) {
    float z = X[i * CLD + cc];
    for (int k = i + 1; k < R; ++k) z -= L[k * LD + i] * X[k * CLD + cc];
    X[i * CLD + cc] = z / L[i * LD + i];
  }
}
template <int R>
__device__ __forceinline__ void lu_solve(const float* M, float* X, int cc) {  // X <- (LU)^{-1} X
  constexpr int LD = R + 1, CLD = kColChunk + 1;
  for (int i = 0; i < R; ++i) {
    float z = X[i * CLD + cc];
    for (int k = 0; k < i; ++k) z -= M[i * LD + k] * X[k * CLD + cc];
    X[i * CLD + cc] = z;
  }
  for (int i = R - 1; i >= 0; --i) {
    float z = X[i * CLD + cc];
    for (int k = i + 1; k < R; ++k) z -= M[i * LD + k] * X[k * CLD + cc];
    X[i * CLD + cc] = z / M[i * LD + i];
  }
}
template <int R>
__device__ __forceinline__ void lu_solve_transposed(const float* M, float* X, int cc) {  // X <- (LU)^{-T} X
  constexpr int LD = R + 1, CLD = kColChunk + 1;
  for (int i = 0; i < R; ++i) {  // U^T y = x  (lower, non-unit)
    float z = X[i * CLD + cc];
    for (int k = 0; k < i; ++k) z -= M[k * LD + i] * X[k * CLD + cc];
    X[i * CLD + cc] = z / M[i * LD + i];
  }
  for (int i = R - 1; i >= 0; --i) {  // L^T x = y  (upper, unit)
    float z = X[i * CLD + cc];
    for (int k = i + 1; k < R; ++k) z -= M[k * LD + i] * X[k * CLD + cc];
    X[i * CLD + cc] = z;
  }
}

template <int R>
size_t solve_forward_smem() {
  return sizeof(float) * (3 * R * (R + 1) + 2 * R * (kColChunk + 1) + R);
}

template <int R>
__global__ void __launch_bounds__(kSolveThreads) solve_forward_kernel(const SolveFwdArgs a) {
  pdl_wait();
  constexpr int LD = R + 1, CLD = kColChunk + 1;
  extern __shared__ __align__(16) float fsm[];
  float* L = fsm;
  float* Mm = L + R * LD;
  float* Th = Mm + R * LD;
  float* Xc = Th + R * LD;
  float* Yc = Xc + R * CLD;
  float* fdiag = Yc + R * CLD;
  const int tid = threadIdx.x;
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / a.H;
  const int h = static_cast<int>(bh % a.H);
  const int d = a.d;
  const float n = a.counts != nullptr ? a.counts[b] : static_cast<float>(a.N);
  const float rsn = 1.0f / sqrtf(n);
  const int NC = R + a.dt;
  const int64_t pstride = static_cast<int64_t>(2 * R) * NC;
  const float* pbase = a.partial + bh * a.nchunks * a.ndt * pstride;
  const TapeLayout tl = tape_layout(a.N, R, d);
  float* tape = a.tape != nullptr ? a.tape + bh * a.tape_stride : nullptr;
  float* Zg = tape != nullptr ? tape + tl.Z : a.zbuf + bh * static_cast<int64_t>(R) * d;

  // 1. G = (hh + lh + lh^T) / n + I  (lower triangle)
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, k = idx % R;
    if (k > i) continue;
    float s = 0.0f;
    for (int ch = 0; ch < a.nchunks; ++ch) {
      const float* P = pbase + static_cast<int64_t>(ch) * a.ndt * pstride;
      s += P[i * NC + k] + P[(R + i) * NC + k] + P[(R + k) * NC + i];
    }
    L[i * LD + k] = s * (rsn * rsn) + (i == k ? 1.0f : 0.0f);
  }
  for (int idx = tid; idx < R * R; idx += kSolveThreads) Th[(idx / R) * LD + idx % R] = 0.0f;
  __syncthreads();
  // 2. Cholesky
  cholesky_inplace<R>(L);
  // 3. Z = L^{-1} S chunk by chunk; Theta accumulator += Z W_drive
  for (int c0 = 0; c0 < d; c0 += kColChunk) {
    const int cw = min(kColChunk, d - c0);
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const int col = c0 + cc, jt = col / a.dt, cl = col % a.dt;
      float s = 0.0f;
      for (int ch = 0; ch < a.nchunks; ++ch) {
        const float* P = pbase + (static_cast<int64_t>(ch) * a.ndt + jt) * pstride;
        s += P[i * NC + R + cl] + P[(R + i) * NC + R + cl];
      }
      Xc[i * CLD + cc] = s * rsn;
    }
    __syncthreads();
    if (tid < cw) forward_subst<R>(L, Xc, tid);
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      Zg[static_cast<int64_t>(i) * d + c0 + cc] = Xc[i * CLD + cc];
    }
    const float* Wd = a.drive + (static_cast<int64_t>(h) * d + c0) * R;
    for (int idx = tid; idx < R * R; idx += kSolveThreads) {
      const int i = idx / R, jj = idx % R;
      float s = 0.0f;
      for (int cc = 0; cc < cw; ++cc) s += Xc[i * CLD + cc] * Wd[cc * R + jj];
      Th[i * LD + jj] += s;
    }
    __syncthreads();
  }
  // 4. Theta = base + acc / sqrt(n);  F diagonal
  const float* base = a.base + static_cast<int64_t>(h) * R * R;
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    Th[i * LD + jj] = base[idx] + Th[i * LD + jj] * rsn;
  }
  __syncthreads();
  for (int i = tid; i < R; i += kSolveThreads) fdiag[i] = softplus20(Th[i * LD + i] + kSoftplusOneOffset);
  __syncthreads();
  // 5. M = I + F F^T + Omega
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    const int kmax = min(i, jj);
    float s = 0.0f;
    for (int k = 0; k <= kmax; ++k) {
      const float fi = k < i ? Th[i * LD + k] : fdiag[i];
      const float fj = k < jj ? Th[jj * LD + k] : fdiag[jj];
      s += fi * fj;
    }
    const float omega = i < jj ? Th[i * LD + jj] : (i > jj ? -Th[jj * LD + i] : 0.0f);
    Mm[i * LD + jj] = (i == jj ? 1.0f : 0.0f) + s + omega;
  }
  __syncthreads();
  if (tape != nullptr) {
    for (int idx = tid; idx < R * R; idx += kSolveThreads) {
      const int i = idx / R, jj = idx % R;
      tape[tl.L + idx] = L[i * LD + jj];
      tape[tl.Theta + idx] = Th[i * LD + jj];
    }
    if (tid == 0) tape[tl.n] = n;
  }
  // 6. LU
  lu_inplace<R>(Mm);
  if (tape != nullptr) {
    for (int idx = tid; idx < R * R; idx += kSolveThreads) tape[tl.LU + idx] = Mm[(idx / R) * LD + idx % R];
  }
  if (a.pivots != nullptr) {
    for (int i = tid; i < R; i += kSolveThreads) a.pivots[bh * R + i] = i + 1;
  }
  // 7./8. U, M' and the readout operand, chunk by chunk.
  const float eta = bounded_complement(a.eta_raw[h]);
  uint8_t* rm = reinterpret_cast<uint8_t*>(a.rmat + bh * a.d_pad * R);
  constexpr uint32_t RSBO = R * 16;
  for (int c0 = 0; c0 < d; c0 += kColChunk) {
    const int cw = min(kColChunk, d - c0);
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const float z = Zg[static_cast<int64_t>(i) * d + c0 + cc];
      Xc[i * CLD + cc] = z;
      Yc[i * CLD + cc] = z;
    }
    __syncthreads();
    if (tid < cw) {
      lu_solve<R>(Mm, Yc, tid);  // U
      for (int i = 0; i < R; ++i) Xc[i * CLD + tid] = 2.0f * Yc[i * CLD + tid] - (1.0f + eta) * Xc[i * CLD + tid];
      backward_subst_transposed<R>(L, Xc, tid);
    }
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const int col = c0 + cc;
      if (tape != nullptr) tape[tl.U + static_cast<int64_t>(i) * d + col] = Yc[i * CLD + cc];
      *reinterpret_cast<bf16*>(rm + kmajor_offset(col, i, RSBO)) = __float2bfloat16_rn(Xc[i * CLD + cc] * rsn);
    }
  }
  for (int idx = tid; idx < (a.d_pad - d) * R; idx += kSolveThreads) {
    const int col = d + idx / R, i = idx % R;
    *reinterpret_cast<bf16*>(rm + kmajor_offset(col, i, RSBO)) = __float2bfloat16_rn(0.0f);
  }
}

// ============================================================================
// Readout: Y[t, c] = eta C[t, c] + sum_i A'[t, i] R_d[i, c]
// One CTA per (b, 128-token tile, h, column block): M = 128 tokens, K = R,
// N = column block; the epilogue adds eta C in FP32 and stores BF16.
// ============================================================================
template <int R>
size_t readout_smem(int nb) {
  return static_cast<size_t>(kTokenTile) * R * 2 + static_cast<size_t>(nb) * R * 2;
}

template <int R>
__global__ void __launch_bounds__(128) readout_kernel(const ReadoutArgs a) {
  pdl_wait();
  constexpr int RQ = R / 8;
  constexpr uint32_t SBO = R * 16;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sA = smem;
  uint8_t* sB = smem + kTokenTile * R * 2;
  __shared__ __align__(8) uint64_t bar, drain;
  __shared__ uint32_t tmem_s;

  int64_t blk = blockIdx.x;
  const int jd = static_cast<int>(blk % a.njd);
  blk /= a.njd;
  const int h = static_cast<int>(blk % a.H);
  blk /= a.H;
  const int tile = static_cast<int>(blk % a.ntiles);
  const int64_t b = blk / a.ntiles;
  const int tid = threadIdx.x;
  const int64_t pb = a.pos_batched ? b : 0;
  const bool vec = a.vec != 0;
  const int nb = min(a.nb, a.d_pad - jd * a.nb);
  const uint32_t tcols = tmem_cols_for(nb);
  const int64_t tok0 = static_cast<int64_t>(tile) * kTokenTile;

  if (tid == 0) {
    mbar_init(smem_u32(&bar), 1);
    mbar_init(smem_u32(&drain), 1);
    fence_mbar_init();
  }
  if (tid < 32) tmem_alloc(smem_u32(&tmem_s), tcols);

  // B operand: the column block of the readout matrix (already in canonical layout).
  const uint8_t* rsrc = reinterpret_cast<const uint8_t*>(a.rmat + (b * a.H + h) * a.d_pad * R) +
                        static_cast<int64_t>(jd) * a.nb * R * 2;
  for (int idx = tid; idx < nb * R * 2 / 16; idx += 128) cp_async_16(smem_u32(sB + idx * 16), rsrc + idx * 16, 16u);
  cp_async_commit();
  // A operand: rotated relation, BF16, K-major.
  for (int idx = tid; idx < kTokenTile * RQ; idx += 128) {
    const int t = idx / RQ, q = idx % RQ;
    const int64_t tok = tok0 + t;
    uint4 rv = make_uint4(0u, 0u, 0u, 0u);
    Phase4 ph = phase_identity();
    if (tok < a.N) {
      rv = load8_bf16(a.proj + (b * a.N + tok) * a.W + static_cast<int64_t>(h) * R + 8 * q, 8, vec);
      ph = load_phase4(a.phase + ((pb * a.N + tok) * (R / 2) + 4 * q));
    }
    float v[8];
    rotate8(rv, ph, v);
    *reinterpret_cast<uint4*>(sA + kmajor_offset(t, 8 * q, SBO)) = pack8_bf16(v);
  }
  cp_async_wait<0>();
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;
  if (tid == 0) {
    const uint32_t idesc = make_idesc(128, nb, false, false);
#pragma unroll
    for (int ks = 0; ks < R / 16; ++ks) {
      mma_bf16(tmem, make_desc(smem_u32(sA) + ks * 256, 128, SBO), make_desc(smem_u32(sB) + ks * 256, 128, SBO),
               idesc, ks > 0 ? 1u : 0u);
    }
    mma_commit(smem_u32(&bar));
  }
  // Prefetch-free epilogue inputs are read after the wait; eta in FP32.
  const float eta = bounded_complement(a.eta_raw[h]);
  bool ok = mbar_wait(smem_u32(&bar), 0, a.status);
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok) {
    const int w = tid >> 5, lane = tid & 31;
    const int t = 32 * w + lane;
    const int64_t tok = tok0 + t;
    const bool live = tok < a.N;
    const bf16* crow = a.proj + (b * a.N + (live ? tok : 0)) * a.W + static_cast<int64_t>(a.H) * R +
                       static_cast<int64_t>(h) * a.d;
    bf16* orow = a.out + (b * a.N + (live ? tok : 0)) * a.out_stride + static_cast<int64_t>(h) * a.d;
    for (int c0 = 0; c0 < nb; c0 += 8) {
      float v[8];
      tmem_ld8(tmem + (static_cast<uint32_t>(32 * w) << 16) + c0, v);
      tmem_ld_wait();
      const int col = jd * a.nb + c0;
      const int cnt = min(8, a.d - col);
      if (live && cnt > 0) {
        const uint4 cv = load8_bf16(crow + col, cnt, vec);
        const float2 c01 = unpack_bf16(cv.x), c23 = unpack_bf16(cv.y), c45 = unpack_bf16(cv.z), c67 = unpack_bf16(cv.w);
        float y[8] = {fmaf(eta, c01.x, v[0]), fmaf(eta, c01.y, v[1]), fmaf(eta, c23.x, v[2]), fmaf(eta, c23.y, v[3]),
                      fmaf(eta, c45.x, v[4]), fmaf(eta, c45.y, v[5]), fmaf(eta, c67.x, v[6]), fmaf(eta, c67.y, v[7])};
        store8_bf16(orow + col, y, cnt, vec);
      }
    }
  }
  if (tid == 0) mma_drain(smem_u32(&drain), a.status);  // tid 0 issued the MMAs
  tc_fence_before();
  __syncthreads();
  if (tid < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

// ============================================================================
// Per-(b, h) backward solve.
//   D  = L^{-1} (A'^T dY) / sqrt(n),  lam = (I+K)^{-T} (2 D),  dK = -lam U^T
//   dTheta through K = F F^T + Omega;  dZ = lam - (1+eta) D + dTheta W^T / sqrt(n)
//   E = M' D^T + dZ Z^T,  Psi = tril(E) + tril(E,-1)^T
//   pass-2 operands:  R_d = L^{-T} M' / sqrt(n),  R_z = L^{-T} dZ / sqrt(n),
//                     Q = L^{-T} Psi L^{-1} / n
// The QR-frame adjoint (top block of Q in QR([A/s; I/s])) reduces to
//   dA = (dP - P Psi) L^{-1},  dP = dY M'^T + C dZ^T,  dP^T P = E.
// ============================================================================
template <int R>
size_t solve_backward_smem() {
  return sizeof(float) * (5 * R * (R + 1) + 4 * R * (kColChunk + 1) + R);
}

template <int R>
__global__ void __launch_bounds__(kSolveThreads) solve_backward_kernel(const SolveBwdArgs a) {
  pdl_wait();
  constexpr int LD = R + 1, CLD = kColChunk + 1;
  extern __shared__ __align__(16) float fsm[];
  float* L = fsm;
  float* Mm = L + R * LD;
  float* Th = Mm + R * LD;
  float* dK = Th + R * LD;   // later dTheta
  float* E = dK + R * LD;
  float* X1 = E + R * LD;    // D chunk
  float* X2 = X1 + R * CLD;  // lambda chunk
  float* X3 = X2 + R * CLD;  // U chunk
  float* X4 = X3 + R * CLD;  // Z chunk
  float* fdiag = X4 + R * CLD;
  __shared__ float red[kSolveThreads / 32];
  const int tid = threadIdx.x;
  const int64_t bh = blockIdx.x;
  const int h = static_cast<int>(bh % a.H);
  const int d = a.d;
  const TapeLayout tl = tape_layout(a.N, R, d);
  const float* tape = a.tape + bh * a.tape_stride;
  const float n = tape[tl.n];
  const float rsn = 1.0f / sqrtf(n);
  const float eta = bounded_complement(a.eta_raw[h]);
  const int NC = a.dt;
  const int64_t pstride = static_cast<int64_t>(2 * R) * NC;
  const float* pbase = a.partial + bh * a.nchunks * a.ndt * pstride;
  float* Dg = a.dbuf + bh * static_cast<int64_t>(R) * d;
  float* Lg = a.lbuf + bh * static_cast<int64_t>(R) * d;
  const float* Wd = a.drive + static_cast<int64_t>(h) * d * R;

  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    L[i * LD + jj] = tape[tl.L + idx];
    Mm[i * LD + jj] = tape[tl.LU + idx];
    Th[i * LD + jj] = tape[tl.Theta + idx];
    dK[i * LD + jj] = 0.0f;
    E[i * LD + jj] = 0.0f;
  }
  __syncthreads();
  for (int i = tid; i < R; i += kSolveThreads) fdiag[i] = softplus20(Th[i * LD + i] + kSoftplusOneOffset);

  // Pass A: D, lambda, dK = -lam U^T, and <D, Z>.
  float dz_dot = 0.0f;
  for (int c0 = 0; c0 < d; c0 += kColChunk) {
    const int cw = min(kColChunk, d - c0);
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const int col = c0 + cc, jt = col / a.dt, cl = col % a.dt;
      float s = 0.0f;
      for (int ch = 0; ch < a.nchunks; ++ch) {
        const float* P = pbase + (static_cast<int64_t>(ch) * a.ndt + jt) * pstride;
        s += P[i * NC + cl] + P[(R + i) * NC + cl];
      }
      X1[i * CLD + cc] = s;
      X3[i * CLD + cc] = tape[tl.U + static_cast<int64_t>(i) * d + col];
      X4[i * CLD + cc] = tape[tl.Z + static_cast<int64_t>(i) * d + col];
    }
    __syncthreads();
    if (tid < cw) {
      forward_subst<R>(L, X1, tid);
      for (int i = 0; i < R; ++i) {
        const float dv = X1[i * CLD + tid] * rsn;
        X1[i * CLD + tid] = dv;
        X2[i * CLD + tid] = 2.0f * dv;
      }
      lu_solve_transposed<R>(Mm, X2, tid);
    }
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      Dg[static_cast<int64_t>(i) * d + c0 + cc] = X1[i * CLD + cc];
      Lg[static_cast<int64_t>(i) * d + c0 + cc] = X2[i * CLD + cc];
      dz_dot += X1[i * CLD + cc] * X4[i * CLD + cc];
    }
    for (int idx = tid; idx < R * R; idx += kSolveThreads) {
      const int i = idx / R, jj = idx % R;
      float s = 0.0f;
      for (int cc = 0; cc < cw; ++cc) s += X2[i * CLD + cc] * X3[jj * CLD + cc];
      dK[i * LD + jj] -= s;
    }
  }
  __syncthreads();
  // dTheta (into E temporarily, then back into dK) and its per-(b,h) base gradient.
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    float v;
    if (i < jj) {
      v = dK[i * LD + jj] - dK[jj * LD + i];
    } else {
      // dF[i][jj] = sum_k (dK + dK^T)[i][k] F[k][jj],  F[k][jj] != 0 for k >= jj
      float s = 0.0f;
      for (int k = jj; k < R; ++k) {
        const float f = k == jj ? fdiag[jj] : Th[k * LD + jj];
        s += (dK[i * LD + k] + dK[k * LD + i]) * f;
      }
      v = i == jj ? s * softplus20_derivative(Th[i * LD + i] + kSoftplusOneOffset) : s;
    }
    E[i * LD + jj] = v;
  }
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    dK[i * LD + jj] = E[i * LD + jj];
    E[i * LD + jj] = 0.0f;
    a.gbase[bh * R * R + idx] = dK[i * LD + jj];
  }
  __syncthreads();

  // Pass B: dZ, drive-gradient partial, E, and the pass-2 operands.
  uint8_t* b1y = reinterpret_cast<uint8_t*>(a.b1y + bh * R * a.d_pad);
  uint8_t* b1c = reinterpret_cast<uint8_t*>(a.b1c + bh * R * a.d_pad);
  uint8_t* b2 = reinterpret_cast<uint8_t*>(a.b2 + bh * a.d_pad * R);
  const uint32_t SBO_Y = static_cast<uint32_t>(a.d_pad) * 16;
  constexpr uint32_t SBO_R = R * 16;
  for (int c0 = 0; c0 < d; c0 += kColChunk) {
    const int cw = min(kColChunk, d - c0);
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const int64_t g = static_cast<int64_t>(i) * d + c0 + cc;
      X1[i * CLD + cc] = Dg[g];
      X2[i * CLD + cc] = Lg[g];
      X3[i * CLD + cc] = tape[tl.U + g];
      X4[i * CLD + cc] = tape[tl.Z + g];
    }
    __syncthreads();
    // X2 <- dZ,  X3 <- M' = 2U - (1+eta) Z
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const float* wrow = Wd + static_cast<int64_t>(c0 + cc) * R;
      float s = 0.0f;
      for (int jj = 0; jj < R; ++jj) s += dK[i * LD + jj] * wrow[jj];
      X2[i * CLD + cc] = X2[i * CLD + cc] - (1.0f + eta) * X1[i * CLD + cc] + s * rsn;
      X3[i * CLD + cc] = 2.0f * X3[i * CLD + cc] - (1.0f + eta) * X4[i * CLD + cc];
    }
    // drive-gradient partial: Z^T dTheta / sqrt(n)   ([d][R])
    for (int idx = tid; idx < cw * R; idx += kSolveThreads) {
      const int cc = idx / R, jj = idx % R;
      float s = 0.0f;
      for (int i = 0; i < R; ++i) s += X4[i * CLD + cc] * dK[i * LD + jj];
      a.gdrive[(bh * d + c0 + cc) * R + jj] = s * rsn;
    }
    __syncthreads();
    // E += M' D^T + dZ Z^T
    for (int idx = tid; idx < R * R; idx += kSolveThreads) {
      const int i = idx / R, k = idx % R;
      float s = 0.0f;
      for (int cc = 0; cc < cw; ++cc) s += X3[i * CLD + cc] * X1[k * CLD + cc] + X2[i * CLD + cc] * X4[k * CLD + cc];
      E[i * LD + k] += s;
    }
    __syncthreads();
    // R_d = L^{-T} M' / sqrt(n) (X3), R_z = L^{-T} dZ / sqrt(n) (X2)
    if (tid < cw) {
      backward_subst_transposed<R>(L, X3, tid);
    } else if (tid >= 128 && tid - 128 < cw) {
      backward_subst_transposed<R>(L, X2, tid - 128);
    }
    __syncthreads();
    for (int idx = tid; idx < R * cw; idx += kSolveThreads) {
      const int i = idx / cw, cc = idx % cw;
      const int col = c0 + cc;
      *reinterpret_cast<bf16*>(b1y + kmajor_offset(i, col, SBO_Y)) = __float2bfloat16_rn(X3[i * CLD + cc] * rsn);
      *reinterpret_cast<bf16*>(b1c + kmajor_offset(i, col, SBO_Y)) = __float2bfloat16_rn(X2[i * CLD + cc] * rsn);
      *reinterpret_cast<bf16*>(b2 + kmajor_offset(col, i, SBO_R)) = __float2bfloat16_rn(X2[i * CLD + cc] * rsn);
    }
  }
  // Zero the padded K columns of b1y/b1c and padded rows of b2.
  for (int idx = tid; idx < (a.d_pad - d) * R; idx += kSolveThreads) {
    const int col = d + idx / R, i = idx % R;
    const bf16 z = __float2bfloat16_rn(0.0f);
    *reinterpret_cast<bf16*>(b1y + kmajor_offset(i, col, SBO_Y)) = z;
    *reinterpret_cast<bf16*>(b1c + kmajor_offset(i, col, SBO_Y)) = z;
    *reinterpret_cast<bf16*>(b2 + kmajor_offset(col, i, SBO_R)) = z;
  }
  __syncthreads();
  // Q = L^{-T} Psi L^{-1} / n, Psi = tril(E) + tril(E,-1)^T.  Two column-wise
  // solves with L^T: X = L^{-T} Psi, then Q^T = L^{-T} X^T (Q symmetric).
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, k = idx % R;
    dK[i * LD + k] = i >= k ? E[i * LD + k] : E[k * LD + i];
  }
  __syncthreads();
  // column-wise L^{-T} on the R x R matrix in dK (thread per column)
  if (tid < R) {
    for (int i = R - 1; i >= 0; --i) {
      float z = dK[i * LD + tid];
      for (int k = i + 1; k < R; ++k) z -= L[k * LD + i] * dK[k * LD + tid];
      dK[i * LD + tid] = z / L[i * LD + i];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, k = idx % R;
    E[i * LD + k] = dK[k * LD + i];
  }
  __syncthreads();
  if (tid < R) {
    for (int i = R - 1; i >= 0; --i) {
      float z = E[i * LD + tid];
      for (int k = i + 1; k < R; ++k) z -= L[k * LD + i] * E[k * LD + tid];
      E[i * LD + tid] = z / L[i * LD + i];
    }
  }
  __syncthreads();
  // E now holds Q^T; B1a[n = i][k = j] = -Q[j][i] / n = -E[i][j] / n
  uint8_t* b1a = reinterpret_cast<uint8_t*>(a.b1a + bh * R * R);
  const float inv_n = rsn * rsn;
  for (int idx = tid; idx < R * R; idx += kSolveThreads) {
    const int i = idx / R, jj = idx % R;
    *reinterpret_cast<bf16*>(b1a + kmajor_offset(i, jj, SBO_R)) = __float2bfloat16_rn(-E[i * LD + jj] * inv_n);
  }
  // <D, Z> for the complement gradient
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dz_dot += __shfl_xor_sync(0xffffffffu, dz_dot, o);
  if ((tid & 31) == 0) red[tid >> 5] = dz_dot;
  __syncthreads();
  if (tid == 0) {
    float s = 0.0f;
    for (int wv = 0; wv < kSolveThreads / 32; ++wv) s += red[wv];
    a.etadot[bh] = s;
  }
}

// ============================================================================
// Gradient pass: per 128-token tile,
//   dA'[t] = dY[t] R_d^T + C[t] R_z^T - A'[t] Q / n      (D1, N = R)
//   dC[t]  = eta dY[t] + A'[t] R_z                      (D2, N = column block)
// then d relation = rotation^T(dA').  K runs over dY/C chunks of 32 columns
// plus the A' block.  The lead CTA (column block 0) also computes D1 and the
// complement statistic sum_t dY . C.
// ============================================================================
template <int R>
size_t grad_smem(int nb) {
  return static_cast<size_t>(kTokenTile) * 2 * kGradChunk * 2 +  // dY|C chunk
         2 * static_cast<size_t>(R) * kGradChunk * 2 +            // B1y, B1c chunks
         static_cast<size_t>(kTokenTile) * R * 2 +                 // A'
         static_cast<size_t>(R) * R * 2 +                          // B1a
         static_cast<size_t>(nb) * R * 2;                          // B2 block
}

template <int R>
__global__ void __launch_bounds__(128) grad_kernel(const GradArgs a) {
  pdl_wait();
  constexpr int RQ = R / 8;
  constexpr uint32_t SBO_R = R * 16;
  constexpr uint32_t SBO_C = 2 * kGradChunk * 16;  // dY|C chunk rows
  constexpr uint32_t SBO_BC = kGradChunk * 16;     // B1 chunk rows
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sAc = smem;
  uint8_t* sBy = sAc + kTokenTile * 2 * kGradChunk * 2;
  uint8_t* sBc = sBy + R * kGradChunk * 2;
  uint8_t* sAp = sBc + R * kGradChunk * 2;
  uint8_t* sBa = sAp + kTokenTile * R * 2;
  uint8_t* sB2 = sBa + R * R * 2;
  __shared__ __align__(8) uint64_t bars[3];  // [2]: teardown drain of the MMA thread
  __shared__ uint32_t tmem_s;
  __shared__ float red[4];

  int64_t blk = blockIdx.x;
  const int jd = static_cast<int>(blk % a.njd);
  blk /= a.njd;
  const int h = static_cast<int>(blk % a.H);
  blk /= a.H;
  const int tile = static_cast<int>(blk % a.ntiles);
  const int64_t b = blk / a.ntiles;
  const int64_t bh = b * a.H + h;
  const bool lead = jd == 0;
  const int tid = threadIdx.x;
  const int64_t pb = a.pos_batched ? b : 0;
  const bool vec = a.vec != 0;
  const int nb = min(a.nb, a.d_pad - jd * a.nb);
  const uint32_t tcols = tmem_cols_for(R + nb);
  const int64_t tok0 = static_cast<int64_t>(tile) * kTokenTile;
  const int d = a.d;
  const int d_pad = a.d_pad;

  if (tid == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    mbar_init(smem_u32(&bars[2]), 1);
    fence_mbar_init();
  }
  if (tid < 32) tmem_alloc(smem_u32(&tmem_s), tcols);

  // Operands shared by every column block: A' and the B2 block; the lead CTA
  // also needs B1a.
  {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.b2 + bh * d_pad * R) + static_cast<int64_t>(jd) * a.nb * R * 2;
    for (int idx = tid; idx < nb * R * 2 / 16; idx += 128) cp_async_16(smem_u32(sB2 + idx * 16), src + idx * 16, 16u);
    if (lead) {
      const uint8_t* s1 = reinterpret_cast<const uint8_t*>(a.b1a + bh * R * R);
      for (int idx = tid; idx < R * R * 2 / 16; idx += 128) cp_async_16(smem_u32(sBa + idx * 16), s1 + idx * 16, 16u);
    }
    cp_async_commit();
  }
  for (int idx = tid; idx < kTokenTile * RQ; idx += 128) {
    const int t = idx / RQ, q = idx % RQ;
    const int64_t tok = tok0 + t;
    uint4 rv = make_uint4(0u, 0u, 0u, 0u);
    Phase4 ph = phase_identity();
    if (tok < a.N) {
      rv = load8_bf16(a.proj + (b * a.N + tok) * a.W + static_cast<int64_t>(h) * R + 8 * q, 8, vec);
      ph = load_phase4(a.phase + ((pb * a.N + tok) * (R / 2) + 4 * q));
    }
    float v[8];
    rotate8(rv, ph, v);
    *reinterpret_cast<uint4*>(sAp + kmajor_offset(t, 8 * q, SBO_R)) = pack8_bf16(v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;
  const uint32_t idesc_r = make_idesc(128, R, false, false);

  bool ok = true;
  float stat = 0.0f;
  if (lead) {
    const int nkc = (d_pad + kGradChunk - 1) / kGradChunk;
    for (int kc = 0; kc < nkc; ++kc) {
      if (kc > 0 && ok) ok = mbar_wait(smem_u32(&bars[0]), (kc - 1) & 1, a.status);
      ok = __syncthreads_and(ok);
      const int k0 = kc * kGradChunk;
      const int w = min(kGradChunk, d_pad - k0);
      const int WQ = w / 8;
      // dY and C columns [k0, k0 + w): dY -> core columns [0, w/8), C -> [4, 4 + w/8)
      for (int idx = tid; idx < kTokenTile * WQ; idx += 128) {
        const int t = idx / WQ, g = idx % WQ;
        const int64_t tok = tok0 + t;
        const int col = k0 + 8 * g;
        const int cnt = min(8, d - col);
        uint4 yv = make_uint4(0u, 0u, 0u, 0u), cv = make_uint4(0u, 0u, 0u, 0u);
        if (tok < a.N && cnt > 0) {
          yv = load8_bf16(a.gout + (b * a.N + tok) * a.D + static_cast<int64_t>(h) * d + col, cnt, vec);
          cv = load8_bf16(a.proj + (b * a.N + tok) * a.W + static_cast<int64_t>(a.H) * R + static_cast<int64_t>(h) * d + col,
                          cnt, vec);
          const uint32_t yy[4] = {yv.x, yv.y, yv.z, yv.w}, ccv[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 y2 = unpack_bf16(yy[e]), c2 = unpack_bf16(ccv[e]);
            stat = fmaf(y2.x, c2.x, stat);
            stat = fmaf(y2.y, c2.y, stat);
          }
        }
        *reinterpret_cast<uint4*>(sAc + kmajor_offset(t, 8 * g, SBO_C)) = yv;
        *reinterpret_cast<uint4*>(sAc + kmajor_offset(t, kGradChunk + 8 * g, SBO_C)) = cv;
      }
      // B1y / B1c column chunks: rows i, K columns [k0, k0 + w)
      {
        const uint8_t* sy = reinterpret_cast<const uint8_t*>(a.b1y + bh * R * d_pad);
        const uint8_t* sc = reinterpret_cast<const uint8_t*>(a.b1c + bh * R * d_pad);
        const int per_row = w * 16 / 16;  // 16-byte pieces per 8-row group: w/8 cores of 128 B
        for (int idx = tid; idx < RQ * per_row; idx += 128) {
          const int ig = idx / per_row, piece = idx % per_row;
          const int64_t goff = static_cast<int64_t>(ig) * d_pad * 16 + static_cast<int64_t>(k0) * 16 + piece * 16;
          const int soff = ig * SBO_BC + piece * 16;
          cp_async_16(smem_u32(sBy + soff), sy + goff, 16u);
          cp_async_16(smem_u32(sBc + soff), sc + goff, 16u);
        }
        cp_async_commit();
      }
      cp_async_wait<0>();
      fence_proxy_async();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (tid == 0 && ok) {
        for (int s = 0; s < w / 16; ++s) {
          mma_bf16(tmem, make_desc(smem_u32(sAc) + s * 256, 128, SBO_C), make_desc(smem_u32(sBy) + s * 256, 128, SBO_BC),
                   idesc_r, (kc > 0 || s > 0) ? 1u : 0u);
        }
        for (int s = 0; s < w / 16; ++s) {
          mma_bf16(tmem, make_desc(smem_u32(sAc) + kGradChunk * 16 + s * 256, 128, SBO_C),
                   make_desc(smem_u32(sBc) + s * 256, 128, SBO_BC), idesc_r, 1u);
        }
        if (kc == nkc - 1) {
#pragma unroll
          for (int s = 0; s < R / 16; ++s) {
            mma_bf16(tmem, make_desc(smem_u32(sAp) + s * 256, 128, SBO_R), make_desc(smem_u32(sBa) + s * 256, 128, SBO_R),
                     idesc_r, 1u);
          }
        }
        mma_commit(smem_u32(&bars[0]));
      }
    }
  } else {
    cp_async_wait<0>();
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (tid == 0 && ok) {
    const uint32_t idesc_c = make_idesc(128, nb, false, false);
#pragma unroll
    for (int s = 0; s < R / 16; ++s) {
      mma_bf16(tmem + R, make_desc(smem_u32(sAp) + s * 256, 128, SBO_R), make_desc(smem_u32(sB2) + s * 256, 128, SBO_R),
               idesc_c, s > 0 ? 1u : 0u);
    }
    mma_commit(smem_u32(&bars[1]));
  }
  const float eta = bounded_complement(a.eta_raw[h]);
  if (ok) ok = mbar_wait(smem_u32(&bars[1]), 0, a.status);
  if (ok && lead) ok = mbar_wait(smem_u32(&bars[0]), ((d_pad + kGradChunk - 1) / kGradChunk - 1) & 1, a.status);
  ok = __syncthreads_and(ok);
  tc_fence_after();

  const int w = tid >> 5, lane = tid & 31;
  const int t = 32 * w + lane;
  const int64_t tok = tok0 + t;
  const bool live = tok < a.N;
  const int64_t row = b * a.N + (live ? tok : 0);
  bf16* grow = a.gproj + row * a.W;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * w) << 16);
  if (ok && lead) {
    for (int r0 = 0; r0 < R; r0 += 8) {
      float g[8], out[8];
      tmem_ld8(lane_addr + r0, g);
      tmem_ld_wait();
      const Phase4 ph = live ? load_phase4(a.phase + ((pb * a.N + tok) * (R / 2) + r0 / 2)) : phase_identity();
      rotate8_transpose(g, ph, out);
      if (live) store8_bf16(grow + static_cast<int64_t>(h) * R + r0, out, 8, vec);
    }
  }
  if (ok) {
    const bf16* yrow = a.gout + row * a.D + static_cast<int64_t>(h) * d;
    bf16* crow = grow + static_cast<int64_t>(a.H) * R + static_cast<int64_t>(h) * d;
    for (int c0 = 0; c0 < nb; c0 += 8) {
      float v[8];
      tmem_ld8(lane_addr + R + c0, v);
      tmem_ld_wait();
      const int col = jd * a.nb + c0;
      const int cnt = min(8, d - col);
      if (live && cnt > 0) {
        const uint4 yv = load8_bf16(yrow + col, cnt, vec);
        const float2 y01 = unpack_bf16(yv.x), y23 = unpack_bf16(yv.y), y45 = unpack_bf16(yv.z), y67 = unpack_bf16(yv.w);
        float o[8] = {fmaf(eta, y01.x, v[0]), fmaf(eta, y01.y, v[1]), fmaf(eta, y23.x, v[2]), fmaf(eta, y23.y, v[3]),
                      fmaf(eta, y45.x, v[4]), fmaf(eta, y45.y, v[5]), fmaf(eta, y67.x, v[6]), fmaf(eta, y67.y, v[7])};
        store8_bf16(crow + col, o, cnt, vec);
      }
    }
  }
  if (lead) {
    const float s = block_sum_128(stat, red);
    if (tid == 0) a.etastat[bh * a.ntiles + tile] = s;
  }
  if (tid == 0) mma_drain(smem_u32(&bars[2]), a.status);  // tid 0 issued the MMAs
  tc_fence_before();
  __syncthreads();
  if (tid < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

// ============================================================================
// Parameter gradients: deterministic sums over samples (ascending b).
// ============================================================================
constexpr int kReduceThreads = 256;

// Blocks [0, main_blocks) sum the base/drive partials over samples, four
// lanes per element; the last H blocks each reduce one head's complement
// statistic over (sample, tile) with a fixed-order tree.  Deterministic.
constexpr int kReduceLanes = 4;
__global__ void __launch_bounds__(kReduceThreads) param_reduce_kernel(const ParamReduceArgs a) {
  pdl_wait();
  const int64_t R = a.R, d = a.d, H = a.H;
  const int64_t nbase = H * R * R, nmain = nbase + H * d * R;
  const int64_t main_blocks = (nmain * kReduceLanes + kReduceThreads - 1) / kReduceThreads;
  if (static_cast<int64_t>(blockIdx.x) < main_blocks) {
    // Sixteen partial sums per element (sample b goes to sum b % 16, ascending
    // b), combined by the pairwise tree acc[j] += acc[j + w], w = 8, 4, 2, 1.
    // Lane l of the element's four holds sums 4l .. 4l+3 (all their loads in
    // flight at once); the tree's first two levels cross lanes by shuffles, so
    // every addition happens in the same order as in one thread.
    const int64_t t = static_cast<int64_t>(blockIdx.x) * kReduceThreads + threadIdx.x;
    const int64_t idx = t / kReduceLanes;
    const int l = static_cast<int>(t % kReduceLanes);
    const bool live = idx < nmain;  // whole groups of four share this
    const bool is_base = idx < nbase;
    const int64_t k = live ? (is_base ? idx : idx - nbase) : 0;
    const int64_t per = is_base ? R * R : d * R;
    const int64_t h = k / per, e = k % per;
    const float* src = (is_base ? a.gbase : a.gdrive) + h * per + e;
    const int64_t stride = H * per;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (live) {
#pragma unroll 4
      for (int64_t b0 = 0; b0 < a.B; b0 += 16) {
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t b = b0 + 4 * l + u;
          v[u] = b < a.B ? __ldg(src + b * stride) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (b0 + 4 * l + u < a.B) acc[u] += v[u];
      }
    }
    float o[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) o[u] = __shfl_down_sync(0xffffffffu, acc[u], 2, kReduceLanes);
    if (l < 2) {
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += o[u];  // w = 8: sums 4l+u and 4(l+2)+u
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) o[u] = __shfl_down_sync(0xffffffffu, acc[u], 1, kReduceLanes);
    if (l != 0 || !live) return;
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] += o[u];  // w = 4: sums u and 4 + u
    acc[0] += acc[2];                              // w = 2
    acc[1] += acc[3];
    const float total = acc[0] + acc[1];           // w = 1
    if (is_base) {
      a.grad_base[k] = total;
    } else {
      a.grad_drive[k] = total;
    }
    return;
  }
  __shared__ float part[kReduceThreads];
  const int64_t h = static_cast<int64_t>(blockIdx.x) - main_blocks;
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < a.B * a.ntiles; i += kReduceThreads) {
    const int64_t b = i / a.ntiles, t = i % a.ntiles;
    s += a.etastat[(b * H + h) * a.ntiles + t];
  }
  for (int64_t b = threadIdx.x; b < a.B; b += kReduceThreads) s -= a.etadot[b * H + h];
  part[threadIdx.x] = s;
  __syncthreads();
  for (int w = kReduceThreads / 2; w > 0; w >>= 1) {
    if (static_cast<int>(threadIdx.x) < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) a.grad_eta[h] = part[0] * bounded_complement_derivative(a.eta_raw[h]);
}

// x *= w over the three per-(b, h) buffers the solve writes for the parameter
// gradients (concatenated index space).
__global__ void param_scale_kernel(float* __restrict__ g0, int64_t n0, float* __restrict__ g1, int64_t n1,
                                   float* __restrict__ g2, int64_t n2, float w) {
  pdl_wait();
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n0) {
    g0[i] *= w;
    return;
  }
  i -= n0;
  if (i < n1) {
    g1[i] *= w;
    return;
  }
  i -= n1;
  if (i < n2) g2[i] *= w;
}

// ============================================================================
// Launchers
// ============================================================================
LaunchHook g_before_launch = nullptr;
LaunchHook g_after_launch = nullptr;

cudaError_t allow_smem(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  struct Entry {
    int device;
    const void* fn;
    size_t bytes;
  };
  static std::mutex lock;
  static std::vector<Entry> done;
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> guard(lock);
  for (const Entry& x : done) {
    if (x.device == device && x.fn == fn && x.bytes >= bytes) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return e;
  for (Entry& x : done) {
    if (x.device == device && x.fn == fn) {
      x.bytes = bytes;
      return cudaSuccess;
    }
  }
  done.push_back({device, fn, bytes});
  return cudaSuccess;
}

static cudaError_t set_smem(const void* fn, size_t bytes) { return allow_smem(fn, bytes); }

static InvFreq inverse_frequencies(int R) {
  InvFreq f{};
  const int half = R / 2;
  for (int k = 0; k < half; ++k) {
    // 10000^(-k/half) evaluated in FP32 like the reference's inv_freq tensor.
    const float e = -static_cast<float>(k) / static_cast<float>(half);
    f.v[k] = powf(10000.0f, e);
  }
  return f;
}

static cudaError_t launch_phase(const Plan& p, const float* pos, float2* table, __half2* table16,
                                cudaStream_t stream) {
  const int half = static_cast<int>(p.R / 2);
  const int threads = 256;
  const dim3 grid(static_cast<unsigned>(ceil_div(p.N * half, threads)),
                  static_cast<unsigned>(p.pos_rows < 65535 ? p.pos_rows : 65535));
  LaunchScope scope("phase", stream);
  launch_pdl(phase_kernel, grid, threads, 0, stream, pos, p.pos_rows, static_cast<int>(p.N), half,
                                             inverse_frequencies(static_cast<int>(p.R)), table, table16);
  return cudaGetLastError();
}

template <int R, bool BWD>
static cudaError_t launch_moments(const Plan& p, MomentArgs args, cudaStream_t stream) {
  constexpr int M_PAD = (2 * R <= 64) ? 64 : 128;
  const size_t smem = static_cast<size_t>(2 * M_PAD * kMomentTile * 2 + 3 * kMomentTile * R * 2 +
                                          3 * static_cast<int>(p.dt) * kMomentTile * 2);
  cudaError_t e = set_smem(reinterpret_cast<const void*>(&moments_kernel<R, BWD>), smem);
  if (e != cudaSuccess) return e;
  const int64_t grid = p.BH * p.nchunks * p.ndt;
  LaunchScope scope(BWD ? "moments_bwd" : "moments_fwd", stream);
  launch_pdl(moments_kernel<R, BWD>, static_cast<unsigned>(grid), 128, smem, stream, args);
  return cudaGetLastError();
}

// Phase table and the forward moment pass (chunk partials into fb.partial).
template <int R>
static cudaError_t forward_moments_r(const Plan& p, const ForwardBuffers& fb, cudaStream_t stream) {
  cudaError_t e = launch_phase(p, fb.positions, fb.phase, fb.phase16, stream);
  if (e != cudaSuccess) return e;
  MomentArgs m{};
  m.proj = fb.projected;
  m.vsrc = fb.projected;
  m.phase = fb.phase;
  m.partial = fb.partial;
  m.status = fb.status;
  m.N = p.N;
  m.W = p.W;
  m.v_stride = p.W;
  m.v_col0 = p.H * p.R;
  m.H = static_cast<int>(p.H);
  m.d = static_cast<int>(p.d);
  m.dt = static_cast<int>(p.dt);
  m.ndt = static_cast<int>(p.ndt);
  m.nchunks = static_cast<int>(p.nchunks);
  m.chunk_len = static_cast<int>(p.chunk_len);
  m.pos_batched = p.pos_rows > 1 ? 1 : 0;
  m.vec = fb.vec;
  if (tiled_usable(p, {fb.projected})) {
    return launch_moments_tiled(p, false, fb.projected, nullptr, fb.phase16, fb.partial, fb.status, p.sms, stream);
  }
  return launch_moments<R, false>(p, m, stream);
}

// Solves (over `nchunks` partials per (b, h)) and the readout; the phase table
// is already in fb.phase.
template <int R>
static cudaError_t forward_finish_r(const Plan& p, const ForwardBuffers& fb, const float* partial, int64_t nchunks,
                                    cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  SolveFwdArgs s{};
  s.partial = partial;
  s.base = fb.base;
  s.drive = fb.drive;
  s.eta_raw = fb.eta_raw;
  s.counts = fb.counts;
  s.zbuf = fb.zbuf;
  s.rmat = fb.rmat;
  s.tape = fb.tape;
  s.pivots = fb.pivots;
  s.N = p.N;
  s.tape_stride = p.tape_stride;
  s.H = static_cast<int>(p.H);
  s.d = static_cast<int>(p.d);
  s.d_pad = static_cast<int>(p.d_pad);
  s.dt = static_cast<int>(p.dt);
  s.ndt = static_cast<int>(p.ndt);
  s.nchunks = static_cast<int>(nchunks);
  if (warp_solves_usable(p)) {
    e = launch_solve_forward_warp(p, s, stream);
  } else {
    const size_t ssm = solve_forward_smem<R>();
    e = set_smem(reinterpret_cast<const void*>(&solve_forward_kernel<R>), ssm);
    if (e != cudaSuccess) return e;
    LaunchScope scope("solve_fwd", stream);
    launch_pdl(solve_forward_kernel<R>, static_cast<unsigned>(p.BH), kSolveThreads, ssm, stream, s);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;

  ReadoutArgs r{};
  r.proj = fb.projected;
  r.phase = fb.phase;
  r.rmat = fb.rmat;
  r.eta_raw = fb.eta_raw;
  r.out = fb.mixed;
  r.status = fb.status;
  r.N = p.N;
  r.W = p.W;
  r.out_stride = p.D;
  r.H = static_cast<int>(p.H);
  r.d = static_cast<int>(p.d);
  r.d_pad = static_cast<int>(p.d_pad);
  r.nb = static_cast<int>(p.nb);
  r.njd = static_cast<int>(p.njd);
  r.ntiles = static_cast<int>(p.ntiles);
  r.pos_batched = p.pos_rows > 1 ? 1 : 0;
  r.vec = fb.vec;
  if (tiled_usable(p, {fb.projected, fb.mixed})) {
    return launch_readout_tiled(p, fb.projected, fb.phase16, fb.rmat, fb.eta_raw, fb.mixed, fb.status, p.sms,
                                stream);
  }
  const size_t rsm = readout_smem<R>(static_cast<int>(p.nb));
  e = set_smem(reinterpret_cast<const void*>(&readout_kernel<R>), rsm);
  if (e != cudaSuccess) return e;
  LaunchScope scope("readout", stream);
  launch_pdl(readout_kernel<R>, static_cast<unsigned>(p.B * p.ntiles * p.H * p.njd), 128, rsm, stream, r);
  return cudaGetLastError();
}

template <int R>
static cudaError_t forward_r(const Plan& p, const ForwardBuffers& fb, cudaStream_t stream) {
  const cudaError_t e = forward_moments_r<R>(p, fb, stream);
  if (e != cudaSuccess) return e;
  return forward_finish_r<R>(p, fb, fb.partial, p.nchunks, stream);
}

// Phase tables and the backward moment pass (chunk partials into bb.partial).
template <int R>
static cudaError_t backward_moments_r(const Plan& p, const BackwardBuffers& bb, cudaStream_t stream) {
  cudaError_t e = launch_phase(p, bb.positions, bb.phase, bb.phase16, stream);
  if (e != cudaSuccess) return e;
  const int pos_batched = p.pos_rows > 1 ? 1 : 0;
  MomentArgs m{};
  m.proj = bb.projected;
  m.vsrc = bb.grad_output;
  m.phase = bb.phase;
  m.partial = bb.partial;
  m.status = bb.status;
  m.N = p.N;
  m.W = p.W;
  m.v_stride = p.D;
  m.v_col0 = 0;
  m.H = static_cast<int>(p.H);
  m.d = static_cast<int>(p.d);
  m.dt = static_cast<int>(p.dt);
  m.ndt = static_cast<int>(p.ndt);
  m.nchunks = static_cast<int>(p.nchunks);
  m.chunk_len = static_cast<int>(p.chunk_len);
  m.pos_batched = pos_batched;
  m.vec = bb.vec;
  if (tiled_usable(p, {bb.projected, bb.grad_output})) {
    return launch_moments_tiled(p, true, bb.projected, bb.grad_output, bb.phase16, bb.partial, bb.status, p.sms,
                                stream);
  }
  return launch_moments<R, true>(p, m, stream);
}

// Backward solves (over `nchunks` partials per (b, h)), the gradient pass and
// the parameter reduction; the phase tables are already in bb.
template <int R>
static SolveBwdArgs solve_backward_args(const Plan& p, const BackwardBuffers& bb, const float* partial,
                                        int64_t nchunks) {
  SolveBwdArgs s{};
  s.partial = partial;
  s.tape = bb.tape;
  s.drive = bb.drive;
  s.eta_raw = bb.eta_raw;
  s.dbuf = bb.dbuf;
  s.lbuf = bb.lbuf;
  s.b1y = bb.b1y;
  s.b1c = bb.b1c;
  s.b1a = bb.b1a;
  s.b2 = bb.b2;
  s.gbase = bb.gbase;
  s.gdrive = bb.gdrive;
  s.etadot = bb.etadot;
  s.N = p.N;
  s.tape_stride = p.tape_stride;
  s.H = static_cast<int>(p.H);
  s.d = static_cast<int>(p.d);
  s.d_pad = static_cast<int>(p.d_pad);
  s.dt = static_cast<int>(p.dt);
  s.ndt = static_cast<int>(p.ndt);
  s.nchunks = static_cast<int>(nchunks);
  return s;
}

// The backward solves: per (b, h) adjoint solves, parameter-gradient partials
// and the gradient pass's operand matrices.
template <int R>
static cudaError_t backward_solve_r(const Plan& p, const BackwardBuffers& bb, const float* partial, int64_t nchunks,
                                    cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  const SolveBwdArgs s = solve_backward_args<R>(p, bb, partial, nchunks);
  if (warp_solves_usable(p)) {
    e = launch_solve_backward_warp(p, s, stream);
  } else {
    const size_t ssm = solve_backward_smem<R>();
    e = set_smem(reinterpret_cast<const void*>(&solve_backward_kernel<R>), ssm);
    if (e != cudaSuccess) return e;
    LaunchScope scope("solve_bwd", stream);
    launch_pdl(solve_backward_kernel<R>, static_cast<unsigned>(p.BH), kSolveThreads, ssm, stream, s);
    e = cudaGetLastError();
  }
  return e;
}

// The gradient pass and the parameter reduction (after the backward solves).
template <int R>
static cudaError_t backward_grads_r(const Plan& p, const BackwardBuffers& bb, float redundant, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  const int pos_batched = p.pos_rows > 1 ? 1 : 0;
  GradArgs g{};
  g.gout = bb.grad_output;
  g.proj = bb.projected;
  g.phase = bb.phase;
  g.b1y = bb.b1y;
  g.b1c = bb.b1c;
  g.b1a = bb.b1a;
  g.b2 = bb.b2;
  g.eta_raw = bb.eta_raw;
  g.gproj = bb.grad_projected;
  g.etastat = bb.etastat;
  g.status = bb.status;
  g.N = p.N;
  g.W = p.W;
  g.D = p.D;
  g.H = static_cast<int>(p.H);
  g.d = static_cast<int>(p.d);
  g.d_pad = static_cast<int>(p.d_pad);
  g.nb = static_cast<int>(p.nb);
  g.njd = static_cast<int>(p.njd);
  g.ntiles = static_cast<int>(p.ntiles);
  g.pos_batched = pos_batched;
  g.vec = bb.vec;
  if (p.tiled_grad && tiled_usable(p, {bb.projected, bb.grad_output, bb.grad_projected})) {
    e = launch_grad_tiled(p, bb.grad_output, bb.projected, bb.phase16, bb.b1y, bb.b1c, bb.b1a, bb.eta_raw,
                          bb.grad_projected, bb.etastat, bb.status, p.sms, stream);
  } else {
    const size_t gsm = grad_smem<R>(static_cast<int>(p.nb));
    e = set_smem(reinterpret_cast<const void*>(&grad_kernel<R>), gsm);
    if (e != cudaSuccess) return e;
    LaunchScope scope("grad", stream);
    launch_pdl(grad_kernel<R>, static_cast<unsigned>(p.B * p.ntiles * p.H * p.njd), 128, gsm, stream, g);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;

  ParamReduceArgs pr{};
  pr.gbase = bb.gbase;
  pr.gdrive = bb.gdrive;
  pr.etastat = bb.etastat;
  pr.etadot = bb.etadot;
  pr.eta_raw = bb.eta_raw;
  pr.grad_base = bb.grad_base;
  pr.grad_drive = bb.grad_drive;
  pr.grad_eta = bb.grad_eta;
  pr.B = p.B;
  pr.H = p.H;
  pr.R = p.R;
  pr.d = p.d;
  pr.ntiles = p.ntiles;
  if (redundant != 1.0f) {
    // Sequence-parallel ranks: weight the solve-computed terms before they are reduced.
    const int64_t n = p.BH * (p.R * p.R + p.d * p.R + 1);
    LaunchScope scope("param_scale", stream);
    launch_pdl(param_scale_kernel, static_cast<unsigned>(ceil_div(n, kReduceThreads)), kReduceThreads, 0, stream, 
        bb.gbase, p.BH * p.R * p.R, bb.gdrive, p.BH * p.d * p.R, bb.etadot, p.BH, redundant);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const int64_t main_blocks = ceil_div((p.H * p.R * p.R + p.H * p.d * p.R) * kReduceLanes, kReduceThreads);
  LaunchScope scope("param_reduce", stream);
  launch_pdl(param_reduce_kernel, static_cast<unsigned>(main_blocks + p.H), kReduceThreads, 0, stream, pr);
  return cudaGetLastError();
}

// Backward solves (over `nchunks` partials per (b, h)), the gradient pass and
// the parameter reduction; the phase tables are already in bb.
template <int R>
static cudaError_t backward_finish_r(const Plan& p, const BackwardBuffers& bb, const float* partial, int64_t nchunks,
                                     float redundant, cudaStream_t stream) {
  const cudaError_t e = backward_solve_r<R>(p, bb, partial, nchunks, stream);
  if (e != cudaSuccess) return e;
  return backward_grads_r<R>(p, bb, redundant, stream);
}

template <int R>
static cudaError_t backward_r(const Plan& p, const BackwardBuffers& bb, cudaStream_t stream) {
  const cudaError_t e = backward_moments_r<R>(p, bb, stream);
  if (e != cudaSuccess) return e;
  return backward_finish_r<R>(p, bb, bb.partial, p.nchunks, 1.0f, stream);
}

template <int R>
static cudaError_t backward_with_wgrad_r(const Plan& p, const BackwardBuffers& bb, const WgradPlan& wp,
                                         const WgradCall& wc, int solve_ctas, const SideStream& side,
                                         cudaStream_t stream) {
  cudaError_t e = backward_moments_r<R>(p, bb, stream);
  if (e != cudaSuccess) return e;
  if (solve_ctas <= 0) {
    e = backward_solve_r<R>(p, bb, bb.partial, p.nchunks, stream);
    if (e == cudaSuccess) e = launch_wgrad(wp, wc, stream);
    if (e != cudaSuccess) return e;
    return backward_grads_r<R>(p, bb, 1.0f, stream);
  }
  // fork: the solves on the side stream, the weight gradient on this one; join before the gradient pass
  e = cudaEventRecord(side.fork, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(side.stream, side.fork, 0);
  if (e != cudaSuccess) return e;
  const SolveBwdArgs s = solve_backward_args<R>(p, bb, bb.partial, p.nchunks);
  e = launch_solve_backward_persistent(p, s, solve_ctas * p.sms, side.stream);
  if (e == cudaSuccess) e = cudaEventRecord(side.join, side.stream);
  if (e != cudaSuccess) return e;
  e = launch_wgrad(wp, wc, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, side.join, 0);
  if (e != cudaSuccess) return e;
  return backward_grads_r<R>(p, bb, 1.0f, stream);
}

// Sum of the chunk partials of every (b, h): out[bh][e] = sum_ch partial[bh][ch][e]
// (ascending chunks), float4 per thread.
__global__ void chunk_sum_kernel(const float4* __restrict__ partial, int64_t BH, int nchunks, int64_t per4,
                                 float4* __restrict__ out) {
  pdl_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= BH * per4) return;
  const int64_t bh = i / per4, e = i - bh * per4;
  const float4* src = partial + bh * nchunks * per4 + e;
  float4 acc = src[0];
  for (int ch = 1; ch < nchunks; ++ch) {
    const float4 v = src[ch * per4];
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  out[i] = acc;
}

static cudaError_t sum_chunks(const Plan& p, bool bwd, const float* partial, float* moments, cudaStream_t stream) {
  const int64_t per = moment_elements(p, bwd) / p.BH;  // a multiple of 4 (R and dt are multiples of 16)
  const int64_t total4 = p.BH * per / 4;
  LaunchScope scope("chunk_sum", stream);
  launch_pdl(chunk_sum_kernel, static_cast<unsigned>(ceil_div(total4, 256)), 256, 0, stream, 
      reinterpret_cast<const float4*>(partial), p.BH, static_cast<int>(p.nchunks), per / 4,
      reinterpret_cast<float4*>(moments));
  return cudaGetLastError();
}

int64_t moment_elements(const Plan& p, bool bwd) {
  return p.BH * p.ndt * 2 * p.R * ((bwd ? 0 : p.R) + p.dt);
}

cudaError_t launch_forward_moments(const Plan& p, const ForwardBuffers& fb, float* moments, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  switch (p.R) {
    case 16: e = forward_moments_r<16>(p, fb, stream); break;
    case 32: e = forward_moments_r<32>(p, fb, stream); break;
    case 48: e = forward_moments_r<48>(p, fb, stream); break;
    case 64: e = forward_moments_r<64>(p, fb, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  return sum_chunks(p, false, fb.partial, moments, stream);
}

cudaError_t launch_forward_finish(const Plan& p, const ForwardBuffers& fb, const float* moments, cudaStream_t stream) {
  const cudaError_t e = launch_phase(p, fb.positions, fb.phase, fb.phase16, stream);
  if (e != cudaSuccess) return e;
  switch (p.R) {
    case 16: return forward_finish_r<16>(p, fb, moments, 1, stream);
    case 32: return forward_finish_r<32>(p, fb, moments, 1, stream);
    case 48: return forward_finish_r<48>(p, fb, moments, 1, stream);
    case 64: return forward_finish_r<64>(p, fb, moments, 1, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_backward_moments(const Plan& p, const BackwardBuffers& bb, float* moments, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  switch (p.R) {
    case 16: e = backward_moments_r<16>(p, bb, stream); break;
    case 32: e = backward_moments_r<32>(p, bb, stream); break;
    case 48: e = backward_moments_r<48>(p, bb, stream); break;
    case 64: e = backward_moments_r<64>(p, bb, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  return sum_chunks(p, true, bb.partial, moments, stream);
}

cudaError_t launch_backward_finish(const Plan& p, const BackwardBuffers& bb, const float* moments, float redundant,
                                   cudaStream_t stream) {
  const cudaError_t e = launch_phase(p, bb.positions, bb.phase, bb.phase16, stream);
  if (e != cudaSuccess) return e;
  switch (p.R) {
    case 16: return backward_finish_r<16>(p, bb, moments, 1, redundant, stream);
    case 32: return backward_finish_r<32>(p, bb, moments, 1, redundant, stream);
    case 48: return backward_finish_r<48>(p, bb, moments, 1, redundant, stream);
    case 64: return backward_finish_r<64>(p, bb, moments, 1, redundant, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_forward(const Plan& p, const ForwardBuffers& fb, cudaStream_t stream) {
  switch (p.R) {
    case 16: return forward_r<16>(p, fb, stream);
    case 32: return forward_r<32>(p, fb, stream);
    case 48: return forward_r<48>(p, fb, stream);
    case 64: return forward_r<64>(p, fb, stream);
    default: return cudaErrorInvalidValue;
  }
}

int solve_ctas_beside(const Plan& p, const WgradPlan& wp, int device) {
  if (!warp_solves_usable(p) || !p.tiled) return 0;
  const CtaFootprint fs = solve_backward_footprint(p);
  const CtaFootprint fw = wgrad_footprint(wp);
  if (fs.threads == 0 || fw.threads == 0) return 0;
  int regs = 0, smem = 0, reserved = 0, threads = 0;
  if (cudaDeviceGetAttribute(&regs, cudaDevAttrMaxRegistersPerMultiprocessor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&threads, cudaDevAttrMaxThreadsPerMultiProcessor, device) != cudaSuccess) {
    return 0;
  }
  // registers are allocated per warp in units of 256
  auto cta_regs = [](const CtaFootprint& f) { return (f.regs * 32 + 255) / 256 * 256 * (f.threads / 32); };
  // Two solve CTAs per SM beside the GEMM, and at most one round of systems more than the solve
  // launched alone takes in waves: a solve CTA's time hardly shrinks with fewer CTAs per SM, so
  // with one CTA per SM (rank 48) the concurrent form measured slower (2.015 -> 2.051 ms per step).
  const int k = 2;
  const bool fit = cta_regs(fw) + k * cta_regs(fs) <= regs &&
                   fw.smem + reserved + k * (fs.smem + reserved) <= static_cast<size_t>(smem) &&
                   fw.threads + k * fs.threads <= threads;
  if (!fit) return 0;
  int alone = 32;  // solve CTAs per SM without the GEMM
  alone = std::min(alone, regs / std::max(1, cta_regs(fs)));
  alone = std::min(alone, static_cast<int>(static_cast<size_t>(smem) / (fs.smem + reserved)));
  alone = std::min(alone, threads / fs.threads);
  if (alone < 1) return 0;
  const int64_t waves = ceil_div(p.BH, static_cast<int64_t>(alone) * p.sms);
  const int64_t rounds = ceil_div(p.BH, static_cast<int64_t>(k) * p.sms);
  return rounds <= waves + 1 ? k : 0;
}

cudaError_t launch_backward_with_wgrad(const Plan& p, const BackwardBuffers& bb, const WgradPlan& wp,
                                       const WgradCall& wc, int solve_ctas, const SideStream& side,
                                       cudaStream_t stream) {
  switch (p.R) {
    case 16: return backward_with_wgrad_r<16>(p, bb, wp, wc, solve_ctas, side, stream);
    case 32: return backward_with_wgrad_r<32>(p, bb, wp, wc, solve_ctas, side, stream);
    case 48: return backward_with_wgrad_r<48>(p, bb, wp, wc, solve_ctas, side, stream);
    case 64: return backward_with_wgrad_r<64>(p, bb, wp, wc, solve_ctas, side, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_backward(const Plan& p, const BackwardBuffers& bb, cudaStream_t stream) {
  switch (p.R) {
    case 16: return backward_r<16>(p, bb, stream);
    case 32: return backward_r<32>(p, bb, stream);
    case 48: return backward_r<48>(p, bb, stream);
    case 64: return backward_r<64>(p, bb, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace lsso
