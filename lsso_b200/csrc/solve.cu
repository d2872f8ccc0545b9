// Per-(sample, head) r x r solves of the LSSO mixer for R <= 32 (sm_100a).
//
// Same algebra as solve_forward_kernel / solve_backward_kernel in mixer.cu
// (reference lsso/ball/reference.py:411-572): Cholesky of the Gram matrix,
// the accretive generator, LU without pivoting, and the triangular solves of
// the forward and the analytic backward.  The difference is the execution
// model: with R <= 32 one lane owns one matrix row, so
//   - Cholesky and LU are R steps in one warp: the pivot row or column is
//     broadcast (shuffle or same-address shared read) and every lane updates
//     its own row with independent fused multiply-adds;
//   - a triangular solve is R shuffle steps per right-hand side, four
//     right-hand sides per warp at a time for instruction-level parallelism,
//     replacing a thread-per-column R^2 chain; transposed solves read the
//     matrix by columns (one column view of the packed LU serves both U^T and
//     the unit L^T);
//   - all d columns of the R x d operands stay in shared memory, split over
//     the CTA's warps.
// One CTA (four warps) per (sample, head).
#include "mixer.h"
#include "mixer_common.cuh"

namespace lsso {

namespace {

constexpr int kWThreads = 256;
constexpr int kWWarps = kWThreads / 32;
constexpr int kNB = 4;  // right-hand sides per warp-level solve
constexpr unsigned kFull = 0xffffffffu;

// Matrices stay in shared memory; lane i works on row i.  The step loops are
// kept rolled (unroll 2) so the code stays small: these kernels run once per
// (sample, head), and fully unrolled R = 32 chains overflow the instruction
// cache.  A matrix element (row, k) is read at M[row * rs + k * cs]: rs = ld,
// cs = 1 for the matrix itself, rs = 1, cs = ld for its transpose.

// Lower-triangular solve T x = b (lane i: b_i in b[q]); rdiag = 1 / T_ii on
// lane i (ignored when UNIT).
template <int R, bool UNIT>
__device__ __forceinline__ void trsv_lower(const float* M, int rs, int cs, float rdiag, float (&b)[kNB]) {
  const int lane = threadIdx.x & 31;
  const float* row = M + (lane < R ? lane : 0) * rs;
#pragma unroll 2
  for (int k = 0; k < R; ++k) {
    const float tk = lane < R ? row[k * cs] : 0.0f;
#pragma unroll
    for (int q = 0; q < kNB; ++q) {
      const float xk = __shfl_sync(kFull, UNIT ? b[q] : b[q] * rdiag, k);
      if (lane == k) {
        b[q] = xk;
      } else if (lane > k) {
        b[q] = fmaf(-tk, xk, b[q]);
      }
    }
  }
}

// Upper-triangular solve T x = b (entries k > i of row i used).
template <int R, bool UNIT>
__device__ __forceinline__ void trsv_upper(const float* M, int rs, int cs, float rdiag, float (&b)[kNB]) {
  const int lane = threadIdx.x & 31;
  const float* row = M + (lane < R ? lane : 0) * rs;
#pragma unroll 2
  for (int k = R - 1; k >= 0; --k) {
    const float tk = lane < R ? row[k * cs] : 0.0f;
#pragma unroll
    for (int q = 0; q < kNB; ++q) {
      const float xk = __shfl_sync(kFull, UNIT ? b[q] : b[q] * rdiag, k);
      if (lane == k) {
        b[q] = xk;
      } else if (lane < k) {
        b[q] = fmaf(-tk, xk, b[q]);
      }
    }
  }
}

// Right-looking Cholesky of the lower triangle of the R x R shared matrix A
// (leading dim ld) in place, spread over the whole CTA with one barrier per
// step: step k subtracts A[i][k] A[j][k] / A[k][k] from the trailing lower
// triangle (it only reads column k, which no thread writes during the step);
// the columns are scaled to L[i][k] = A[i][k] / sqrt(A[k][k]) at the end.
// dinv[i] = 1 / L_ii; the upper triangle is zeroed.  All threads call it.
template <int R>
__device__ __forceinline__ void cholesky_block(float* A, int ld, float* dinv) {
  const int tid = threadIdx.x;
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll 1
  for (int k = 0; k < R - 1; ++k) {
    const float rkk = 1.0f / A[k * ld + k];
    // rows over warps, columns over lanes (R <= 32: one column pass)
    const int j = k + 1 + lane;
    const float ajk = j < R ? A[j * ld + k] : 0.0f;
    for (int i = k + 1 + warp; i < R; i += kWWarps) {
      if (j <= i) A[i * ld + j] = fmaf(-A[i * ld + k] * rkk, ajk, A[i * ld + j]);
    }
    __syncthreads();
  }
  for (int e = tid; e < R * R; e += kWThreads) {
    const int i = e / R, j = e - i * R;
    if (j < i) A[i * ld + j] = A[i * ld + j] / sqrtf(A[j * ld + j]);
    if (j > i) A[i * ld + j] = 0.0f;
  }
  __syncthreads();
  for (int i = tid; i < R; i += kWThreads) {
    const float piv = sqrtf(A[i * ld + i]);
    A[i * ld + i] = piv;
    dinv[i] = 1.0f / piv;
  }
  __syncthreads();
}

// Doolittle LU without pivoting of the R x R shared matrix M in place, spread
// over the CTA with one barrier per step: step k subtracts
// M[i][k] M[k][j] / M[k][k] from the trailing block (reading only row and
// column k, which no thread writes during the step); the unit lower factor
// M[i][k] / M[k][k] is formed at the end.  uinv[i] = 1 / U_ii.  All threads call it.
template <int R>
__device__ __forceinline__ void lu_block(float* M, int ld, float* uinv) {
  const int tid = threadIdx.x;
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll 1
  for (int k = 0; k < R - 1; ++k) {
    const float rkk = 1.0f / M[k * ld + k];
    // rows over warps, columns over lanes (R <= 32: one column pass)
    const int j = k + 1 + lane;
    const float ukj = j < R ? M[k * ld + j] : 0.0f;
    for (int i = k + 1 + warp; i < R; i += kWWarps) {
      if (j < R) M[i * ld + j] = fmaf(-M[i * ld + k] * rkk, ukj, M[i * ld + j]);
    }
    __syncthreads();
  }
  for (int e = tid; e < R * R; e += kWThreads) {
    const int i = e / R, k = e - i * R;
    if (i > k) M[i * ld + k] = M[i * ld + k] / M[k * ld + k];
  }
  for (int i = tid; i < R; i += kWThreads) uinv[i] = 1.0f / M[i * ld + i];
  __syncthreads();
}

// Columns [c0, c0 + kNB) of the R x d operand X (row-major, leading dim xld)
// into / out of the lane = row layout; columns past cend read as zero.
__device__ __forceinline__ void get_cols(const float* X, int xld, int R, int c0, int cend, float (&b)[kNB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < kNB; ++q) b[q] = (lane < R && c0 + q < cend) ? X[lane * xld + c0 + q] : 0.0f;
}
__device__ __forceinline__ void put_cols(float* X, int xld, int R, int c0, int cend, const float (&b)[kNB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < kNB; ++q)
    if (lane < R && c0 + q < cend) X[lane * xld + c0 + q] = b[q];
}

// The column range of warp w when `cols` columns are split over the CTA.
__device__ __forceinline__ void warp_cols(int cols, int& c_begin, int& c_end) {
  const int w = threadIdx.x >> 5;
  const int per = (cols + kWWarps - 1) / kWWarps;
  c_begin = min(cols, w * per);
  c_end = min(cols, c_begin + per);
}

// Ps[m] = sum over chunks of P[ch * stride + m], m < stride (a multiple of 4),
// in float4 steps: every load is coalesced and independent of the others.
__device__ __forceinline__ void sum_partials(const float* P, int nchunks, int64_t stride, float* Ps) {
  const int n4 = static_cast<int>(stride / 4);
  const float4* P4 = reinterpret_cast<const float4*>(P);
  for (int e = threadIdx.x; e < n4; e += kWThreads) {
    float4 acc = __ldg(P4 + e);
    for (int ch = 1; ch < nchunks; ++ch) {
      const float4 v = __ldg(P4 + static_cast<int64_t>(ch) * n4 + e);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    reinterpret_cast<float4*>(Ps)[e] = acc;
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.0f;
  for (int w = 0; w < kWWarps; ++w) s += red[w];
  return s;
}

// ============================================================================
// Forward: G = A'^T A'/n + I = L L^T, Z = L^{-1} S, Theta = base + Z W/sqrt(n),
// M = I + F F^T + Omega = LU, U = M^{-1} Z, R_d = L^{-T}(2U - (1+eta) Z)/sqrt(n).
// ============================================================================
template <int R>
__global__ void __launch_bounds__(kWThreads) solve_forward_warp_kernel(const SolveFwdArgs a) {
  constexpr int LD = R + 1;
  extern __shared__ __align__(16) float fsm[];
  const int d = a.d;
  const int XLD = d + 1;
  float* L = fsm;              // [R][LD]
  float* Th = L + R * LD;      // [R][LD]
  float* Mm = Th + R * LD;     // [R][LD]
  float* Zs = Mm + R * LD;     // [R][XLD]  S, then Z
  float* fdiag = Zs + R * XLD; // [R]
  float* dinv = fdiag + R;     // [R] 1 / L_ii
  float* uinv = dinv + R;      // [R] 1 / U_ii
  float* Ws = uinv + R;        // [d][R + 1] W_drive of this head
  float* Ps = fsm + ((static_cast<int>(Ws - fsm) + d * LD + 3) & ~3);  // [2R][R + dt] summed partials
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t bh = blockIdx.x;
  const int64_t b = bh / a.H;
  const int h = static_cast<int>(bh % a.H);
  const float n = a.counts != nullptr ? a.counts[b] : static_cast<float>(a.N);
  const float rsn = 1.0f / sqrtf(n);
  const int NC = R + a.dt;
  const int64_t pstride = static_cast<int64_t>(2 * R) * NC;
  const float* pbase = a.partial + bh * a.nchunks * a.ndt * pstride;
  const TapeLayout tl = tape_layout(a.N, R, d);
  float* tape = a.tape != nullptr ? a.tape + bh * a.tape_stride : nullptr;
  float* Zg = tape != nullptr ? tape + tl.Z : a.zbuf + bh * static_cast<int64_t>(R) * d;

  const float* Wd = a.drive + static_cast<int64_t>(h) * d * R;
  for (int idx = tid; idx < d * R; idx += kWThreads) Ws[(idx / R) * LD + idx % R] = Wd[idx];
  // 1. Sum the chunk partials (coalesced float4 reads, ndt == 1), then
  //    G = (hh + lh + lh^T)/n + I (lower triangle) and S = (hC + lC)/sqrt(n).
  sum_partials(pbase, a.nchunks, pstride, Ps);
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    if (k > i) continue;
    const float s = Ps[i * NC + k] + Ps[(R + i) * NC + k] + Ps[(R + k) * NC + i];
    L[i * LD + k] = s * (rsn * rsn) + (i == k ? 1.0f : 0.0f);
  }
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    Zs[i * XLD + col] = (Ps[i * NC + R + col] + Ps[(R + i) * NC + R + col]) * rsn;
  }
  __syncthreads();
  // 2. Cholesky
  cholesky_block<R>(L, LD, dinv);
  // 3. Z = L^{-1} S (columns over the warps)
  {
    const float rd = lane < R ? dinv[lane] : 1.0f;
    int cb, ce;
    warp_cols(d, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float x[kNB];
      get_cols(Zs, XLD, R, c0, ce, x);
      trsv_lower<R, false>(L, LD, 1, rd, x);
      put_cols(Zs, XLD, R, c0, ce, x);
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    Zg[static_cast<int64_t>(i) * d + col] = Zs[i * XLD + col];
  }
  // 4. Theta = base + Z W_drive / sqrt(n);  F diagonal
  const float* base = a.base + static_cast<int64_t>(h) * R * R;
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    float s = 0.0f;
    for (int c = 0; c < d; ++c) s = fmaf(Zs[i * XLD + c], Ws[c * LD + jj], s);
    Th[i * LD + jj] = base[idx] + s * rsn;
  }
  __syncthreads();
  for (int i = tid; i < R; i += kWThreads) fdiag[i] = softplus20(Th[i * LD + i] + kSoftplusOneOffset);
  __syncthreads();
  // 5. M = I + F F^T + Omega
  for (int idx = tid; idx < R * R; idx += kWThreads) {
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
    for (int idx = tid; idx < R * R; idx += kWThreads) {
      const int i = idx / R, jj = idx % R;
      tape[tl.L + idx] = L[i * LD + jj];
      tape[tl.Theta + idx] = Th[i * LD + jj];
    }
    if (tid == 0) tape[tl.n] = n;
  }
  // 6. LU
  lu_block<R>(Mm, LD, uinv);
  if (tape != nullptr) {
    for (int idx = tid; idx < R * R; idx += kWThreads) tape[tl.LU + idx] = Mm[(idx / R) * LD + idx % R];
  }
  if (a.pivots != nullptr) {
    for (int i = tid; i < R; i += kWThreads) a.pivots[bh * R + i] = i + 1;
  }
  // 7. U = M^{-1} Z;  R_d = L^{-T} (2U - (1+eta) Z) / sqrt(n)
  const float eta = bounded_complement(a.eta_raw[h]);
  uint8_t* rm = reinterpret_cast<uint8_t*>(a.rmat + bh * a.d_pad * R);
  constexpr uint32_t RSBO = R * 16;
  {
    const float ru = lane < R ? uinv[lane] : 1.0f;
    const float rd = lane < R ? dinv[lane] : 1.0f;
    int cb, ce;
    warp_cols(d, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float z[kNB], u[kNB];
      get_cols(Zs, XLD, R, c0, ce, z);
#pragma unroll
      for (int q = 0; q < kNB; ++q) u[q] = z[q];
      trsv_lower<R, true>(Mm, LD, 1, 1.0f, u);   // unit lower factor of M
      trsv_upper<R, false>(Mm, LD, 1, ru, u);    // U
      float x[kNB];
#pragma unroll
      for (int q = 0; q < kNB; ++q) x[q] = 2.0f * u[q] - (1.0f + eta) * z[q];
      trsv_upper<R, false>(L, 1, LD, rd, x);     // L^T
#pragma unroll
      for (int q = 0; q < kNB; ++q) {
        const int col = c0 + q;
        if (lane < R && col < ce) {
          if (tape != nullptr) tape[tl.U + static_cast<int64_t>(lane) * d + col] = u[q];
          *reinterpret_cast<bf16*>(rm + kmajor_offset(col, lane, RSBO)) = __float2bfloat16_rn(x[q] * rsn);
        }
      }
    }
  }
  for (int idx = tid; idx < (a.d_pad - d) * R; idx += kWThreads) {
    const int col = d + idx / R, i = idx % R;
    *reinterpret_cast<bf16*>(rm + kmajor_offset(col, i, RSBO)) = __float2bfloat16_rn(0.0f);
  }
}

// ============================================================================
// Backward (see solve_backward_kernel in mixer.cu for the derivation):
//   D = L^{-1}(A'^T dY)/sqrt(n), lam = M^{-T} 2D, dK = -lam U^T, dTheta,
//   dZ = lam - (1+eta) D + dTheta W^T/sqrt(n), E = M' D^T + dZ Z^T,
//   R_d = L^{-T} M'/sqrt(n), R_z = L^{-T} dZ/sqrt(n), Q = L^{-T} Psi L^{-1}/n.
// ============================================================================
template <int R>
__global__ void __launch_bounds__(kWThreads) solve_backward_warp_kernel(const SolveBwdArgs a) {
  constexpr int LD = R + 1;
  extern __shared__ __align__(16) float fsm[];
  const int d = a.d;
  const int XLD = d + 1;
  float* L = fsm;               // [R][LD]
  float* Mm = L + R * LD;       // [R][LD] packed LU
  float* Th = Mm + R * LD;      // [R][LD]
  float* dK = Th + R * LD;      // [R][LD] dK, then dTheta, then Psi
  float* E = dK + R * LD;       // [R][LD]
  float* X1 = E + R * LD;       // [R][XLD] D
  float* X2 = X1 + R * XLD;     // [R][XLD] lambda, then dZ
  float* X3 = X2 + R * XLD;     // [R][XLD] U, then M'
  float* X4 = X3 + R * XLD;     // [R][XLD] Z
  float* fdiag = X4 + R * XLD;  // [R]
  float* dinv = fdiag + R;      // [R] 1 / L_ii
  float* uinv = dinv + R;       // [R] 1 / U_ii
  float* Ws = uinv + R;         // [d][R + 1] W_drive of this head
  float* Ps = fsm + ((static_cast<int>(Ws - fsm) + d * LD + 3) & ~3);  // [2R][dt] summed partials
  __shared__ float red[kWWarps];
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t bh = blockIdx.x;
  const int h = static_cast<int>(bh % a.H);
  const TapeLayout tl = tape_layout(a.N, R, d);
  const float* tape = a.tape + bh * a.tape_stride;
  const float n = tape[tl.n];
  const float rsn = 1.0f / sqrtf(n);
  const float eta = bounded_complement(a.eta_raw[h]);
  const int NC = a.dt;
  const int64_t pstride = static_cast<int64_t>(2 * R) * NC;
  const float* pbase = a.partial + bh * a.nchunks * a.ndt * pstride;
  const float* Wd = a.drive + static_cast<int64_t>(h) * d * R;

  for (int idx = tid; idx < d * R; idx += kWThreads) Ws[(idx / R) * LD + idx % R] = Wd[idx];
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    L[i * LD + jj] = tape[tl.L + idx];
    Mm[i * LD + jj] = tape[tl.LU + idx];
    Th[i * LD + jj] = tape[tl.Theta + idx];
  }
  sum_partials(pbase, a.nchunks, pstride, Ps);
  __syncthreads();
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    X1[i * XLD + col] = Ps[i * NC + col] + Ps[(R + i) * NC + col];
    X3[i * XLD + col] = tape[tl.U + static_cast<int64_t>(i) * d + col];
    X4[i * XLD + col] = tape[tl.Z + static_cast<int64_t>(i) * d + col];
  }
  __syncthreads();
  for (int i = tid; i < R; i += kWThreads) {
    fdiag[i] = softplus20(Th[i * LD + i] + kSoftplusOneOffset);
    dinv[i] = 1.0f / L[i * LD + i];
    uinv[i] = 1.0f / Mm[i * LD + i];
  }
  __syncthreads();

  // Pass A: D = L^{-1} X1 / sqrt(n);  lam = M^{-T} (2 D) = L_u^{-T} U^{-T} (2 D)
  {
    const float rd = lane < R ? dinv[lane] : 1.0f;
    const float ru = lane < R ? uinv[lane] : 1.0f;
    int cb, ce;
    warp_cols(d, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float x[kNB];
      get_cols(X1, XLD, R, c0, ce, x);
      trsv_lower<R, false>(L, LD, 1, rd, x);
      float lam[kNB];
#pragma unroll
      for (int q = 0; q < kNB; ++q) {
        x[q] *= rsn;
        lam[q] = 2.0f * x[q];
      }
      put_cols(X1, XLD, R, c0, ce, x);
      // columns of the packed LU: U^T (entries j <= i), unit L^T (entries j > i)
      trsv_lower<R, false>(Mm, 1, LD, ru, lam);  // U^T y = 2D
      trsv_upper<R, true>(Mm, 1, LD, 1.0f, lam); // L_u^T lam = y
      put_cols(X2, XLD, R, c0, ce, lam);
    }
  }
  __syncthreads();
  float dz_dot = 0.0f;
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    dz_dot = fmaf(X1[i * XLD + col], X4[i * XLD + col], dz_dot);
  }
  // dK = -lam U^T
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    float s = 0.0f;
    for (int c = 0; c < d; ++c) s = fmaf(X2[i * XLD + c], X3[jj * XLD + c], s);
    dK[i * LD + jj] = -s;
  }
  __syncthreads();
  // dTheta through K = F F^T + Omega (into E, then back into dK)
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    float v;
    if (i < jj) {
      v = dK[i * LD + jj] - dK[jj * LD + i];
    } else {
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
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    const float v = E[i * LD + jj];
    dK[i * LD + jj] = v;
    a.gbase[bh * R * R + idx] = v;
  }
  __syncthreads();
  // Pass B: dZ (X2), M' = 2U - (1+eta) Z (X3), drive-gradient partial Z^T dTheta / sqrt(n)
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    const float* wrow = Ws + col * LD;
    float s = 0.0f;
    for (int jj = 0; jj < R; ++jj) s = fmaf(dK[i * LD + jj], wrow[jj], s);
    X2[i * XLD + col] = X2[i * XLD + col] - (1.0f + eta) * X1[i * XLD + col] + s * rsn;
    X3[i * XLD + col] = 2.0f * X3[i * XLD + col] - (1.0f + eta) * X4[i * XLD + col];
  }
  for (int idx = tid; idx < d * R; idx += kWThreads) {
    const int col = idx / R, jj = idx % R;
    float s = 0.0f;
    for (int i = 0; i < R; ++i) s = fmaf(X4[i * XLD + col], dK[i * LD + jj], s);
    a.gdrive[(bh * d + col) * R + jj] = s * rsn;
  }
  __syncthreads();
  // E = M' D^T + dZ Z^T
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    float s = 0.0f;
    for (int c = 0; c < d; ++c) s += X3[i * XLD + c] * X1[k * XLD + c] + X2[i * XLD + c] * X4[k * XLD + c];
    E[i * LD + k] = s;
  }
  // R_d = L^{-T} M' / sqrt(n) -> B1y,  R_z = L^{-T} dZ / sqrt(n) -> B1c and B2
  uint8_t* b1y = reinterpret_cast<uint8_t*>(a.b1y + bh * R * a.d_pad);
  uint8_t* b1c = reinterpret_cast<uint8_t*>(a.b1c + bh * R * a.d_pad);
  uint8_t* b2 = reinterpret_cast<uint8_t*>(a.b2 + bh * a.d_pad * R);
  const uint32_t SBO_Y = static_cast<uint32_t>(a.d_pad) * 16;
  constexpr uint32_t SBO_R = R * 16;
  {
    const float rd = lane < R ? dinv[lane] : 1.0f;
    int cb, ce;
    warp_cols(d, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float xm[kNB], xz[kNB];
      get_cols(X3, XLD, R, c0, ce, xm);
      get_cols(X2, XLD, R, c0, ce, xz);
      trsv_upper<R, false>(L, 1, LD, rd, xm);
      trsv_upper<R, false>(L, 1, LD, rd, xz);
#pragma unroll
      for (int q = 0; q < kNB; ++q) {
        const int col = c0 + q;
        if (lane < R && col < ce) {
          *reinterpret_cast<bf16*>(b1y + kmajor_offset(lane, col, SBO_Y)) = __float2bfloat16_rn(xm[q] * rsn);
          const bf16 rz = __float2bfloat16_rn(xz[q] * rsn);
          *reinterpret_cast<bf16*>(b1c + kmajor_offset(lane, col, SBO_Y)) = rz;
          *reinterpret_cast<bf16*>(b2 + kmajor_offset(col, lane, SBO_R)) = rz;
        }
      }
    }
  }
  for (int idx = tid; idx < (a.d_pad - d) * R; idx += kWThreads) {
    const int col = d + idx / R, i = idx % R;
    const bf16 z = __float2bfloat16_rn(0.0f);
    *reinterpret_cast<bf16*>(b1y + kmajor_offset(i, col, SBO_Y)) = z;
    *reinterpret_cast<bf16*>(b1c + kmajor_offset(i, col, SBO_Y)) = z;
    *reinterpret_cast<bf16*>(b2 + kmajor_offset(col, i, SBO_R)) = z;
  }
  __syncthreads();
  // Q = L^{-T} Psi L^{-1} / n with Psi = tril(E) + tril(E,-1)^T (symmetric):
  // X = L^{-T} Psi column by column, then Q^T = L^{-T} X^T.
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    dK[i * LD + k] = i >= k ? E[i * LD + k] : E[k * LD + i];
  }
  __syncthreads();
  {
    const float rd = lane < R ? dinv[lane] : 1.0f;
    int cb, ce;
    warp_cols(R, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float x[kNB];
      get_cols(dK, LD, R, c0, ce, x);
      trsv_upper<R, false>(L, 1, LD, rd, x);
      // store transposed: E[c][i] = X[i][c]
#pragma unroll
      for (int q = 0; q < kNB; ++q)
        if (lane < R && c0 + q < ce) E[(c0 + q) * LD + lane] = x[q];
    }
    __syncthreads();
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float x[kNB];
      get_cols(E, LD, R, c0, ce, x);
      trsv_upper<R, false>(L, 1, LD, rd, x);
      put_cols(dK, LD, R, c0, ce, x);
    }
  }
  __syncthreads();
  // dK now holds Q^T; B1a[n = i][k = j] = -Q[j][i] / n = -dK[i][j] / n
  uint8_t* b1a = reinterpret_cast<uint8_t*>(a.b1a + bh * R * R);
  const float inv_n = rsn * rsn;
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    *reinterpret_cast<bf16*>(b1a + kmajor_offset(i, jj, SBO_R)) = __float2bfloat16_rn(-dK[i * LD + jj] * inv_n);
  }
  const float s = block_sum(dz_dot, red);
  if (tid == 0) a.etadot[bh] = s;
}

// Shared-memory floats before the partial-sum block, rounded up to 4 floats.
template <int R>
int fwd_head(int d) {
  return (3 * R * (R + 1) + R * (d + 1) + 3 * R + d * (R + 1) + 3) / 4 * 4;
}
template <int R>
int bwd_head(int d) {
  return (5 * R * (R + 1) + 4 * R * (d + 1) + 3 * R + d * (R + 1) + 3) / 4 * 4;
}
// The partial-sum block holds one whole chunk partial: 2R rows of R + dt
// (forward) or dt (backward) columns, dt = d_pad >= d.
template <int R>
size_t fwd_smem(int d, int dt) {
  return sizeof(float) * (fwd_head<R>(d) + 2 * R * (R + dt));
}
template <int R>
size_t bwd_smem(int d, int dt) {
  return sizeof(float) * (bwd_head<R>(d) + 2 * R * dt);
}

}  // namespace

bool warp_solves_usable(const Plan& p) {
  // One content tile per chunk partial (d_pad <= 128), shared memory well inside one SM.
  const int d = static_cast<int>(p.d), dt = static_cast<int>(p.dt);
  return (p.R == 16 || p.R == 32) && p.ndt == 1 && fwd_smem<32>(d, dt) <= 160 * 1024 &&
         bwd_smem<32>(d, dt) <= 160 * 1024;
}

cudaError_t launch_solve_forward_warp(const Plan& p, const SolveFwdArgs& s, cudaStream_t stream) {
  const int d = static_cast<int>(p.d);
  const int dt = static_cast<int>(p.dt);
  const size_t smem = p.R == 16 ? fwd_smem<16>(d, dt) : fwd_smem<32>(d, dt);
  const void* fn = p.R == 16 ? reinterpret_cast<const void*>(&solve_forward_warp_kernel<16>)
                             : reinterpret_cast<const void*>(&solve_forward_warp_kernel<32>);
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope("solve_fwd", stream);
  if (p.R == 16) {
    solve_forward_warp_kernel<16><<<static_cast<unsigned>(p.BH), kWThreads, smem, stream>>>(s);
  } else {
    solve_forward_warp_kernel<32><<<static_cast<unsigned>(p.BH), kWThreads, smem, stream>>>(s);
  }
  return cudaGetLastError();
}

cudaError_t launch_solve_backward_warp(const Plan& p, const SolveBwdArgs& s, cudaStream_t stream) {
  const int d = static_cast<int>(p.d);
  const int dt = static_cast<int>(p.dt);
  const size_t smem = p.R == 16 ? bwd_smem<16>(d, dt) : bwd_smem<32>(d, dt);
  const void* fn = p.R == 16 ? reinterpret_cast<const void*>(&solve_backward_warp_kernel<16>)
                             : reinterpret_cast<const void*>(&solve_backward_warp_kernel<32>);
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope("solve_bwd", stream);
  if (p.R == 16) {
    solve_backward_warp_kernel<16><<<static_cast<unsigned>(p.BH), kWThreads, smem, stream>>>(s);
  } else {
    solve_backward_warp_kernel<32><<<static_cast<unsigned>(p.BH), kWThreads, smem, stream>>>(s);
  }
  return cudaGetLastError();
}

}  // namespace lsso
