// Per-(sample, head) r x r solves of the LSSO mixer (sm_100a), r in {16, 32, 48, 64}.
//
// Same algebra as solve_forward_kernel / solve_backward_kernel in mixer.cu
// (reference lsso/ball/reference.py:411-572): Cholesky of the Gram matrix,
// the accretive generator, LU without pivoting, and the triangular solves of
// the forward and the analytic backward.  The difference is the execution
// model: lane l of a warp owns matrix rows l, l + 32, ... (P = ceil(R/32)
// register slots), so
//   - a triangular solve is R shuffle steps per right-hand side, four
//     right-hand sides per warp at a time for instruction-level parallelism,
//     replacing a thread-per-column R^2 chain; transposed solves read the
//     matrix by columns (one column view of the packed LU serves both U^T and
//     the unit L^T);
//   - Cholesky and LU advance eight columns per panel: warp 0 factorises the
//     panel in registers with shuffles, the CTA applies the panel's updates to
//     the trailing block (2-3 barriers per panel);
//   - the r x r and r x d products are register-blocked over a 16 x 16 thread
//     grid;
//   - all d columns of the R x d operands stay in shared memory, split over
//     the CTA's warps;
//   - the chunk partials of the moment pass are summed with coalesced float4
//     loads straight into the matrices that use them.
// One CTA (eight warps) per (sample, head).
#include "mixer.h"
#include "mixer_common.cuh"

namespace lsso {

namespace {

constexpr int kWThreads = 256;
constexpr int kWWarps = kWThreads / 32;
constexpr int kNB = 4;  // right-hand sides per warp-level solve
constexpr unsigned kFull = 0xffffffffu;
constexpr size_t kWarpSolveSmemLimit = 200 * 1024;

// Rows per lane.
template <int R>
__host__ __device__ constexpr int rows_per_lane() {
  return (R + 31) / 32;
}

// Matrices stay in shared memory; lane l works on rows 32 p + l.  The step
// loops are kept rolled (unroll 2) so the code stays small: these kernels run
// once per (sample, head), and fully unrolled chains overflow the instruction
// cache.  A matrix element (row, k) is read at M[row * rs + k * cs]: rs = ld,
// cs = 1 for the matrix itself, rs = 1, cs = ld for its transpose.

// Lower-triangular solve T x = b (lane l, slot p: b_{32p+l} in b[p][q]);
// rdiag[p] = 1 / T_ii of the lane's row i in slot p (ignored when UNIT).
template <int R, bool UNIT>
__device__ __forceinline__ void trsv_lower(const float* M, int rs, int cs, const float (&rdiag)[rows_per_lane<R>()],
                                           float (&b)[rows_per_lane<R>()][kNB]) {
  constexpr int P = rows_per_lane<R>();
  const int lane = threadIdx.x & 31;
  const float* row[P];
#pragma unroll
  for (int p = 0; p < P; ++p) row[p] = M + (32 * p + lane < R ? 32 * p + lane : 0) * rs;
#pragma unroll
  for (int s = 0; s < P; ++s) {
    const int kend = 32 * s + 32 < R ? 32 * s + 32 : R;
#pragma unroll 2
    for (int k = 32 * s; k < kend; ++k) {
      const int src = k - 32 * s;
      float tk[P];
#pragma unroll
      for (int p = s; p < P; ++p) tk[p] = 32 * p + lane < R ? row[p][k * cs] : 0.0f;
#pragma unroll
      for (int q = 0; q < kNB; ++q) {
        const float xk = __shfl_sync(kFull, UNIT ? b[s][q] : b[s][q] * rdiag[s], src);
        if (lane == src) {
          b[s][q] = xk;
        } else if (lane > src) {
          b[s][q] = fmaf(-tk[s], xk, b[s][q]);
        }
#pragma unroll
        for (int p = s + 1; p < P; ++p) b[p][q] = fmaf(-tk[p], xk, b[p][q]);
      }
    }
  }
}

// Upper-triangular solve T x = b (entries k > i of row i used).
template <int R, bool UNIT>
__device__ __forceinline__ void trsv_upper(const float* M, int rs, int cs, const float (&rdiag)[rows_per_lane<R>()],
                                           float (&b)[rows_per_lane<R>()][kNB]) {
  constexpr int P = rows_per_lane<R>();
  const int lane = threadIdx.x & 31;
  const float* row[P];
#pragma unroll
  for (int p = 0; p < P; ++p) row[p] = M + (32 * p + lane < R ? 32 * p + lane : 0) * rs;
#pragma unroll
  for (int s = P - 1; s >= 0; --s) {
    const int kend = 32 * s + 32 < R ? 32 * s + 32 : R;
#pragma unroll 2
    for (int k = kend - 1; k >= 32 * s; --k) {
      const int src = k - 32 * s;
      float tk[P];
#pragma unroll
      for (int p = 0; p <= s; ++p) tk[p] = 32 * p + lane < R ? row[p][k * cs] : 0.0f;
#pragma unroll
      for (int q = 0; q < kNB; ++q) {
        const float xk = __shfl_sync(kFull, UNIT ? b[s][q] : b[s][q] * rdiag[s], src);
        if (lane == src) {
          b[s][q] = xk;
        } else if (lane < src) {
          b[s][q] = fmaf(-tk[s], xk, b[s][q]);
        }
#pragma unroll
        for (int p = 0; p < s; ++p) b[p][q] = fmaf(-tk[p], xk, b[p][q]);
      }
    }
  }
}

// rd[p] = v[32 p + lane] (1 past R).
template <int R>
__device__ __forceinline__ void lane_rows(const float* v, float (&rd)[rows_per_lane<R>()]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < rows_per_lane<R>(); ++p) rd[p] = 32 * p + lane < R ? v[32 * p + lane] : 1.0f;
}

// Panel factorisations: the factorisation advances kPanel columns at a time.
// Warp 0 factorises the column panel in registers (lane l holds the panel
// entries of rows l and l + 32; the panel's steps are unrolled, pivots and
// multipliers broadcast by shuffles, no barrier), then the CTA applies the
// panel's rank-1 updates to the trailing block in step order, so every
// element receives exactly the operations, in exactly the order, of the
// one-step-per-barrier algorithm, with 2 (Cholesky) or 3 (LU) barriers per
// panel instead of one per step.  Pn ([R][kPanel] floats) holds the panel's
// multipliers A[i][k] / A[k][k].
constexpr int kPanel = 8;

// Value of row `row` (panel register slot row >> 5) held by lane row & 31,
// broadcast to the warp.
template <int P>
__device__ __forceinline__ float row_value(const float (&x)[P][kPanel], int row, int c) {
  const float v = (P > 1 && (row >> 5) != 0) ? x[P - 1][c] : x[0][c];
  return __shfl_sync(kFull, v, row & 31);
}

template <int R>
__device__ __forceinline__ void cholesky_panels(float* A, int ld, float* dinv, float* Pn) {
  constexpr int P = rows_per_lane<R>();
  const int tid = threadIdx.x, lane = tid & 31;
  __syncthreads();
#pragma unroll 1
  for (int k0 = 0; k0 < R - 1; k0 += kPanel) {
    const int pw = min(kPanel, R - 1 - k0);  // steps in this panel
    if (tid < 32) {
      float x[P][kPanel];
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int c = 0; c < kPanel; ++c) {
          const int row = 32 * p + lane;
          x[p][c] = (row < R && k0 + c < R) ? A[row * ld + k0 + c] : 0.0f;
        }
#pragma unroll
      for (int t = 0; t < kPanel; ++t) {
        if (t < pw) {
          const int kt = k0 + t;
          const float rkk = 1.0f / row_value<P>(x, kt, t);
          float l[P];
#pragma unroll
          for (int p = 0; p < P; ++p) l[p] = x[p][t] * rkk;
#pragma unroll
          for (int c = t + 1; c < kPanel; ++c) {
            const float ajk = row_value<P>(x, (k0 + c) < R ? k0 + c : R - 1, t);  // A[k0+c][kt]
#pragma unroll
            for (int p = 0; p < P; ++p)
              if (32 * p + lane > kt) x[p][c] = fmaf(-l[p], ajk, x[p][c]);
          }
#pragma unroll
          for (int p = 0; p < P; ++p) {
            const int row = 32 * p + lane;
            if (row < R) Pn[row * kPanel + t] = row > kt ? l[p] : 0.0f;
          }
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int c = 0; c < kPanel; ++c) {
          const int row = 32 * p + lane;
          if (row < R && k0 + c < R) A[row * ld + k0 + c] = x[p][c];
        }
    }
    __syncthreads();
    const int j0 = k0 + kPanel, n = R - j0;
    for (int e = tid; e < n * n; e += kWThreads) {
      const int ii = j0 + e / n, jj = j0 + e % n;
      if (jj > ii) continue;
      float acc = A[ii * ld + jj];
#pragma unroll
      for (int t = 0; t < kPanel; ++t)
        if (t < pw) acc = fmaf(-Pn[ii * kPanel + t], A[jj * ld + k0 + t], acc);
      A[ii * ld + jj] = acc;
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

template <int R>
__device__ __forceinline__ void lu_panels(float* M, int ld, float* uinv, float* Pn) {
  constexpr int P = rows_per_lane<R>();
  const int tid = threadIdx.x, lane = tid & 31;
  __syncthreads();
#pragma unroll 1
  for (int k0 = 0; k0 < R - 1; k0 += kPanel) {
    const int pw = min(kPanel, R - 1 - k0);
    if (tid < 32) {
      float x[P][kPanel];
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int c = 0; c < kPanel; ++c) {
          const int row = 32 * p + lane;
          x[p][c] = (row < R && k0 + c < R) ? M[row * ld + k0 + c] : 0.0f;
        }
#pragma unroll
      for (int t = 0; t < kPanel; ++t) {
        if (t < pw) {
          const int kt = k0 + t;
          const float rkk = 1.0f / row_value<P>(x, kt, t);
          float l[P];
#pragma unroll
          for (int p = 0; p < P; ++p) l[p] = x[p][t] * rkk;
#pragma unroll
          for (int c = t + 1; c < kPanel; ++c) {
            const float ukj = row_value<P>(x, kt, c);  // M[kt][k0+c]
#pragma unroll
            for (int p = 0; p < P; ++p)
              if (32 * p + lane > kt) x[p][c] = fmaf(-l[p], ukj, x[p][c]);
          }
#pragma unroll
          for (int p = 0; p < P; ++p) {
            const int row = 32 * p + lane;
            if (row < R) Pn[row * kPanel + t] = row > kt ? l[p] : 0.0f;
          }
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int c = 0; c < kPanel; ++c) {
          const int row = 32 * p + lane;
          if (row < R && k0 + c < R) M[row * ld + k0 + c] = x[p][c];
        }
    }
    __syncthreads();
    // the panel rows right of the panel: row k0+t receives the steps k0 .. k0+t-1, in order
    const int j0 = k0 + kPanel, n = R - j0;
    for (int jj = tid; jj < n; jj += kWThreads) {
      const int j = j0 + jj;
      float u[kPanel];
#pragma unroll
      for (int t = 0; t < kPanel; ++t) u[t] = k0 + t < R ? M[(k0 + t) * ld + j] : 0.0f;
#pragma unroll
      for (int t = 1; t < kPanel; ++t)
#pragma unroll
        for (int q = 0; q < t; ++q)
          if (q < pw) u[t] = fmaf(-Pn[(k0 + t) * kPanel + q], u[q], u[t]);
#pragma unroll
      for (int t = 1; t < kPanel; ++t)
        if (k0 + t < R) M[(k0 + t) * ld + j] = u[t];
    }
    __syncthreads();
    for (int e = tid; e < n * n; e += kWThreads) {
      const int ii = j0 + e / n, jj = j0 + e % n;
      float acc = M[ii * ld + jj];
#pragma unroll
      for (int t = 0; t < kPanel; ++t)
        if (t < pw) acc = fmaf(-Pn[ii * kPanel + t], M[(k0 + t) * ld + jj], acc);
      M[ii * ld + jj] = acc;
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

// out(i, j) = sum_k a(i, k) b(k, j) for the R rows and `ncols` columns, as
// register tiles (rows ty + 16 a, columns c0 + tx + 16 b in passes of 16 NB
// columns), k ascending; store(i, j, acc) receives each result.
// With SYNC the CTA synchronises before the stores (single pass only), so the
// result may overwrite an operand.
template <int R, int NB, bool SYNC = false, typename FA, typename FB, typename FS>
__device__ __forceinline__ void tile_gemm(int ncols, int kdim, FA a_at, FB b_at, FS store) {
  constexpr int T = R / 16;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  for (int c0 = 0; c0 < ncols; c0 += 16 * NB) {
    float acc[T][NB];
#pragma unroll
    for (int a = 0; a < T; ++a)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[a][b] = 0.0f;
#pragma unroll 2
    for (int k = 0; k < kdim; ++k) {
      float av[T], bv[NB];
#pragma unroll
      for (int a = 0; a < T; ++a) av[a] = a_at(ty + 16 * a, k);
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int j = c0 + tx + 16 * b;
        bv[b] = j < ncols ? b_at(k, j) : 0.0f;
      }
#pragma unroll
      for (int a = 0; a < T; ++a)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
    }
    if (SYNC) __syncthreads();
#pragma unroll
    for (int a = 0; a < T; ++a)
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        const int j = c0 + tx + 16 * b;
        if (j < ncols) store(ty + 16 * a, j, acc[a][b]);
      }
  }
}

// Columns per register-tile pass: R x R products use all R columns at once.
template <int R>
__host__ __device__ constexpr int square_nb() {
  return R / 16;
}

// Columns [c0, c0 + kNB) of the R x d operand X (row-major, leading dim xld)
// into / out of the lane = row layout; columns past cend read as zero.
template <int R>
__device__ __forceinline__ void get_cols(const float* X, int xld, int c0, int cend,
                                         float (&b)[rows_per_lane<R>()][kNB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < rows_per_lane<R>(); ++p) {
    const int row = 32 * p + lane;
#pragma unroll
    for (int q = 0; q < kNB; ++q) b[p][q] = (row < R && c0 + q < cend) ? X[row * xld + c0 + q] : 0.0f;
  }
}
template <int R>
__device__ __forceinline__ void put_cols(float* X, int xld, int c0, int cend,
                                         const float (&b)[rows_per_lane<R>()][kNB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int p = 0; p < rows_per_lane<R>(); ++p) {
    const int row = 32 * p + lane;
#pragma unroll
    for (int q = 0; q < kNB; ++q)
      if (row < R && c0 + q < cend) X[row * xld + c0 + q] = b[p][q];
  }
}

// The column range of warp w when `cols` columns are split over the CTA.
__device__ __forceinline__ void warp_cols(int cols, int& c_begin, int& c_end) {
  const int w = threadIdx.x >> 5;
  const int per = (cols + kWWarps - 1) / kWWarps;
  c_begin = min(cols, w * per);
  c_end = min(cols, c_begin + per);
}

__device__ __forceinline__ void add4(float4& a, const float4 b) {
  a.x += b.x;
  a.y += b.y;
  a.z += b.z;
  a.w += b.w;
}

// Chunk partials [nchunks][2R][cols] (rows R.. hold the low halves): element
// e of the first R rows summed over the chunks, high and low rows separately,
// in float4 steps (every load coalesced and independent of the others).
// fn(row, col, hi4, lo4) receives the four columns starting at col.
template <int R, int BATCH, typename Fn>
__device__ __forceinline__ void sum_chunks(const float* partial, int nchunks, int cols, Fn fn) {
  const int c4 = cols / 4;
  const int64_t lo = static_cast<int64_t>(R) * c4;
  const int64_t stride = 2 * lo;
  const float4* P4 = reinterpret_cast<const float4*>(partial);
  for (int e = threadIdx.x; e < R * c4; e += kWThreads) {
    float4 hi = __ldg(P4 + e);
    float4 lw = __ldg(P4 + lo + e);
    // The chunks BATCH at a time: their loads are all in flight before the
    // additions, which still go in chunk order (the partials come from L2 or
    // DRAM, so one round trip per chunk would dominate the sum).
    for (int ch = 1; ch < nchunks; ch += BATCH) {
      float4 h[BATCH], l[BATCH];
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        if (ch + u < nchunks) {
          h[u] = __ldg(P4 + (ch + u) * stride + e);
          l[u] = __ldg(P4 + (ch + u) * stride + lo + e);
        }
      }
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        if (ch + u < nchunks) {
          add4(hi, h[u]);
          add4(lw, l[u]);
        }
      }
    }
    const int row = e / c4;
    fn(row, (e - row * c4) * 4, hi, lw);
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
__global__ void __launch_bounds__(kWThreads, 4) solve_forward_warp_kernel(const SolveFwdArgs a) {
  pdl_wait();
  constexpr int LD = R + 1;
  constexpr int P = rows_per_lane<R>();
  extern __shared__ __align__(16) float fsm[];
  const int d = a.d;
  const int XLD = d + 1;
  float* L = fsm;              // [R][LD]
  float* Th = L + R * LD;      // [R][LD] low Gram half, then Theta
  float* Mm = Th + R * LD;     // [R][LD]
  float* Zs = Mm + R * LD;     // [R][XLD]  S, then Z
  float* fdiag = Zs + R * XLD; // [R]
  float* dinv = fdiag + R;     // [R] 1 / L_ii
  float* uinv = dinv + R;      // [R] 1 / U_ii
  float* Ws = uinv + R;        // [d][R + 1] W_drive of this head
  float* buf = Ws + d * LD;    // [R * kPanel] panel multipliers of the factorisations
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
  // 1. Sum the chunk partials (ndt == 1): L <- hh + lh, Th <- lh, S = (hC + lC)/sqrt(n);
  //    then G = (hh + lh + lh^T)/n + I on the lower triangle.
  sum_chunks<R, 3>(pbase, a.nchunks, NC, [&](int i, int c, float4 hi, float4 lo) {
    const float hv[4] = {hi.x, hi.y, hi.z, hi.w};
    const float lv[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int cc = c + u;
      if (cc < R) {
        L[i * LD + cc] = hv[u] + lv[u];
        Th[i * LD + cc] = lv[u];
      } else if (cc - R < d) {
        Zs[i * XLD + cc - R] = (hv[u] + lv[u]) * rsn;
      }
    }
  });
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    if (k > i) continue;
    L[i * LD + k] = (L[i * LD + k] + Th[k * LD + i]) * (rsn * rsn) + (i == k ? 1.0f : 0.0f);
  }
  // 2. Cholesky
  cholesky_panels<R>(L, LD, dinv, buf);
  // 3. Z = L^{-1} S (columns over the warps)
  {
    float rd[P];
    lane_rows<R>(dinv, rd);
    int cb, ce;
    warp_cols(d, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float x[P][kNB];
      get_cols<R>(Zs, XLD, c0, ce, x);
      trsv_lower<R, false>(L, LD, 1, rd, x);
      put_cols<R>(Zs, XLD, c0, ce, x);
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    Zg[static_cast<int64_t>(i) * d + col] = Zs[i * XLD + col];
  }
  // 4. Theta = base + Z W_drive / sqrt(n);  F diagonal
  const float* base = a.base + static_cast<int64_t>(h) * R * R;
  tile_gemm<R, square_nb<R>()>(
      R, d, [&](int i, int c) { return Zs[i * XLD + c]; }, [&](int c, int j) { return Ws[c * LD + j]; },
      [&](int i, int j, float acc) { Th[i * LD + j] = base[i * R + j] + acc * rsn; });
  __syncthreads();
  for (int i = tid; i < R; i += kWThreads) fdiag[i] = softplus20(Th[i * LD + i] + kSoftplusOneOffset);
  __syncthreads();
  // 5. M = I + F F^T + Omega
  //    (F: strict lower triangle of Theta, softplus diagonal, zero above; built in Mm first)
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    Mm[i * LD + k] = k < i ? Th[i * LD + k] : (k == i ? fdiag[i] : 0.0f);
  }
  __syncthreads();
  tile_gemm<R, square_nb<R>(), true>(
      R, R, [&](int i, int k) { return Mm[i * LD + k]; }, [&](int k, int j) { return Mm[j * LD + k]; },
      [&](int i, int j, float acc) {
        const float omega = i < j ? Th[i * LD + j] : (i > j ? -Th[j * LD + i] : 0.0f);
        Mm[i * LD + j] = (i == j ? 1.0f : 0.0f) + acc + omega;
      });
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
  lu_panels<R>(Mm, LD, uinv, buf);
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
    float ru[P], rd[P], one[P];
    lane_rows<R>(uinv, ru);
    lane_rows<R>(dinv, rd);
#pragma unroll
    for (int p = 0; p < P; ++p) one[p] = 1.0f;
    int cb, ce;
    warp_cols(d, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float z[P][kNB], u[P][kNB];
      get_cols<R>(Zs, XLD, c0, ce, z);
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < kNB; ++q) u[p][q] = z[p][q];
      trsv_lower<R, true>(Mm, LD, 1, one, u);   // unit lower factor of M
      trsv_upper<R, false>(Mm, LD, 1, ru, u);   // U
      float x[P][kNB];
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < kNB; ++q) x[p][q] = 2.0f * u[p][q] - (1.0f + eta) * z[p][q];
      trsv_upper<R, false>(L, 1, LD, rd, x);    // L^T
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int row = 32 * p + lane;
#pragma unroll
        for (int q = 0; q < kNB; ++q) {
          const int col = c0 + q;
          if (row < R && col < ce) {
            if (tape != nullptr) tape[tl.U + static_cast<int64_t>(row) * d + col] = u[p][q];
            *reinterpret_cast<bf16*>(rm + kmajor_offset(col, row, RSBO)) = __float2bfloat16_rn(x[p][q] * rsn);
          }
        }
      }
    }
  }
  for (int idx = tid; idx < (a.d_pad - d) * R; idx += kWThreads) {
    const int col = d + idx / R, i = idx % R;
    *reinterpret_cast<bf16*>(rm + kmajor_offset(col, i, RSBO)) = __float2bfloat16_rn(0.0f);
  }
  // (end of the forward solve)
}

// ============================================================================
// Backward (see solve_backward_kernel in mixer.cu for the derivation):
//   D = L^{-1}(A'^T dY)/sqrt(n), lam = M^{-T} 2D, dK = -lam U^T, dTheta,
//   dZ = lam - (1+eta) D + dTheta W^T/sqrt(n), E = M' D^T + dZ Z^T,
//   R_d = L^{-T} M'/sqrt(n), R_z = L^{-T} dZ/sqrt(n), Q = L^{-T} Psi L^{-1}/n.
// ============================================================================
// One CTA per system, or (systems > gridDim.x) a persistent grid whose CTAs
// take systems blockIdx.x, blockIdx.x + gridDim.x, ...: the form that runs
// beside a weight-gradient GEMM, two CTAs per SM next to its CTA (at R <= 32
// the register cap of five CTAs per SM, 48 per thread, is what lets the three
// share an SM's register file).
template <int R>
__global__ void __launch_bounds__(kWThreads, R <= 32 ? 5 : 4)
    solve_backward_warp_kernel(const SolveBwdArgs a, int64_t systems) {
  pdl_wait();
  constexpr int LD = R + 1;
  constexpr int P = rows_per_lane<R>();
  extern __shared__ __align__(16) float fsm[];
  const int d = a.d;
  const int XLD = d + 1;
  __shared__ float red[kWWarps];
  const int tid = threadIdx.x, lane = tid & 31;
  for (int64_t bh = blockIdx.x; bh < systems; bh += gridDim.x) {
  float* L = fsm;               // [R][LD] L, then L^{-1}
  float* Mm = L + R * LD;       // [R][LD] packed LU, then L^{-1}; after pass A dTheta, then E, then Psi L^{-1}
  float* Th = Mm + R * LD;      // [R][LD]
  float* dK = Th + R * LD;      // [R][LD] M^{-1}, then dK, then dTheta, then Psi, then Q^T
  float* E = Mm;
  float* X1 = dK + R * LD;      // [R][XLD] A'^T dY, then D
  float* X2 = X1 + R * XLD;     // [R][XLD] lambda, then dZ
  float* X3 = X2 + R * XLD;     // [R][XLD] U, then M'
  float* X4 = X3 + R * XLD;     // [R][XLD] Z
  float* fdiag = X4 + R * XLD;  // [R]
  float* dinv = fdiag + R;      // [R] 1 / L_ii
  float* uinv = dinv + R;       // [R] 1 / U_ii
  float* Ws = uinv + R;         // [d][R + 1] W_drive of this head
  float* Li = L;                // L^{-1} replaces L (computed in Mm, then copied)
  float* Mi = dK;               // M^{-1} until pass A is done
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
  // X1 = A'^T dY summed over the chunks (high + low halves)
  sum_chunks<R, 1>(pbase, a.nchunks, NC, [&](int i, int c, float4 hi, float4 lo) {
    const float v[4] = {hi.x + lo.x, hi.y + lo.y, hi.z + lo.z, hi.w + lo.w};
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (c + u < d) X1[i * XLD + c + u] = v[u];
  });
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
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

  // The explicit inverses M^{-1} = U^{-1} L_u^{-1} (into dK) and L^{-1} (into Mm, then
  // over L), identity columns over the warps: three triangular-solve chains, after which
  // every solve of this kernel (D, lambda, R_d, R_z and both sides of Q) is a
  // register-blocked product instead of a chain.  No extra shared memory: at r = 64 the
  // block must stay small enough for two CTAs per SM.
  {
    float rd[P], ru[P], one[P];
    lane_rows<R>(dinv, rd);
    lane_rows<R>(uinv, ru);
#pragma unroll
    for (int p = 0; p < P; ++p) one[p] = 1.0f;
    int cb, ce;
    warp_cols(R, cb, ce);
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float y[P][kNB];
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < kNB; ++q) y[p][q] = (32 * p + lane == c0 + q) ? 1.0f : 0.0f;
      trsv_lower<R, true>(Mm, LD, 1, one, y);  // unit lower factor of M
      trsv_upper<R, false>(Mm, LD, 1, ru, y);  // U
      put_cols<R>(Mi, LD, c0, ce, y);
    }
    __syncthreads();
    for (int c0 = cb; c0 < ce; c0 += kNB) {
      float x[P][kNB];
#pragma unroll
      for (int p = 0; p < P; ++p)
#pragma unroll
        for (int q = 0; q < kNB; ++q) x[p][q] = (32 * p + lane == c0 + q) ? 1.0f : 0.0f;
      trsv_lower<R, false>(L, LD, 1, rd, x);
      put_cols<R>(Mm, LD, c0, ce, x);
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    Li[i * LD + k] = Mm[i * LD + k];
  }
  __syncthreads();
  // Pass A: D = L^{-1} (A'^T dY) / sqrt(n) into X2, then lam = M^{-T} (2 D) into X1; the two
  // buffers then swap names (X1 = D, X2 = lam).
  tile_gemm<R, 2>(
      d, R, [&](int i, int k) { return Li[i * LD + k]; }, [&](int k, int c) { return X1[k * XLD + c]; },
      [&](int i, int c, float acc) { X2[i * XLD + c] = acc * rsn; });
  __syncthreads();
  tile_gemm<R, 2>(
      d, R, [&](int i, int k) { return Mi[k * LD + i]; }, [&](int k, int c) { return X2[k * XLD + c]; },
      [&](int i, int c, float acc) { X1[i * XLD + c] = 2.0f * acc; });
  __syncthreads();
  {
    float* t = X1;
    X1 = X2;
    X2 = t;
  }
  float dz_dot = 0.0f;
  for (int idx = tid; idx < R * d; idx += kWThreads) {
    const int i = idx / d, col = idx % d;
    dz_dot = fmaf(X1[i * XLD + col], X4[i * XLD + col], dz_dot);
  }
  // dK = -lam U^T
  tile_gemm<R, square_nb<R>()>(
      R, d, [&](int i, int c) { return X2[i * XLD + c]; }, [&](int c, int j) { return X3[j * XLD + c]; },
      [&](int i, int j, float acc) { dK[i * LD + j] = -acc; });
  __syncthreads();
  // dTheta through K = F F^T + Omega (into E, then back into dK):
  //   i < j: dK_ij - dK_ji;  i >= j: sum_{k >= j} (dK_ik + dK_ki) F_kj (times softplus' on the diagonal)
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int k = idx / R, j = idx % R;
    E[k * LD + j] = k > j ? Th[k * LD + j] : (k == j ? fdiag[j] : 0.0f);
  }
  __syncthreads();
  tile_gemm<R, square_nb<R>(), true>(
      R, R, [&](int i, int k) { return dK[i * LD + k] + dK[k * LD + i]; }, [&](int k, int j) { return E[k * LD + j]; },
      [&](int i, int j, float acc) {
        float v;
        if (i < j) {
          v = dK[i * LD + j] - dK[j * LD + i];
        } else {
          v = i == j ? acc * softplus20_derivative(Th[i * LD + i] + kSoftplusOneOffset) : acc;
        }
        E[i * LD + j] = v;
      });
  __syncthreads();
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, jj = idx % R;
    const float v = E[i * LD + jj];
    dK[i * LD + jj] = v;
    a.gbase[bh * R * R + idx] = v;
  }
  __syncthreads();
  // Pass B: dZ (X2), M' = 2U - (1+eta) Z (X3), drive-gradient partial Z^T dTheta / sqrt(n)
  tile_gemm<R, 2>(
      d, R, [&](int i, int jj) { return dK[i * LD + jj]; }, [&](int jj, int col) { return Ws[col * LD + jj]; },
      [&](int i, int col, float acc) {
        X2[i * XLD + col] = X2[i * XLD + col] - (1.0f + eta) * X1[i * XLD + col] + acc * rsn;
        X3[i * XLD + col] = 2.0f * X3[i * XLD + col] - (1.0f + eta) * X4[i * XLD + col];
      });
  tile_gemm<R, 2>(
      d, R, [&](int jj, int i) { return dK[i * LD + jj]; }, [&](int i, int col) { return X4[i * XLD + col]; },
      [&](int jj, int col, float acc) { a.gdrive[(bh * d + col) * R + jj] = acc * rsn; });
  __syncthreads();
  // E = M' D^T + dZ Z^T  (k < d: the first product, k >= d: the second)
  tile_gemm<R, square_nb<R>()>(
      R, 2 * d,
      [&](int i, int k) { return k < d ? X3[i * XLD + k] : X2[i * XLD + k - d]; },
      [&](int k, int j) { return k < d ? X1[j * XLD + k] : X4[j * XLD + k - d]; },
      [&](int i, int j, float acc) { E[i * LD + j] = acc; });
  // R_d = L^{-T} M' / sqrt(n) -> B1y,  R_z = L^{-T} dZ / sqrt(n) -> B1c and B2
  uint8_t* b1y = reinterpret_cast<uint8_t*>(a.b1y + bh * R * a.d_pad);
  uint8_t* b1c = reinterpret_cast<uint8_t*>(a.b1c + bh * R * a.d_pad);
  uint8_t* b2 = reinterpret_cast<uint8_t*>(a.b2 + bh * a.d_pad * R);
  const uint32_t SBO_Y = static_cast<uint32_t>(a.d_pad) * 16;
  constexpr uint32_t SBO_R = R * 16;
  tile_gemm<R, 2>(
      d, R, [&](int i, int k) { return Li[k * LD + i]; }, [&](int k, int c) { return X3[k * XLD + c]; },
      [&](int i, int c, float acc) {
        *reinterpret_cast<bf16*>(b1y + kmajor_offset(i, c, SBO_Y)) = __float2bfloat16_rn(acc * rsn);
      });
  tile_gemm<R, 2>(
      d, R, [&](int i, int k) { return Li[k * LD + i]; }, [&](int k, int c) { return X2[k * XLD + c]; },
      [&](int i, int c, float acc) {
        const bf16 rz = __float2bfloat16_rn(acc * rsn);
        *reinterpret_cast<bf16*>(b1c + kmajor_offset(i, c, SBO_Y)) = rz;
        *reinterpret_cast<bf16*>(b2 + kmajor_offset(c, i, SBO_R)) = rz;
      });
  for (int idx = tid; idx < (a.d_pad - d) * R; idx += kWThreads) {
    const int col = d + idx / R, i = idx % R;
    const bf16 z = __float2bfloat16_rn(0.0f);
    *reinterpret_cast<bf16*>(b1y + kmajor_offset(i, col, SBO_Y)) = z;
    *reinterpret_cast<bf16*>(b1c + kmajor_offset(i, col, SBO_Y)) = z;
    *reinterpret_cast<bf16*>(b2 + kmajor_offset(col, i, SBO_R)) = z;
  }
  __syncthreads();
  // Q = L^{-T} Psi L^{-1} / n with Psi = tril(E) + tril(E,-1)^T (symmetric): Psi L^{-1}
  // into E, then L^{-T} (Psi L^{-1}) into dK, stored transposed.
  for (int idx = tid; idx < R * R; idx += kWThreads) {
    const int i = idx / R, k = idx % R;
    dK[i * LD + k] = i >= k ? E[i * LD + k] : E[k * LD + i];
  }
  __syncthreads();
  tile_gemm<R, square_nb<R>()>(
      R, R, [&](int i, int k) { return dK[i * LD + k]; }, [&](int k, int j) { return Li[k * LD + j]; },
      [&](int i, int j, float acc) { E[i * LD + j] = acc; });
  __syncthreads();
  tile_gemm<R, square_nb<R>()>(
      R, R, [&](int i, int k) { return Li[k * LD + i]; }, [&](int k, int j) { return E[k * LD + j]; },
      [&](int i, int j, float acc) { dK[j * LD + i] = acc; });
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
  __syncthreads();  // the next system overwrites this one's shared memory (and red)
  }
}

template <int R>
size_t fwd_smem(int d) {
  return sizeof(float) * (3 * R * (R + 1) + R * (d + 1) + 3 * R + d * (R + 1) + kPanel * R);
}
template <int R>
size_t bwd_smem(int d) {
  return sizeof(float) * (4 * R * (R + 1) + 4 * R * (d + 1) + 3 * R + d * (R + 1));
}

template <int R>
cudaError_t launch_fwd(const SolveFwdArgs& s, int64_t systems, cudaStream_t stream) {
  const size_t smem = fwd_smem<R>(s.d);
  cudaError_t e = allow_smem(reinterpret_cast<const void*>(&solve_forward_warp_kernel<R>), smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope("solve_fwd", stream);
  launch_pdl(solve_forward_warp_kernel<R>, static_cast<unsigned>(systems), kWThreads, smem, stream, s);
  return cudaGetLastError();
}

template <int R>
cudaError_t launch_bwd(const SolveBwdArgs& s, int64_t systems, cudaStream_t stream) {
  const size_t smem = bwd_smem<R>(s.d);
  cudaError_t e = allow_smem(reinterpret_cast<const void*>(&solve_backward_warp_kernel<R>), smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope("solve_bwd", stream);
  launch_pdl(solve_backward_warp_kernel<R>, static_cast<unsigned>(systems), kWThreads, smem, stream, s, systems);
  return cudaGetLastError();
}

template <int R>
cudaError_t launch_bwd_persistent(const SolveBwdArgs& s, int64_t systems, int grid, cudaStream_t stream) {
  const size_t smem = bwd_smem<R>(s.d);
  cudaError_t e = allow_smem(reinterpret_cast<const void*>(&solve_backward_warp_kernel<R>), smem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&solve_backward_warp_kernel<R>),
                           cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  const int64_t g = systems < grid ? systems : grid;
  LaunchScope scope("solve_bwd", stream);
  launch_pdl(solve_backward_warp_kernel<R>, static_cast<unsigned>(g), kWThreads, smem, stream, s, systems);
  return cudaGetLastError();
}

template <int R>
CtaFootprint bwd_footprint(int d) {
  cudaFuncAttributes fa{};
  CtaFootprint f{};
  if (cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(&solve_backward_warp_kernel<R>)) != cudaSuccess) {
    return f;
  }
  f.threads = kWThreads;
  f.regs = fa.numRegs;
  f.smem = bwd_smem<R>(d) + fa.sharedSizeBytes;
  return f;
}

template <int R>
bool fits(int d) {
  return fwd_smem<R>(d) <= kWarpSolveSmemLimit && bwd_smem<R>(d) <= kWarpSolveSmemLimit;
}

}  // namespace

bool warp_solves_usable(const Plan& p) {
  // One content tile per chunk partial (ndt == 1), shared memory inside one SM.
  if (p.ndt != 1) return false;
  const int d = static_cast<int>(p.d);
  switch (p.R) {
    case 16: return fits<16>(d);
    case 32: return fits<32>(d);
    case 48: return fits<48>(d);
    case 64: return fits<64>(d);
    default: return false;
  }
}

cudaError_t launch_solve_forward_warp(const Plan& p, const SolveFwdArgs& s, cudaStream_t stream) {
  switch (p.R) {
    case 16: return launch_fwd<16>(s, p.BH, stream);
    case 32: return launch_fwd<32>(s, p.BH, stream);
    case 48: return launch_fwd<48>(s, p.BH, stream);
    case 64: return launch_fwd<64>(s, p.BH, stream);
    default: return cudaErrorInvalidValue;
  }
}

CtaFootprint solve_backward_footprint(const Plan& p) {
  const int d = static_cast<int>(p.d);
  switch (p.R) {
    case 16: return bwd_footprint<16>(d);
    case 32: return bwd_footprint<32>(d);
    case 48: return bwd_footprint<48>(d);
    case 64: return bwd_footprint<64>(d);
    default: return CtaFootprint{};
  }
}

cudaError_t launch_solve_backward_persistent(const Plan& p, const SolveBwdArgs& s, int grid, cudaStream_t stream) {
  switch (p.R) {
    case 16: return launch_bwd_persistent<16>(s, p.BH, grid, stream);
    case 32: return launch_bwd_persistent<32>(s, p.BH, grid, stream);
    case 48: return launch_bwd_persistent<48>(s, p.BH, grid, stream);
    case 64: return launch_bwd_persistent<64>(s, p.BH, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_solve_backward_warp(const Plan& p, const SolveBwdArgs& s, cudaStream_t stream) {
  switch (p.R) {
    case 16: return launch_bwd<16>(s, p.BH, stream);
    case 32: return launch_bwd<32>(s, p.BH, stream);
    case 48: return launch_bwd<48>(s, p.BH, stream);
    case 64: return launch_bwd<64>(s, p.BH, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace lsso
