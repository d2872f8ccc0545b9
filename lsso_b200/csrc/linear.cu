// Projection GEMMs of the LSSO layer on sm_100a (tcgen05 + TMA).
//
//   out[t, n] = sum_k bf16(A[t, k]) * bf16(W[n, k])  (+ bias[n])   -> BF16 / FP16 / FP32
//   dW[n, k]  = sum_t bf16(G[t, n]) * bf16(X[t, k])                  -> FP32 (weight gradient)
//
// FP32 accumulation and one final rounding, masked rows zero: the
// tensor_core_linear contract of the reference (lsso/ball/reference.py:
// 58-97,170-247,347-408).  FP16 operands are rounded to BF16 in shared memory
// (never re-written to HBM), so the reference's FP16 -> BF16 cast costs no
// DRAM pass.
//
// Operands are staged by TMA with 128-byte inner boxes and
// CU_TENSOR_MAP_SWIZZLE_128B, which lands them directly in the tcgen05
// 128-byte-swizzled canonical layout (K-major for activations and weights,
// MN-major for the weight-gradient operands).  No multicast.
//
// Both kernels are warp-specialised, 512 threads, one CTA per SM:
//   warp 0      TMA producer (one lane issues);
//   warp 1      MMA issuer (one lane issues tcgen05.mma kind::f16, M=128);
//   warps 2-7   FP16 -> BF16 rounding and row masking of staged tiles;
//   warps 8-15  epilogue, two warps per TMEM sub-partition.
// Every wait is bounded and an abort flag stops all roles after a timeout.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>

#include "linear.h"
#include "mixer.h"
#include "tc.cuh"

namespace lsso {

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr uint32_t kStageBytes = kBM * kBK * 2;  // 16 KB: 128 rows x 128 bytes
constexpr int kThreads = 512;
constexpr int kConvWarps = 6;
constexpr int kConvThreads = kConvWarps * 32;
constexpr int kEpiWarps = 8;
constexpr uint32_t kEpiStage = 4096;  // per epilogue warp: two 32x32 16-bit boxes or one FP32 box

struct LinearArgs {
  const uint8_t* bprep;     // prepared weight: NT tiles of [BN x K_pad], K-major SW128 canonical
  const float* bias;        // nullable [Nout]
  const uint8_t* row_mask;  // nullable [M], nonzero = valid
  void* out;
  int64_t ldo;
  int out_dtype;            // 0 BF16, 1 FP16, 2 FP32
  int M, Nout, K_pad, BN, NT, a_fp16;
  int tma_out;              // output written by TMA tensor stores (else direct stores)
  int b_stream;             // weight k-blocks ride in the stages instead of staying resident
  int stages;               // pipeline stages (<= kStages)
  uint32_t stage_bytes;     // A box (16 KB) [+ streamed weight k-block]
  int rev;                  // M tiles in reverse order (start with the rows the producer wrote last)
  int* status;
};

// Bounded wait that also gives up as soon as another role aborted.
__device__ __forceinline__ bool lwait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  return mbar_wait_bounded(bar, parity, abort_flag, status);
}
// The same wait by a whole warp that goes on to tcgen05.ld (warp-collective):
// its lanes agree on the outcome, so after an abort none runs a load the others skip.
__device__ __forceinline__ bool lwait_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, status));
}

__device__ __forceinline__ uint32_t half2_to_bf162(uint32_t h) {
  __half2 v = *reinterpret_cast<__half2*>(&h);
  const float2 f = __half22float2(v);
  return pack_bf16(f.x, f.y);
}

__device__ __forceinline__ uint4 half8_to_bf16(uint4 x) {
  return make_uint4(half2_to_bf162(x.x), half2_to_bf162(x.y), half2_to_bf162(x.z), half2_to_bf162(x.w));
}

// Store 32 consecutive outputs of one row (compile-time indexing only, so the
// values stay in registers).
template <int OUT>
__device__ __forceinline__ void store_row32(void* out, int64_t ldo, int64_t t, int n0, const float (&v)[32], int count,
                                            bool vec) {
  if (OUT == 2) {
    float* o = static_cast<float*>(out) + t * ldo + n0;
    if (vec && count == 32) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < count) o[j] = v[j];
    }
    return;
  }
  uint16_t* o = static_cast<uint16_t*>(out) + t * ldo + n0;
  if (vec && count == 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 w;
      if (OUT == 0) {
        w = make_uint4(pack_bf16(v[j], v[j + 1]), pack_bf16(v[j + 2], v[j + 3]), pack_bf16(v[j + 4], v[j + 5]),
                       pack_bf16(v[j + 6], v[j + 7]));
      } else {
        __half2 h0 = __floats2half2_rn(v[j], v[j + 1]), h1 = __floats2half2_rn(v[j + 2], v[j + 3]);
        __half2 h2 = __floats2half2_rn(v[j + 4], v[j + 5]), h3 = __floats2half2_rn(v[j + 6], v[j + 7]);
        w = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                       *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
      }
      *reinterpret_cast<uint4*>(o + j) = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < count) {
        if (OUT == 0) {
          __nv_bfloat16 b = __float2bfloat16_rn(v[j]);
          o[j] = *reinterpret_cast<uint16_t*>(&b);
        } else {
          __half h = __float2half_rn(v[j]);
          o[j] = *reinterpret_cast<uint16_t*>(&h);
        }
      }
    }
  }
}

// Write one 32-value output row into a TMA staging box (row = lane): 16-bit
// outputs as 64-byte rows in the 64-byte swizzle (16-byte chunk c of row r at
// chunk c ^ ((r >> 1) & 3)), FP32 as 128-byte rows in the 128-byte swizzle
// (chunk c ^ (r & 7)).  Either way the eight lanes of one store phase hit
// distinct banks.
template <int OUT>
__device__ __forceinline__ void stage_row32(uint8_t* box, int r, const float (&v)[32]) {
  if (OUT == 2) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      *reinterpret_cast<float4*>(box + r * 128 + ((c ^ (r & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
    }
  } else {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = 8 * c;
      uint4 w;
      if (OUT == 0) {
        w = make_uint4(pack_bf16(v[j], v[j + 1]), pack_bf16(v[j + 2], v[j + 3]), pack_bf16(v[j + 4], v[j + 5]),
                       pack_bf16(v[j + 6], v[j + 7]));
      } else {
        __half2 h0 = __floats2half2_rn(v[j], v[j + 1]), h1 = __floats2half2_rn(v[j + 2], v[j + 3]);
        __half2 h2 = __floats2half2_rn(v[j + 4], v[j + 5]), h3 = __floats2half2_rn(v[j + 6], v[j + 7]);
        w = make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                       *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
      }
      *reinterpret_cast<uint4*>(box + r * 64 + ((c ^ ((r >> 1) & 3)) << 4)) = w;
    }
  }
}

// ============================================================================
// Forward-type projection: out = A W^T (+ bias), persistent over M tiles.
// Each CTA owns one N tile of the weight (resident in shared memory) and
// streams 128 x 64 activation boxes through a 4-stage ring; two TMEM
// accumulators let the epilogue of tile i overlap the MMAs of tile i+1.  The
// epilogue stages each 32-row x 32-column box in shared memory and writes it
// with one TMA tensor store, so a warp's output leaves as whole lines instead
// of 32 row-strided 16-byte pieces per store instruction.
// ============================================================================
template <int OUT>
__global__ void __launch_bounds__(kThreads, 1) linear_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                             const __grid_constant__ CUtensorMap tmap_out,
                                                             const LinearArgs a) {
  pdl_wait();
  extern __shared__ __align__(1024) uint8_t smem[];
  // Resident weight: [weight tile | stages | epilogue staging]; streamed: [stages | staging].
  uint8_t* sB = smem;
  uint8_t* sA = a.b_stream ? smem : smem + static_cast<size_t>(a.BN) * a.K_pad * 2;  // a multiple of 1024
  const uint32_t SB = a.stage_bytes;
  const int S = a.stages;
  uint8_t* sOut = sA + S * SB;
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], conv[kStages], tfull[2], tempty[2], bbar, mdrain;
  __shared__ uint32_t tmem_s;
  __shared__ int abort_flag;
  __shared__ __align__(16) float sbias[256];  // this N tile's bias (zero past Nout)
  volatile int* abort_v = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = static_cast<int>(blockIdx.x % a.NT);
  const int mstart = static_cast<int>(blockIdx.x / a.NT);
  const int mstep = static_cast<int>(gridDim.x / a.NT);
  const int mtiles = (a.M + kBM - 1) / kBM;
  const int ntile_local = mstart < mtiles ? (mtiles - mstart + mstep - 1) / mstep : 0;
  const int KB = a.K_pad / kBK;
  const int BN = a.BN;
  const uint32_t tcols = tmem_cols_for(2 * BN);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
      mbar_init(smem_u32(&conv[s]), kConvWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), kEpiWarps);
    }
    mbar_init(smem_u32(&bbar), 1);
    mbar_init(smem_u32(&mdrain), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (a.bias != nullptr) {
    for (int i = threadIdx.x; i < BN; i += blockDim.x) {
      const int n = nt * BN + i;
      sbias[i] = n < a.Nout ? a.bias[n] : 0.0f;
    }
  }
  if (warp == 1) tmem_alloc(smem_u32(&tmem_s), tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;

  if (warp == 0) {
    // ---------------- producer
    const uint32_t bbytes = static_cast<uint32_t>(BN) * a.K_pad * 2;
    const uint8_t* bsrc = a.bprep + static_cast<size_t>(nt) * bbytes;
    const uint32_t b_region = static_cast<uint32_t>(BN) * 128;  // one 64-wide K region of the weight tile
    if (lane == 0) {
      prefetch_tmap(&tmap_a);
      if (!a.b_stream) {
        mbar_arrive_expect_tx(smem_u32(&bbar), bbytes);
        for (uint32_t off = 0; off < bbytes; off += 32768u) {
          const uint32_t chunk = min(32768u, bbytes - off);
          bulk_load(smem_u32(sB + off), bsrc + off, chunk, smem_u32(&bbar));
        }
      }
    }
    __syncwarp();
    RingPos rp;
    bool ok = true;
    int last_use[kStages];  // lane 0: the use of each stage whose load was issued last
    for (int s = 0; s < kStages; ++s) last_use[s] = -1;
    for (int i = 0; i < ntile_local && ok; ++i) {
      const int m = a.rev ? mtiles - 1 - (mstart + i * mstep) : mstart + i * mstep;
      for (int kb = 0; kb < KB && ok; ++kb, rp.next(S)) {
        const int s = rp.s, u = rp.u;
        ok = lwait(smem_u32(&empty[s]), (u & 1) ^ 1, abort_v, a.status);
        if (ok && lane == 0) {
          uint8_t* stage = sA + s * SB;
          mbar_arrive_expect_tx(smem_u32(&full[s]), SB);
          tma_load_2d(smem_u32(stage), &tmap_a, kb * kBK, m * kBM, smem_u32(&full[s]));
          // Streamed weight: k-block kb of this N tile (L2-resident, reused by every M tile).
          if (a.b_stream) bulk_load(smem_u32(stage + kStageBytes), bsrc + kb * b_region, b_region, smem_u32(&full[s]));
          last_use[s] = u;
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      // loads still in flight (only after an abort): wait for them, bounded
      if (!a.b_stream) mbar_wait(smem_u32(&bbar), 0, a.status);
      for (int s = 0; s < S; ++s) {
        if (last_use[s] >= 0) mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>(last_use[s]) & 1u, a.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer
    bool ok = a.b_stream ? true : lwait(smem_u32(&bbar), 0, abort_v, a.status);
    const uint32_t idesc = make_idesc(kBM, BN, false, false);
    const uint32_t sa0 = smem_u32(sA), sb0 = smem_u32(sB);
    const uint32_t b_region = static_cast<uint32_t>(BN) * 128;  // one 64-wide K region of the weight tile
    RingPos rp;
    for (int i = 0; i < ntile_local && ok; ++i) {
      const int b = i & 1, v = i >> 1;
      ok = lwait(smem_u32(&tempty[b]), (v & 1) ^ 1, abort_v, a.status);
      tc_fence_after();
      const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
      for (int kb = 0; kb < KB && ok; ++kb, rp.next(S)) {
        const int s = rp.s, u = rp.u;
        ok = lwait(smem_u32(a.a_fp16 ? &conv[s] : &full[s]), u & 1, abort_v, a.status);
        tc_fence_after();
        if (ok && lane == 0) {
          const uint32_t stage = sa0 + s * SB;
          const uint32_t bk = a.b_stream ? stage + kStageBytes : sb0 + kb * b_region;
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks) {
            const uint64_t ad = make_desc_sw128(stage + ks * 32, 16, 1024);
            const uint64_t bd = make_desc_sw128(bk + ks * 32, 16, 1024);
            mma_bf16(d, ad, bd, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          mma_commit(smem_u32(&empty[s]));
        }
        __syncwarp();
      }
      if (ok && lane == 0) mma_commit(smem_u32(&tfull[b]));
      __syncwarp();
    }
    if (lane == 0) mma_drain(smem_u32(&mdrain), a.status);
    __syncwarp();
  } else if (warp < 2 + kConvWarps) {
    // ---------------- FP16 -> BF16 rounding in shared memory
    if (a.a_fp16) {
      const int ct = threadIdx.x - 64;
      RingPos rp;
      bool ok = true;
      for (int i = 0; i < ntile_local && ok; ++i) {
        for (int kb = 0; kb < KB && ok; ++kb, rp.next(S)) {
          const int s = rp.s, u = rp.u;
          ok = lwait(smem_u32(&full[s]), u & 1, abort_v, a.status);
          if (ok) {
            uint4* p = reinterpret_cast<uint4*>(sA + s * SB);  // the A box (first 16 KB of the stage)
            // every chunk of the thread read before any is written back, so the
            // shared-memory loads overlap instead of waiting behind the stores
            constexpr int kPer = (kStageBytes / 16 + kConvThreads - 1) / kConvThreads;
            uint4 v[kPer];
#pragma unroll
            for (int q = 0; q < kPer; ++q) {
              const int j = ct + q * kConvThreads;
              if (j < static_cast<int>(kStageBytes / 16)) v[q] = p[j];
            }
#pragma unroll
            for (int q = 0; q < kPer; ++q) {
              const int j = ct + q * kConvThreads;
              if (j < static_cast<int>(kStageBytes / 16)) p[j] = half8_to_bf16(v[q]);
            }
            fence_proxy_async();
          }
          __syncwarp();
          if (ok && lane == 0) mbar_arrive(smem_u32(&conv[s]));
        }
      }
    }
  } else {
    // ---------------- epilogue: two warps per TMEM sub-partition
    const int sub = warp & 3;
    const int half = (warp - (2 + kConvWarps)) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(32 * sub) << 16);
    const bool vec = (a.ldo % (OUT == 2 ? 4 : 8)) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15u) == 0;
    uint8_t* stage = sOut + (warp - (2 + kConvWarps)) * kEpiStage;
    int sbuf = 0;
    if (a.tma_out && lane == 0) prefetch_tmap(&tmap_out);
    bool ok = true;
    for (int i = 0; i < ntile_local && ok; ++i) {
      const int b = i & 1, v = i >> 1;
      const int m = a.rev ? mtiles - 1 - (mstart + i * mstep) : mstart + i * mstep;
      ok = lwait_warp(smem_u32(&tfull[b]), v & 1, abort_v, a.status);
      tc_fence_after();
      if (ok) {
        const int64_t row0 = static_cast<int64_t>(m) * kBM + 32 * sub;
        const int64_t t = row0 + lane;
        const bool inside = t < a.M;
        const bool live = inside && (a.row_mask == nullptr || a.row_mask[t] != 0);
        for (int c0 = 32 * half; c0 < BN; c0 += 64) {
          float vals[32];
          tmem_ld32(lane_addr + static_cast<uint32_t>(b * BN + c0), vals);
          tmem_ld_wait();
          const int n0 = nt * BN + c0;
          const int count = min(32, a.Nout - n0);
          if (count <= 0 || row0 >= a.M) continue;  // warp-uniform
          // Bias from shared memory, masked rows zero.  (A per-element
          // predicated global bias load here made the epilogue, and with it
          // the whole GEMM, several times slower.)
          if (a.bias != nullptr) {
            const float4* bsm = reinterpret_cast<const float4*>(sbias + c0);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 bv = bsm[j];
              vals[4 * j] += bv.x;
              vals[4 * j + 1] += bv.y;
              vals[4 * j + 2] += bv.z;
              vals[4 * j + 3] += bv.w;
            }
          }
          if (!live) {
#pragma unroll
            for (int j = 0; j < 32; ++j) vals[j] = 0.0f;
          }
          if (a.tma_out) {
            uint8_t* box = stage + (OUT == 2 ? 0 : sbuf * 2048);
            // The store that last read this box (two commits ago; one for FP32) is done reading.
            if (lane == 0) {
              if (OUT == 2) {
                bulk_wait_read<0>();
              } else {
                bulk_wait_read<1>();
              }
            }
            __syncwarp();
            stage_row32<OUT>(box, lane, vals);
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmap_out, smem_u32(box), n0, static_cast<int>(row0));
              bulk_commit();
            }
            sbuf ^= 1;
          } else if (inside) {
            store_row32<OUT>(a.out, a.ldo, t, n0, vals, count, vec);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[b]));
    }
    if (a.tma_out && lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

// Weight (FP32, [Nout, K] or transposed [K, Nout]) -> BF16 K-major SW128
// canonical tiles of BN rows: 64-wide K regions of BN rows x 128 bytes; row n
// at (n/8)*1024 + (n%8)*128, its 16-byte chunk c stored at chunk c ^ (n%8).
// Zero outside [Nout, K].  Element idx of the image (32-bit index arithmetic:
// a weight tile set is far below 2^31 elements).
__device__ __forceinline__ void prep_weight_element(const float* __restrict__ w, int Nout, int K, int transposed,
                                                    int BN, int K_pad, uint8_t* __restrict__ out, int idx) {
  const int tile = BN * K_pad;
  const int j = idx / tile;
  const int rem = idx - j * tile;
  const int nl = rem / K_pad, k = rem - nl * K_pad;
  const int n = j * BN + nl;
  float v = 0.0f;
  if (n < Nout && k < K) v = transposed ? w[static_cast<int64_t>(k) * Nout + n] : w[static_cast<int64_t>(n) * K + k];
  const int kk = k % kBK;
  const size_t off = static_cast<size_t>(j) * tile * 2 + static_cast<size_t>(k / kBK) * BN * 128 +
                     static_cast<size_t>(nl / 8) * 1024 + (nl % 8) * 128 + ((((kk * 2) / 16) ^ (nl % 8)) * 16) +
                     (kk * 2) % 16;
  *reinterpret_cast<__nv_bfloat16*>(out + off) = __float2bfloat16_rn(v);
}

__global__ void prep_weight_kernel(const float* __restrict__ w, int Nout, int K, int transposed, int BN, int K_pad,
                                   int NT, uint8_t* __restrict__ out) {
  pdl_wait();
  const int total = NT * BN * K_pad;
  const int idx = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  prep_weight_element(w, Nout, K, transposed, BN, K_pad, out, idx);
}

// Several images in one launch: the grid covers their elements back to back
// (image e owns [end[e-1], end[e])).
struct PrepBatch {
  const float* w[kMaxImages];
  uint8_t* out[kMaxImages];
  int Nout[kMaxImages], K[kMaxImages], transposed[kMaxImages], BN[kMaxImages], K_pad[kMaxImages];
  int end[kMaxImages];
  int count;
};

__global__ void prep_weights_kernel(const __grid_constant__ PrepBatch b) {
  pdl_wait();
  const int idx = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  int e = 0, begin = 0;
  while (e < b.count && idx >= b.end[e]) begin = b.end[e++];
  if (e >= b.count) return;
  prep_weight_element(b.w[e], b.Nout[e], b.K[e], b.transposed[e], b.BN[e], b.K_pad[e], b.out[e], idx - begin);
}

// ============================================================================
// Weight gradient: dW[n, k] = sum_t bf16(G[t, n]) * bf16(X[t, k]) over tokens
// whose row_mask is set, FP32 (reference.py:229-234).  The kernel computes
// C[m, c] = sum_t A[t, m] B[t, c] with M = 128 features of A per tile, N = BNW
// features of B (a multiple of 64, up to 512: two N = 256 MMAs per K-step),
// K = tokens; both operands MN-major SW128, each stage 64 tokens, one 8 KB TMA
// box per 64 features.  The plan puts an FP16 operand on the A side when only
// one operand is FP16, so each of its elements is rounded to BF16 once (the
// B side is re-read by every A tile); C is then dW^T and the reduce writes it
// transposed.  The token axis is split over CTAs; each CTA accumulates one
// 128 x BNW tile in TMEM and writes an FP32 partial; wgrad_reduce sums the
// partials in split order (deterministic, no atomics).
// ============================================================================
constexpr int kWT = 64;  // tokens per stage
constexpr int kWMaxStages = 4;
constexpr uint32_t kWBox = 64 * kWT * 2;  // 8 KB: 64 tokens x 64 features

struct WgradArgs {
  const uint8_t* row_mask;  // nullable [T]
  float* partial;           // [splits][tiles][128][BNW]
  int T, BNW, mtiles, ntilesw, splits, tokens_per_split, a_fp16, b_fp16, stages;
  int* status;
};

__global__ void __launch_bounds__(kThreads, 1) wgrad_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                            const __grid_constant__ CUtensorMap tmap_b,
                                                            const WgradArgs a) {
  pdl_wait();
  extern __shared__ __align__(1024) uint8_t smem[];
  const int BNW = a.BNW;
  const int S = a.stages;
  const uint32_t a_bytes = 2 * kWBox;                                // 128 features
  const uint32_t b_bytes = static_cast<uint32_t>(BNW / 64) * kWBox;  // BNW features
  const uint32_t stage_bytes = a_bytes + b_bytes;
  __shared__ __align__(8) uint64_t full[kWMaxStages], empty[kWMaxStages], conv[kWMaxStages], done, mdrain;
  __shared__ uint32_t tmem_s;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = a.mtiles * a.ntilesw;
  const int tile = static_cast<int>(blockIdx.x % tiles);
  const int split = static_cast<int>(blockIdx.x / tiles);
  const int mt = tile / a.ntilesw, ntw = tile % a.ntilesw;
  const int t_begin = split * a.tokens_per_split;
  const int t_end = min(a.T, t_begin + a.tokens_per_split);
  const int nst = t_begin < t_end ? (t_end - t_begin + kWT - 1) / kWT : 0;
  const bool masked = a.row_mask != nullptr;
  const bool need_conv = a.a_fp16 || a.b_fp16 || masked;
  const uint32_t tcols = tmem_cols_for(BNW);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
      mbar_init(smem_u32(&conv[s]), kConvWarps);
    }
    mbar_init(smem_u32(&done), 1);
    mbar_init(smem_u32(&mdrain), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(&tmem_s), tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_s;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmap_a);
      prefetch_tmap(&tmap_b);
    }
    bool ok = true;
    RingPos rp;
    int last_use[kWMaxStages];  // lane 0: the use of each stage whose load was issued last
    for (int s = 0; s < kWMaxStages; ++s) last_use[s] = -1;
    for (int i = 0; i < nst && ok; ++i, rp.next(S)) {
      const int s = rp.s, u = rp.u;
      ok = lwait(smem_u32(&empty[s]), (u & 1) ^ 1, abort_v, a.status);
      if (ok && lane == 0) {
        const uint32_t dst = smem_u32(smem + s * stage_bytes);
        const int t0 = t_begin + i * kWT;
        mbar_arrive_expect_tx(smem_u32(&full[s]), stage_bytes);
        tma_load_2d(dst, &tmap_a, mt * 128, t0, smem_u32(&full[s]));
        tma_load_2d(dst + kWBox, &tmap_a, mt * 128 + 64, t0, smem_u32(&full[s]));
        for (int g = 0; g < BNW / 64; ++g) {
          tma_load_2d(dst + a_bytes + g * kWBox, &tmap_b, ntw * BNW + g * 64, t0, smem_u32(&full[s]));
        }
        last_use[s] = u;
      }
      __syncwarp();
    }
    if (lane == 0) {
      // loads still in flight (only after an abort): wait for them, bounded
      for (int s = 0; s < S; ++s) {
        if (last_use[s] >= 0) mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>(last_use[s]) & 1u, a.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    bool ok = true;
    RingPos rp;
    for (int i = 0; i < nst && ok; ++i, rp.next(S)) {
      const int s = rp.s, u = rp.u;
      ok = lwait(smem_u32(need_conv ? &conv[s] : &full[s]), u & 1, abort_v, a.status);
      tc_fence_after();
      if (ok && lane == 0) {
        const uint32_t base = smem_u32(smem + s * stage_bytes);
#pragma unroll
        for (int ks = 0; ks < kWT / 16; ++ks) {
          const uint64_t ad = make_desc_sw128(base + ks * 2048, kWBox, 1024);
          for (int nb = 0; nb < BNW; nb += 256) {
            const int n = min(256, BNW - nb);
            const uint64_t bd = make_desc_sw128(base + a_bytes + (nb / 64) * kWBox + ks * 2048, kWBox, 1024);
            mma_bf16(tmem + static_cast<uint32_t>(nb), ad, bd, make_idesc(128, n, true, true), (i | ks) != 0 ? 1u : 0u);
          }
        }
        mma_commit(smem_u32(&empty[s]));
      }
      __syncwarp();
    }
    if (lane == 0) {
      if (ok && nst > 0) {
        mma_commit(smem_u32(&done));
      } else {
        mbar_arrive(smem_u32(&done));
      }
      mma_drain(smem_u32(&mdrain), a.status);
    }
    __syncwarp();
  } else if (warp < 2 + kConvWarps) {
    if (need_conv) {
      // Only the regions that need work: an FP16 operand (rounded to BF16) or,
      // with a row mask, every chunk (masked tokens zeroed).
      const int ct = threadIdx.x - 64;
      const int a_chunks = static_cast<int>(a_bytes / 16), total = static_cast<int>(stage_bytes / 16);
      const int j0 = (masked || a.a_fp16) ? 0 : a_chunks;
      const int j1 = (masked || a.b_fp16) ? total : a_chunks;
      bool ok = true;
      RingPos rp;
      for (int i = 0; i < nst && ok; ++i, rp.next(S)) {
        const int s = rp.s, u = rp.u;
        ok = lwait(smem_u32(&full[s]), u & 1, abort_v, a.status);
        if (ok) {
          uint4* p = reinterpret_cast<uint4*>(smem + s * stage_bytes);
          const int t0 = t_begin + i * kWT;
          // in batches of four chunks, each read before any of it is written back
          for (int jb = j0 + ct; jb < j1; jb += 4 * kConvThreads) {
            uint4 v[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int j = jb + q * kConvThreads;
              if (j < j1) v[q] = p[j];
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int j = jb + q * kConvThreads;
              if (j >= j1) break;
              const bool is_a = j < a_chunks;
              uint4 w = v[q];
              if (is_a ? a.a_fp16 : a.b_fp16) w = half8_to_bf16(w);
              if (masked) {
                const int t = t0 + ((j % 512) >> 3);  // each 128-byte row of a box is one token
                if (t >= a.T || a.row_mask[t] == 0) w = make_uint4(0u, 0u, 0u, 0u);
              }
              p[j] = w;
            }
          }
          fence_proxy_async();
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(smem_u32(&conv[s]));
      }
    }
  } else {
    const int sub = warp & 3;
    const int half = (warp - (2 + kConvWarps)) >> 2;
    const int row = 32 * sub + lane;  // feature m within the tile
    bool ok = lwait_warp(smem_u32(&done), 0, abort_v, a.status);
    tc_fence_after();
    float* out = a.partial + (static_cast<size_t>(split) * tiles + tile) * 128 * BNW + static_cast<size_t>(row) * BNW;
    for (int c0 = 32 * half; c0 < BNW; c0 += 64) {
      float vals[32];
      if (ok && nst > 0) {
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * sub) << 16) + c0, vals);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) vals[j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(out + c0 + j) = make_float4(vals[j], vals[j + 1], vals[j + 2], vals[j + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tcols);
  }
}

// C[m, c] = sum over splits of the partial tiles, four adjacent columns per
// group of kSplitLanes lanes: lane g sums splits g, g + 8, ... (float4 reads,
// all independent, so a lane keeps its whole share in flight), then the eight
// lane sums are combined by a fixed butterfly (deterministic order).  Written
// to dw[m, c] ([Mdim, Ndim]) or, when the operands were swapped, to dw[c, m].
constexpr int kSplitLanes = 8;
__global__ void wgrad_reduce_kernel(const float* __restrict__ partial, int splits, int mtiles, int ntilesw, int BNW,
                                    int Mdim, int Ndim, int swapped, float* __restrict__ dw) {
  pdl_wait();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t q = t / kSplitLanes;
  const int g = static_cast<int>(t % kSplitLanes);
  const bool live = q < static_cast<int64_t>(Mdim) * Ndim / 4;  // whole lane groups share this
  const int64_t idx = 4 * (live ? q : 0);
  const int m = static_cast<int>(idx / Ndim), c = static_cast<int>(idx % Ndim);  // Ndim % 4 == 0
  const int tiles = mtiles * ntilesw;
  const int tile = (m / 128) * ntilesw + c / BNW;
  const size_t inner = static_cast<size_t>(m % 128) * BNW + (c % BNW);
  const float4* src = reinterpret_cast<const float4*>(partial + static_cast<size_t>(tile) * 128 * BNW + inner);
  const size_t stride4 = static_cast<size_t>(tiles) * 128 * BNW / 4;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (live) {
#pragma unroll 4
    for (int sp = g; sp < splits; sp += kSplitLanes) {
      const float4 v = __ldg(src + sp * stride4);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
  }
#pragma unroll
  for (int o = 1; o < kSplitLanes; o <<= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
    acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
  }
  if (!live || g != 0) return;
  if (swapped) {
    dw[static_cast<int64_t>(c) * Mdim + m] = acc.x;
    dw[static_cast<int64_t>(c + 1) * Mdim + m] = acc.y;
    dw[static_cast<int64_t>(c + 2) * Mdim + m] = acc.z;
    dw[static_cast<int64_t>(c + 3) * Mdim + m] = acc.w;
  } else {
    *reinterpret_cast<float4*>(dw + idx) = acc;
  }
}

// Row-major [rows, cols] 16-bit tensor, 64-column x box_rows boxes, 128-byte swizzle.
CUresult encode_rows(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* ptr, int64_t rows,
                     int64_t cols, int fp16, int box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return encode(map, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  }
  return fn;
}

LinearPlan make_linear_plan(int64_t M, int64_t K, int64_t Nout, int sm_count) {
  LinearPlan p{};
  p.M = M;
  p.K = K;
  p.Nout = Nout;
  p.K_pad = (K + kBK - 1) / kBK * kBK;
  const int64_t n16 = (Nout + 15) / 16 * 16;
  int bn = 256;
  while (bn > 16 && (static_cast<int64_t>(bn) * p.K_pad * 2 > 128 * 1024 || bn / 2 >= n16)) bn /= 2;
  // When keeping the weight tile resident would force a narrower tile (long K),
  // stream its k-blocks through the stages instead and keep the wide tile: the
  // A tile then goes through fewer, wider MMAs and is read once per N tile less.
  int bn_wide = 256;
  while (bn_wide > 16 && bn_wide / 2 >= n16) bn_wide /= 2;
  p.b_stream = bn_wide > bn ? 1 : 0;
  if (p.b_stream) bn = bn_wide;
  p.BN = bn;
  p.NT = static_cast<int>((Nout + bn - 1) / bn);
  const int64_t mtiles = (M + kBM - 1) / kBM;
  int64_t groups = (sm_count > 0 ? sm_count : 148) / p.NT;
  if (groups < 1) groups = 1;
  if (groups > mtiles) groups = mtiles;
  p.grid = static_cast<int>(groups * p.NT);
  if (p.b_stream) {
    p.stage_bytes = kStageBytes + static_cast<uint32_t>(bn) * 128;
    const size_t room = 230400 - 1024 - static_cast<size_t>(kEpiWarps) * kEpiStage;
    p.stages = static_cast<int>(room / p.stage_bytes);
    if (p.stages > kStages) p.stages = kStages;
    p.smem = static_cast<size_t>(p.stages) * p.stage_bytes + kEpiWarps * kEpiStage;
  } else {
    p.stage_bytes = kStageBytes;
    p.stages = kStages;
    p.smem = static_cast<size_t>(bn) * p.K_pad * 2 + kStages * kStageBytes + kEpiWarps * kEpiStage;
  }
  p.prep_bytes = static_cast<size_t>(p.NT) * bn * p.K_pad * 2;
  return p;
}

bool linear_shape_supported(int64_t K) { return K % 8 == 0 && K > 0 && K <= 1024; }

WgradPlan make_wgrad_plan(int64_t T, int64_t Nout, int64_t K, int sm_count, int g_fp16, int x_fp16,
                          int max_stages) {
  WgradPlan p{};
  p.T = T;
  p.Nout = Nout;
  p.K = K;
  // An FP16 operand goes on the A (M) side, where each element is rounded once.
  p.swapped = (x_fp16 && !g_fp16) ? 1 : 0;
  p.Mdim = p.swapped ? K : Nout;
  p.Ndim = p.swapped ? Nout : K;
  // A multiple of 64 (MN-major operands come in 64-feature TMA boxes), at most
  // 256: the kernel takes up to 512, but a 256-wide tile keeps four 48 KB
  // stages in flight where a 512-wide one keeps two of 80 KB (measured: the
  // input-projection weight gradient 12% faster, with half the partials, although
  // each FP16 tile is then rounded by two CTAs).
  p.BNW = p.Ndim <= 256 ? static_cast<int>((p.Ndim + 63) / 64 * 64) : 256;
  p.mtiles = static_cast<int>((p.Mdim + 127) / 128);
  p.ntilesw = static_cast<int>((p.Ndim + p.BNW - 1) / p.BNW);
  const size_t stage = static_cast<size_t>(2 + p.BNW / 64) * kWBox;
  p.stages = static_cast<int>((200 * 1024) / stage);
  if (p.stages > kWMaxStages) p.stages = kWMaxStages;
  if (max_stages >= 2 && p.stages > max_stages) p.stages = max_stages;
  const int tiles = p.mtiles * p.ntilesw;
  const int sms = sm_count > 0 ? sm_count : 148;
  int splits = sms / tiles;
  if (splits < 1) splits = 1;
  const int64_t max_splits = (T + kWT - 1) / kWT;
  if (splits > max_splits) splits = static_cast<int>(max_splits);
  int64_t per = (T + splits - 1) / splits;
  per = (per + kWT - 1) / kWT * kWT;
  p.tokens_per_split = static_cast<int>(per);
  p.splits = static_cast<int>((T + per - 1) / per);
  p.grid = p.splits * tiles;
  p.smem = static_cast<size_t>(p.stages) * stage;
  p.partial_bytes = static_cast<size_t>(p.splits) * tiles * 128 * p.BNW * sizeof(float);
  return p;
}

size_t image_bytes(int64_t K, int64_t Nout, int sm_count) { return make_linear_plan(1, K, Nout, sm_count).prep_bytes; }

cudaError_t launch_prepare_images(const WeightImage* images, int count, int sm_count, cudaStream_t stream) {
  if (count < 1 || count > kMaxImages) return cudaErrorInvalidValue;
  PrepBatch b{};
  int64_t total = 0;
  for (int e = 0; e < count; ++e) {
    const WeightImage& im = images[e];
    const LinearPlan p = make_linear_plan(1, im.K, im.Nout, sm_count);
    b.w[e] = im.weight;
    b.out[e] = im.image;
    b.Nout[e] = static_cast<int>(p.Nout);
    b.K[e] = static_cast<int>(p.K);
    b.transposed[e] = im.transposed;
    b.BN[e] = p.BN;
    b.K_pad[e] = static_cast<int>(p.K_pad);
    total += static_cast<int64_t>(p.NT) * p.BN * p.K_pad;
    if (total >= (int64_t{1} << 31)) return cudaErrorInvalidValue;
    b.end[e] = static_cast<int>(total);
  }
  b.count = count;
  LaunchScope scope("prep_weight", stream);
  launch_pdl(prep_weights_kernel, static_cast<unsigned>((total + 255) / 256), 256, 0, stream, b);
  return cudaGetLastError();
}

cudaError_t launch_linear(const LinearPlan& p, const LinearCall& c, cudaStream_t stream) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return cudaErrorNotSupported;
  if (!c.prepared) {
    const int64_t total = static_cast<int64_t>(p.NT) * p.BN * p.K_pad;
    LaunchScope scope("prep_weight", stream);
    if (total >= (int64_t{1} << 31)) return cudaErrorInvalidValue;
    launch_pdl(prep_weight_kernel, static_cast<unsigned>((total + 255) / 256), 256, 0, stream, 
        c.weight, static_cast<int>(p.Nout), static_cast<int>(p.K), c.weight_transposed, p.BN,
        static_cast<int>(p.K_pad), p.NT, c.prep);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  CUtensorMap tmap{}, tmap_out{};
  if (encode_rows(encode, &tmap, c.a, p.M, p.K, c.a_fp16, kBM) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const int64_t esize = c.out_dtype == 2 ? 4 : 2;
  bool tma_out = (reinterpret_cast<uintptr_t>(c.out) & 15u) == 0 && (c.ldo * esize) % 16 == 0 && p.Nout >= 32 &&
                 p.M >= 32;
  if (tma_out) {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.Nout), static_cast<cuuint64_t>(p.M)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(c.ldo * esize)};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = c.out_dtype == 0   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : c.out_dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    tma_out = encode(&tmap_out, dt, 2, c.out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     c.out_dtype == 2 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  }
  LinearArgs a{};
  a.tma_out = tma_out ? 1 : 0;
  a.b_stream = p.b_stream;
  a.stages = p.stages;
  a.stage_bytes = p.stage_bytes;
  a.bprep = c.prep;
  a.bias = c.bias;
  a.row_mask = c.row_mask;
  a.out = c.out;
  a.ldo = c.ldo;
  a.out_dtype = c.out_dtype;
  a.M = static_cast<int>(p.M);
  a.Nout = static_cast<int>(p.Nout);
  a.K_pad = static_cast<int>(p.K_pad);
  a.BN = p.BN;
  a.NT = p.NT;
  a.a_fp16 = c.a_fp16;
  a.rev = c.reverse;
  a.status = c.status;
  cudaError_t e = cudaSuccess;
  LaunchScope scope("linear", stream);
  switch (c.out_dtype) {
    case 0:
      e = allow_smem(reinterpret_cast<const void*>(&linear_kernel<0>), p.smem);
      if (e == cudaSuccess) launch_pdl(linear_kernel<0>, p.grid, kThreads, p.smem, stream, tmap, tmap_out, a);
      break;
    case 1:
      e = allow_smem(reinterpret_cast<const void*>(&linear_kernel<1>), p.smem);
      if (e == cudaSuccess) launch_pdl(linear_kernel<1>, p.grid, kThreads, p.smem, stream, tmap, tmap_out, a);
      break;
    default:
      e = allow_smem(reinterpret_cast<const void*>(&linear_kernel<2>), p.smem);
      if (e == cudaSuccess) launch_pdl(linear_kernel<2>, p.grid, kThreads, p.smem, stream, tmap, tmap_out, a);
      break;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

CtaFootprint wgrad_footprint(const WgradPlan& p) {
  cudaFuncAttributes fa{};
  CtaFootprint f{};
  if (cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(&wgrad_kernel)) != cudaSuccess) return f;
  f.threads = kThreads;
  f.regs = fa.numRegs;
  f.smem = p.smem + fa.sharedSizeBytes;
  return f;
}

cudaError_t launch_wgrad(const WgradPlan& p, const WgradCall& c, cudaStream_t stream) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (encode == nullptr) return cudaErrorNotSupported;
  const void* pa = p.swapped ? c.x : c.g;
  const void* pb = p.swapped ? c.g : c.x;
  const int a16 = p.swapped ? c.x_fp16 : c.g_fp16;
  const int b16 = p.swapped ? c.g_fp16 : c.x_fp16;
  CUtensorMap ma{}, mb{};
  if (encode_rows(encode, &ma, pa, p.T, p.Mdim, a16, kWT) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_rows(encode, &mb, pb, p.T, p.Ndim, b16, kWT) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  WgradArgs a{};
  a.row_mask = c.row_mask;
  a.partial = c.partial;
  a.T = static_cast<int>(p.T);
  a.BNW = p.BNW;
  a.mtiles = p.mtiles;
  a.ntilesw = p.ntilesw;
  a.splits = p.splits;
  a.tokens_per_split = p.tokens_per_split;
  a.a_fp16 = a16;
  a.b_fp16 = b16;
  a.stages = p.stages;
  a.status = c.status;
  cudaError_t e = allow_smem(reinterpret_cast<const void*>(&wgrad_kernel), p.smem);
  if (e != cudaSuccess) return e;
  if (p.stages < kWMaxStages) {
    // sharing its SMs with another kernel: the carveout that leaves room for both
    e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&wgrad_kernel),
                             cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
  }
  {
    LaunchScope scope("wgrad", stream);
    launch_pdl(wgrad_kernel, p.grid, kThreads, p.smem, stream, ma, mb, a);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t lanes = p.Mdim * p.Ndim / 4 * kSplitLanes;
  LaunchScope scope("wgrad_reduce", stream);
  launch_pdl(wgrad_reduce_kernel, static_cast<unsigned>((lanes + 255) / 256), 256, 0, stream, 
      c.partial, p.splits, p.mtiles, p.ntilesw, p.BNW, static_cast<int>(p.Mdim), static_cast<int>(p.Ndim), p.swapped,
      c.dw);
  return cudaGetLastError();
}

}  // namespace lsso
