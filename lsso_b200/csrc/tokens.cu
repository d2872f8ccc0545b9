// Token passes of the LSSO mixer on head-group tiles (sm_100a).
//
// A work item is one 128-token tile of one sample for a group of `hg` heads
// whose relation features (hg * R) and content features (hg * d) each fill
// whole 64-feature boxes.  One persistent CTA per SM walks the items; inside
// a CTA the work is split by warp role:
//
//   warp 0        TMA producer: 128-token x 64-feature boxes of the packed
//                 projection [B][N][W] (and of dY [B][N][D]) through 3-D
//                 tensor maps with the 128-byte swizzle (tokens past N read
//                 as zero), plus bulk copies of the per-(b, h) operand
//                 matrices the solves produced;
//   warp 1        tcgen05 MMA issuer (one lane);
//   warps 2-9     Rank-Rotary rotation of the relation boxes in place (the
//                 moment pass uses warps 2-13, adding the BF16 hi/lo split
//                 into the MN-major operand buffer);
//   warps 10-17   epilogue (moment pass: warps 14-17): TMEM -> registers, combine with the staged
//                 content / dY boxes and write the result back into the boxes,
//                 or drain moment accumulators to the partials;
//   warp 18       (readout and gradient passes) storer: TMA tensor stores of
//                 the finished boxes (tokens past N are clipped), slot release.
//
// Kernels (same algebra as the per-head kernels of mixer.cu; reference
// lsso/ball/reference.py:411-572,691-724, lsso/ball/model.py:245-268):
//   moments_tile_kernel<R, false>  G/S partials  [hi|lo]^T [hi | C] per chunk of tiles
//   moments_tile_kernel<R, true>   A'^T dY partials [hi|lo]^T dY
//   readout_tile_kernel<R>         Y = eta C + A' R_d
//   grad_tile_kernel<R>            dA' = dY B1y + C B1c + A' B1a (rotated back), dC = eta dY + A' B2
//                                  (B2 = B1c^T, read from the B1c matrix as an MN-major operand),
//                                  and the per-tile complement statistic sum(dY * C)
//
// Every wait is bounded (the status word records a timeout and all roles
// stop); before exit the producer waits, bounded, for its last loads.
#include <algorithm>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "linear.h"
#include "mixer.h"
#include "mixer_common.cuh"

namespace lsso {

namespace {

constexpr int kTT = kTileTokens;             // tokens per tile
constexpr uint32_t kBox = kTileBox;          // 128 tokens x 64 BF16 features: 16 KB
constexpr int kMaxSlots = kTileMaxSlots;
constexpr int kXWarp0 = 2, kXWarps = 8;      // rotation / split warps
constexpr int kEWarp0 = 10, kEWarps = 8;      // epilogue warps (two per TMEM sub-partition)
constexpr int kXThreads = kXWarps * 32;
// Readout and gradient passes add one storer warp: it waits for a tile's
// epilogue, issues the TMA stores and frees the slot once they have read it,
// so no epilogue warp blocks on store completion.
constexpr int kSWarp = kEWarp0 + kEWarps;
constexpr int kThreadsS = (kSWarp + 1) * 32;
// The moment pass drains TMEM only at the end of a chunk, so it gives most of
// its warps to the rotation / hi-lo split: 12 of them, and 4 drain warps (one
// per TMEM sub-partition).
constexpr int kMXWarps = 12, kMEWarp0 = kXWarp0 + kMXWarps, kMEWarps = 4;
constexpr int kMXThreads = kMXWarps * 32;
constexpr int kMThreads = (kMEWarp0 + kMEWarps) * 32;
constexpr size_t kSmemFloor = 120 * 1024;    // forces one CTA per SM (each allocates all of TMEM)

struct TileArgs {
  const __half2* phase16;   // FP16 (cos, sin) table [pos_rows][N][R/2], staged per slot by the producer
  const float* eta_raw;
  const bf16* m0;  // readout: R_d;  grad: B1y
  const bf16* m1;  // grad: B1c
  const bf16* m2;  // grad: B1a
  float* partial;  // moment partials [B*H][nchunks][2R][NC]
  bf16* gproj;     // gradient pass: packed gradient [B][N][W], for relation features outside whole boxes
  float* etastat;  // [B*H][ntiles]
  int* status;
  int N, H, d, hg, groups, nrel, nval, ntiles, ct, nchunks, items, pos_batched, slots, nbuf, cols;
  int rel_tma;          // gradient pass: relation boxes wholly inside the group (stored by TMA)
  int rev;              // walk the items in reverse order (ItemWalk)
  int loring;           // moment pass: boxes in the lo ring (1 or 2)
  int wdg, wdm, wdb;    // the grid stride as (group, tile or chunk, sample) steps of the item walk
  int W;                // packed width
  uint32_t slot_bytes;  // bytes per slot (multiple of 1024)
  uint32_t off_val;     // content (or dY) boxes
  uint32_t off_aux;     // grad: dY boxes
  uint32_t off_rel;     // moments: relation boxes
  uint32_t off_slots;   // moments: first slot (the lo ring, two boxes, sits below it)
  uint32_t off_mat;     // operand matrices
  uint32_t off_ph;      // the tile's FP16 phase rows
  uint32_t load_bytes;  // transaction bytes per slot fill, phase rows excluded
};

struct TileShared {
  uint64_t full[kMaxSlots];   // producer -> transform (TMA / bulk bytes landed)
  uint64_t xdone[kMaxSlots];  // transform -> MMA
  uint64_t sfree[kMaxSlots];  // slot released (MMA done, or output stored)
  uint64_t edone[kMaxSlots];  // epilogue warps -> storing thread
  uint64_t tfull[4];          // MMA -> epilogue (accumulator ready)
  uint64_t tempty[4];         // epilogue -> MMA (accumulator drained)
  uint64_t lofree[2];         // moment pass: lo box free (MMA done with it)
  uint64_t mdrain;            // teardown: the MMA thread's last commit (mma_drain)
  uint32_t tmem;
  int abort_flag;
  float red[kMaxSlots][4][4];  // per slot, head, sub-partition: complement statistic
};

__device__ __forceinline__ bool twait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  return mbar_wait_bounded(bar, parity, abort_flag, status);
}
// The same wait by a whole warp that goes on to warp-collective instructions
// (tcgen05.ld, shuffles): its lanes agree on the outcome, so after an abort
// none of them runs a collective the others skip.
__device__ __forceinline__ bool twait_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, status));
}

// 16-byte chunk c (features 8c .. 8c+7) of token row r in a 128B-swizzled box
// (1024-byte aligned): chunk c of row r lives at chunk c ^ (r % 8).
__device__ __forceinline__ uint8_t* box_chunk(uint8_t* box, int r, int c) {
  return box + r * 128 + ((c ^ (r & 7)) << 4);
}

// Common prologue: barriers, TMEM (all 512 columns), 1024-byte aligned base.
__device__ __forceinline__ uint8_t* tile_setup(TileShared& sh, uint8_t* raw, int slots, int nbuf, int tcount_mma,
                                               int tcount_free, int xwarps, int ewarps) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      mbar_init(smem_u32(&sh.full[s]), 1);
      mbar_init(smem_u32(&sh.xdone[s]), xwarps);
      mbar_init(smem_u32(&sh.sfree[s]), tcount_free);
      mbar_init(smem_u32(&sh.edone[s]), ewarps);
    }
    for (int b = 0; b < nbuf; ++b) {
      mbar_init(smem_u32(&sh.tfull[b]), tcount_mma);
      mbar_init(smem_u32(&sh.tempty[b]), ewarps);
    }
    for (int b = 0; b < 2; ++b) mbar_init(smem_u32(&sh.lofree[b]), 1);
    mbar_init(smem_u32(&sh.mdrain), 1);
    sh.abort_flag = 0;
    fence_mbar_init();
  }
  if ((threadIdx.x >> 5) == 1) tmem_alloc(smem_u32(&sh.tmem), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t base = smem_u32(raw);
  return raw + (((base + 1023u) & ~1023u) - base);
}

// Common epilogue: the MMA thread (warp 1, lane 0 in every tile kernel) waits
// for its tensor-core operations and the producer (thread 0) for its last
// loads, both bounded; then TMEM is freed.  Each storing role has already
// waited for its bulk stores.  After an abort this is what keeps the CTA from
// freeing TMEM or exiting under operations still in flight.
__device__ __forceinline__ void tile_teardown(TileShared& sh, int slots, const int* last_use, int* status) {
  if (threadIdx.x == 32) mma_drain(smem_u32(&sh.mdrain), status);
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < slots; ++s) {
      if (last_use[s] >= 0) mbar_wait(smem_u32(&sh.full[s]), static_cast<uint32_t>(last_use[s]) & 1u, status);
    }
  }
  if ((threadIdx.x >> 5) == 1) {
    tc_fence_after();
    tmem_dealloc(sh.tmem, 512);
  }
}

// Item decode for the per-tile kernels: head group fastest, then tile, then
// sample, so the CTAs in flight together cover whole projection rows (every
// group's slice of the same tokens) instead of one 128-byte slice per row.
struct TileItem {
  int b, g, t;
};
__device__ __forceinline__ TileItem decode_tile(int it, int ntiles, int groups) {
  TileItem x;
  x.g = it % groups;
  const int rest = it / groups;
  x.t = rest % ntiles;
  x.b = rest / ntiles;
  return x;
}

// The items of one persistent CTA, it = blockIdx.x + i * gridDim.x, as
// (g fastest, then m, then b), advanced by one CTA stride without division
// (the stride's own decomposition comes precomputed in the arguments): the
// integer divisions run once per role, not once per tile.
struct ItemWalk {
  int g, m, b;
  bool rev;
  // rev: the items in reverse (it -> items - 1 - it), so that a pass can start
  // with the rows its producer wrote last, which are still in L2.
  __device__ __forceinline__ void start(int groups, int mids, int reverse = 0, int items = 0) {
    rev = reverse != 0;
    const int it = rev ? items - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
    const TileItem x = decode_tile(it, mids, groups);
    g = x.g;
    m = x.t;
    b = x.b;
  }
  // (dg, dm, db): gridDim.x decomposed the same way.
  __device__ __forceinline__ void next(int groups, int mids, int dg, int dm, int db) {
    if (!rev) {
      g += dg;
      int c = g >= groups ? 1 : 0;
      g -= c * groups;
      m += dm + c;
      c = m >= mids ? 1 : 0;
      m -= c * mids;
      b += db + c;
    } else {
      g -= dg;
      int c = g < 0 ? 1 : 0;
      g += c * groups;
      m -= dm + c;
      c = m < 0 ? 1 : 0;
      m += c * mids;
      b -= db + c;
    }
  }
  __device__ __forceinline__ TileItem item() const { return TileItem{b, g, m}; }
};


// 4 (cos, sin) pairs of rank chunk q of tile row r from FP16 phase rows staged
// in shared memory (R/2 half2 per row); tokens past N rotate by the identity.
__device__ __forceinline__ Phase4 phase_rows16(const uint8_t* rows, int r, int tok, int N, int R, int q) {
  if (tok >= N) return phase_identity();
  const uint4 h = *reinterpret_cast<const uint4*>(rows + r * (R * 2) + q * 16);
  const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
  const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
  const float2 p2 = __half22float2(*reinterpret_cast<const __half2*>(&h.z));
  const float2 p3 = __half22float2(*reinterpret_cast<const __half2*>(&h.w));
  return Phase4{make_float4(p0.x, p0.y, p1.x, p1.y), make_float4(p2.x, p2.y, p3.x, p3.y)};
}

// Bytes of the FP16 phase rows of tile rows [t0, t0 + 128) inside the sequence.
__device__ __forceinline__ uint32_t phase16_bytes(int t0, int N, int R) {
  const int rows = min(kTT, N - t0);
  return static_cast<uint32_t>(rows * R * 2);
}

// Relation chunks (8 features x 1 token) per transform thread and tile: the
// thread owns chunks xt + k * kXThreads, k < nrel * 1024 / kXThreads (nrel <= 2).
constexpr int kMaxChunks = 2 * kTT * 8 / kXThreads;

__device__ __forceinline__ void chunk_coords(int idx, int& j, int& r, int& c) {
  j = idx / (kTT * 8);
  const int rem = idx % (kTT * 8);
  r = rem >> 3;
  c = rem & 7;
}

// Rotate the relation boxes in place with phases from staged FP16 rows.
template <int R>
__device__ __forceinline__ void rotate_boxes16(uint8_t* rel, int nrel, const uint8_t* rows, int tok0, int N, int xt) {
  const int nch = nrel * (kTT * 8) / kXThreads;
  // In batches of four chunks, each read before any of it is written back.
#pragma unroll
  for (int k0 = 0; k0 < kMaxChunks; k0 += 4) {
    uint4 in[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k0 + k < nch) {
        int j, r, c;
        chunk_coords(xt + (k0 + k) * kXThreads, j, r, c);
        in[k] = *reinterpret_cast<const uint4*>(box_chunk(rel + j * kBox, r, c));
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k0 + k < nch) {
        int j, r, c;
        chunk_coords(xt + (k0 + k) * kXThreads, j, r, c);
        const Phase4 ph = phase_rows16(rows, r, tok0 + r, N, R, ((j * 64 + 8 * c) % R) >> 3);
        float v[8];
        rotate8(in[k], ph, v);
        *reinterpret_cast<uint4*>(box_chunk(rel + j * kBox, r, c)) = pack8_bf16(v);
      }
    }
  }
}

// Drain one moment-pass item's accumulator into its heads' partials
// partial[(b*H + h)][chunk][2R][NC] (NC = R + d forward, d backward).  `taddr`
// is the accumulator's first column at this warp's TMEM sub-partition (lanes
// 32 sub ..).  TMEM lane = (lo ? 0 : 64) + f for feature f of the relation
// box: feature f = 32 (sub & 1) + lane is rank f % R of the item's head f / R
// (at R = 48 the box's last 16 features belong to the next head: computed, not
// stored).  Columns: forward [hi Gram block of the box | value box], backward
// [dY box].  A TMEM load takes one column address per warp, so a warp whose
// 32 lanes span two heads (R = 16) loads once per head.
template <int R, bool BWD>
__device__ __forceinline__ void drain_moments(uint32_t taddr, int sub, int lane, float* partial, int b, int g,
                                              int chunk, int H, int hg, int d, int nchunks) {
  constexpr int M2 = 2 * R;  // rows of one head's partial
  const int NC = (BWD ? 0 : R) + d;
  const int f0 = 32 * (sub & 1);
  const int f = f0 + lane;
  const int hl = f / R;
  const bool mine = hl < hg;
  const int row = (sub < 2 ? R : 0) + f % R;
  const int voff = (g * hg * d) & 63;  // the item's first head inside the value box
  const int64_t bh = static_cast<int64_t>(b) * H + g * hg + (mine ? hl : 0);
  float* out = partial + ((bh * nchunks + chunk) * M2 + row) * static_cast<int64_t>(NC);
  const int hw_last = min(hg - 1, (f0 + 31) / R);
  for (int hw = f0 / R; hw <= hw_last; ++hw) {
    // Gram columns (forward only), in pieces of at most 32, then the value columns
    for (int c0 = 0; c0 < NC; c0 += 32) {
      const bool gram = !BWD && c0 < R;
      const int n = gram ? min(32, R - c0) : 32;
      const int tc = BWD ? voff + hw * d + c0 : (gram ? hw * R + c0 : 64 + voff + hw * d + (c0 - R));
      float v[32];
      tmem_ld32(taddr + static_cast<uint32_t>(tc), v);
      tmem_ld_wait();
      if (mine && hl == hw) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (j < n) *reinterpret_cast<float4*>(out + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
      if (gram && n < 32) c0 -= 32 - n;  // the value columns start right after the Gram columns
    }
  }
}

// ============================================================================
// Moment pass.  Item = (sample, head group, chunk of ct tiles), K = 128 tokens
// per tile, accumulated in TMEM over the chunk; at its end the epilogue drains
// partial[(b*H + h)][chunk][2R][NC] (rows [0, R) hi products, [R, 2R) lo).
//
// The item's relation features fill one 64-feature box (two heads at R = 32,
// one head at R = 64): slot = [relation box, rotated to hi in place | value
// box]; the lo box comes from a ring of two below the slots, so a slot holds
// only loaded data and more loads fit in flight.  Per K-step ONE MMA covers
// the box: A = [lo | hi] (M = 128: the 64 lo rows, then the 64 hi rows; LBO
// = the distance from the lo box to the slot), B = [hi | values] (forward:
// N = 128) or B = dY (backward: N = 64), consecutive boxes (LBO = 16 KB).
// The value / dY box is the 64-feature box
// holding the item's heads (at R = 64, d = 32 it also holds the neighbouring
// head, whose columns are computed and ignored, as are the cross-head blocks
// at R = 32).
// ============================================================================
template <int R, bool BWD>
__global__ void __launch_bounds__(kMThreads, 1) moments_tile_kernel(const __grid_constant__ CUtensorMap tm_rel,
                                                                     const __grid_constant__ CUtensorMap tm_val,
                                                                     const TileArgs a) {
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  __shared__ TileShared sh;
  volatile int* abort_v = &sh.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.d;
  uint8_t* smem = tile_setup(sh, smem_raw, a.slots, a.nbuf, 1, 1, kMXWarps, kMEWarps);
  const int nloc = (a.items - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                   static_cast<int>(gridDim.x);
  int last_use[kMaxSlots] = {-1, -1, -1, -1, -1, -1};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tm_rel);
      prefetch_tmap(&tm_val);
    }
    ItemWalk w;
    w.start(a.groups, a.nchunks, a.rev, a.items);
    RingPos sp;
    bool ok = true;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.nchunks, a.wdg, a.wdm, a.wdb)) {
      const int b = w.b, g = w.g, t0 = w.m * a.ct, nt = min(a.ct, a.ntiles - t0);
      for (int tt = 0; tt < nt && ok; ++tt, sp.next(a.slots)) {
        const int s = sp.s, u = sp.u;
        ok = twait(smem_u32(&sh.sfree[s]), (u & 1) ^ 1, abort_v, a.status);
        if (ok && lane == 0) {
          uint8_t* slot = smem + a.off_slots + static_cast<size_t>(s) * a.slot_bytes;
          const uint32_t bar = smem_u32(&sh.full[s]);
          const int row = (t0 + tt) * kTT;
          const uint32_t pb = phase16_bytes(row, a.N, R);
          mbar_arrive_expect_tx(bar, a.load_bytes + pb);
          const int64_t prow = a.pos_batched ? static_cast<int64_t>(b) * a.N : 0;
          bulk_load(smem_u32(slot + a.off_ph), a.phase16 + (prow + row) * (R / 2), pb, bar);
          for (int j = 0; j < a.nrel; ++j)
            tma_load_3d(smem_u32(slot + a.off_rel + j * kBox), &tm_rel, g * a.hg * R + j * 64, row, b, bar);
          // the 64-feature boxes holding the item's heads (their first feature rounded down)
          const int vcol0 = (BWD ? 0 : a.H * R) + ((g * a.hg * d) & ~63);
          for (int j = 0; j < a.nval; ++j)
            tma_load_3d(smem_u32(slot + a.off_val + j * kBox), &tm_val, vcol0 + j * 64, row, b, bar);
          last_use[s] = u;
        }
        __syncwarp();
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc_f = make_idesc(128, BWD ? 64 * a.nval : 64 + 64 * a.nval, true, true);
    ItemWalk w;
    w.start(a.groups, a.nchunks, a.rev, a.items);
    RingPos sp, bp, lp;
    bool ok = true;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.nchunks, a.wdg, a.wdm, a.wdb), bp.next(a.nbuf)) {
      const int t0 = w.m * a.ct, nt = min(a.ct, a.ntiles - t0);
      const int tb = bp.s, tu = bp.u;
      ok = twait(smem_u32(&sh.tempty[tb]), (tu & 1) ^ 1, abort_v, a.status);
      tc_fence_after();
      for (int tt = 0; tt < nt && ok; ++tt, sp.next(a.slots), lp.next(a.loring)) {
        const int s = sp.s, u = sp.u;
        ok = twait(smem_u32(&sh.xdone[s]), u & 1, abort_v, a.status);
        tc_fence_after();
        if (ok && lane == 0) {
          const uint32_t slot = smem_u32(smem + a.off_slots + static_cast<size_t>(s) * a.slot_bytes);
          const uint32_t lo = smem_u32(smem) + static_cast<uint32_t>(lp.s) * kBox;
          const uint32_t dcol = sh.tmem + static_cast<uint32_t>(tb * a.cols);
          const uint32_t bsrc = slot + (BWD ? a.off_val : a.off_rel);
          // A = [lo | hi]: the lo box of the ring, then the slot's (rotated) relation box
          const uint32_t lbo = slot + a.off_rel - lo;
#pragma unroll
          for (int ks = 0; ks < kTT / 16; ++ks) {
            mma_bf16(dcol, make_desc_sw128(lo + ks * 2048, lbo, 1024),
                     make_desc_sw128(bsrc + ks * 2048, kBox, 1024), idesc_f, (tt > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(smem_u32(&sh.sfree[s]));
          mma_commit(smem_u32(&sh.lofree[lp.s]));
          if (tt == nt - 1) mma_commit(smem_u32(&sh.tfull[tb]));
        }
        __syncwarp();
      }
    }
  } else if (warp < kXWarp0 + kMXWarps) {
    // ------------------------------------------------------------ rotate + hi/lo split
    // The phases arrive with the boxes: the producer stages the tile's FP16
    // phase rows in the slot, so the rotation waits on no global load.
    constexpr int NCH = (kTT * 8 + kMXThreads - 1) / kMXThreads;  // chunks per thread (one relation box)
    const int xt = threadIdx.x - kXWarp0 * 32;
    const int total = a.nrel * kTT * 8;
    ItemWalk w;
    w.start(a.groups, a.nchunks, a.rev, a.items);
    RingPos sp, lp;
    bool ok = true;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.nchunks, a.wdg, a.wdm, a.wdb)) {
      const int t0 = w.m * a.ct, nt = min(a.ct, a.ntiles - t0);
      for (int tt = 0; tt < nt && ok; ++tt, sp.next(a.slots), lp.next(a.loring)) {
        const int s = sp.s, u = sp.u;
        ok = twait(smem_u32(&sh.full[s]), u & 1, abort_v, a.status);
        if (ok) ok = twait(smem_u32(&sh.lofree[lp.s]), (lp.u & 1) ^ 1, abort_v, a.status);
        if (ok) {
          uint8_t* slot = smem + a.off_slots + static_cast<size_t>(s) * a.slot_bytes;
          uint8_t* rel = slot + a.off_rel;
          const uint8_t* rows = slot + a.off_ph;
          uint8_t* op = smem + static_cast<size_t>(lp.s) * kBox;  // this tile's lo box
          const int tok0 = (t0 + tt) * kTT;
          // In batches of three chunks, each read before any of it is written,
          // so the shared-memory loads overlap instead of waiting behind stores.
#pragma unroll
          for (int b0 = 0; b0 < NCH; b0 += 3) {
            uint4 in[3];
#pragma unroll
            for (int q = 0; q < 3; ++q) {
              const int idx = xt + (b0 + q) * kMXThreads;
              if (b0 + q < NCH && idx < total) {
                int j, r, c;
                chunk_coords(idx, j, r, c);
                in[q] = *reinterpret_cast<const uint4*>(box_chunk(rel + j * kBox, r, c));
              }
            }
#pragma unroll
            for (int q = 0; q < 3; ++q) {
              const int kk = b0 + q;
              const int idx = xt + kk * kMXThreads;
              if (kk >= NCH || idx >= total) break;
              int j, r, c;
              chunk_coords(idx, j, r, c);
              uint8_t* src = box_chunk(rel + j * kBox, r, c);
              float v[8];
              rotate8(in[q], phase_rows16(rows, r, tok0 + r, a.N, R, ((j * 64 + 8 * c) % R) >> 3), v);
              const uint4 hi = pack8_bf16(v);
              const float2 h0 = unpack_bf16(hi.x), h1 = unpack_bf16(hi.y), h2 = unpack_bf16(hi.z), h3 = unpack_bf16(hi.w);
              float lo[8] = {v[0] - h0.x, v[1] - h0.y, v[2] - h1.x, v[3] - h1.y,
                             v[4] - h2.x, v[5] - h2.y, v[6] - h3.x, v[7] - h3.y};
              *reinterpret_cast<uint4*>(src) = hi;                                        // hi in place
              *reinterpret_cast<uint4*>(box_chunk(op + j * kBox, r, c)) = pack8_bf16(lo);  // lo, same position
            }
          }
          fence_proxy_async();
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(smem_u32(&sh.xdone[s]));
      }
    }
  } else {
    // ------------------------------------------------------------ drain accumulators (one warp per sub-partition)
    const int sub = warp & 3;
    const uint32_t lane_base = sh.tmem + (static_cast<uint32_t>(32 * sub) << 16);
    ItemWalk w;
    w.start(a.groups, a.nchunks, a.rev, a.items);
    RingPos bp;
    bool ok = true;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.nchunks, a.wdg, a.wdm, a.wdb), bp.next(a.nbuf)) {
      const int tb = bp.s, tu = bp.u;
      ok = twait_warp(smem_u32(&sh.tfull[tb]), tu & 1, abort_v, a.status);
      tc_fence_after();
      if (ok) {
        drain_moments<R, BWD>(lane_base + static_cast<uint32_t>(tb * a.cols), sub, lane, a.partial, w.b, w.g, w.m,
                              a.H, a.hg, d, a.nchunks);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sh.tempty[tb]));
    }
  }
  tile_teardown(sh, a.slots, last_use, a.status);
}

// ============================================================================
// Readout: Y = eta C + A' R_d per (sample, head group, tile).  MMA per head:
// M = 128 tokens, K = R (rotated relation, K-major straight from its box),
// N = d (R_d, K-major canonical from the solve).  The epilogue writes
// eta C + acc over the content box and stores it to the mixed output.
// ============================================================================
template <int R>
__global__ void __launch_bounds__(kThreadsS, 1) readout_tile_kernel(const __grid_constant__ CUtensorMap tm_proj,
                                                                     const __grid_constant__ CUtensorMap tm_out,
                                                                     const TileArgs a) {
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  __shared__ TileShared sh;
  volatile int* abort_v = &sh.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.d;
  uint8_t* smem = tile_setup(sh, smem_raw, a.slots, a.nbuf, 1, 1, kXWarps, kEWarps);
  const int nloc = (a.items - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                   static_cast<int>(gridDim.x);
  int last_use[kMaxSlots] = {-1, -1, -1, -1, -1, -1};
  const uint32_t mat_bytes = static_cast<uint32_t>(a.hg * d * R * 2);

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_proj);
      prefetch_tmap(&tm_out);
    }
    bool ok = true;
    ItemWalk w;
    w.start(a.groups, a.ntiles, a.rev, a.items);
    RingPos sp;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots)) {
      const TileItem x = w.item();
      const int s = sp.s, u = sp.u;
      ok = twait(smem_u32(&sh.sfree[s]), (u & 1) ^ 1, abort_v, a.status);
      if (ok && lane == 0) {
        uint8_t* slot = smem + static_cast<size_t>(s) * a.slot_bytes;
        const uint32_t bar = smem_u32(&sh.full[s]);
        const int row = x.t * kTT;
        const uint32_t pb = phase16_bytes(row, a.N, R);
        mbar_arrive_expect_tx(bar, a.load_bytes + pb);
        const int64_t prow = a.pos_batched ? static_cast<int64_t>(x.b) * a.N : 0;
        bulk_load(smem_u32(slot + a.off_ph), a.phase16 + (prow + row) * (R / 2), pb, bar);
        for (int j = 0; j < a.nrel; ++j)
          tma_load_3d(smem_u32(slot + j * kBox), &tm_proj, x.g * a.hg * R + j * 64, row, x.b, bar);
        for (int j = 0; j < a.nval; ++j)
          tma_load_3d(smem_u32(slot + a.off_val + j * kBox), &tm_proj, a.H * R + x.g * a.hg * d + j * 64, row, x.b,
                      bar);
        const int64_t bh0 = static_cast<int64_t>(x.b) * a.H + x.g * a.hg;
        bulk_load(smem_u32(slot + a.off_mat), a.m0 + bh0 * d * R, mat_bytes, bar);
        last_use[s] = u;
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    const uint32_t idesc = make_idesc(128, d, false, false);
    bool ok = true;
    RingPos sp, bp;
    for (int i = 0; i < nloc && ok; ++i, sp.next(a.slots), bp.next(a.nbuf)) {
      const int s = sp.s, u = sp.u;
      const int tb = bp.s, tu = bp.u;
      ok = twait(smem_u32(&sh.xdone[s]), u & 1, abort_v, a.status);
      if (ok) ok = twait(smem_u32(&sh.tempty[tb]), (tu & 1) ^ 1, abort_v, a.status);
      tc_fence_after();
      if (ok && lane == 0) {
        const uint32_t slot = smem_u32(smem + static_cast<size_t>(s) * a.slot_bytes);
        for (int hl = 0; hl < a.hg; ++hl) {
          const uint32_t dcol = sh.tmem + static_cast<uint32_t>(tb * a.cols + hl * d);
#pragma unroll
          for (int ks = 0; ks < R / 16; ++ks) {
            const int f = hl * R + 16 * ks;
            const uint64_t ad = make_desc_sw128(slot + (f >> 6) * kBox + (f & 63) * 2, 16, 1024);
            const uint64_t bd = make_desc(slot + a.off_mat + hl * d * R * 2 + ks * 256, 128, R * 16);
            mma_bf16(dcol, ad, bd, idesc, ks > 0 ? 1u : 0u);
          }
        }
        mma_commit(smem_u32(&sh.tfull[tb]));
      }
      __syncwarp();
    }
  } else if (warp < kXWarp0 + kXWarps) {
    const int xt = threadIdx.x - kXWarp0 * 32;
    bool ok = true;
    ItemWalk w;
    w.start(a.groups, a.ntiles, a.rev, a.items);
    RingPos sp;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots)) {
      const TileItem x = w.item();
      const int s = sp.s, u = sp.u;
      ok = twait(smem_u32(&sh.full[s]), u & 1, abort_v, a.status);
      if (ok) {
        uint8_t* slot = smem + static_cast<size_t>(s) * a.slot_bytes;
        rotate_boxes16<R>(slot, a.nrel, slot + a.off_ph, x.t * kTT, a.N, xt);
        fence_proxy_async();
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(smem_u32(&sh.xdone[s]));
    }
  } else if (warp < kSWarp) {
    const int sub = warp & 3, half = (warp - kEWarp0) >> 2;
    const int r = 32 * sub + lane;
    const uint32_t lane_base = sh.tmem + (static_cast<uint32_t>(32 * sub) << 16);
    bool ok = true;
    ItemWalk w;
    w.start(a.groups, a.ntiles, a.rev, a.items);
    RingPos sp, bp;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots), bp.next(a.nbuf)) {
      const TileItem x = w.item();
      const int s = sp.s;
      const int tb = bp.s, tu = bp.u;
      ok = twait_warp(smem_u32(&sh.tfull[tb]), tu & 1, abort_v, a.status);
      tc_fence_after();
      uint8_t* con = smem + static_cast<size_t>(s) * a.slot_bytes + a.off_val;
      if (ok) {
        for (int hl = half; hl < a.hg; hl += 2) {
          const float eta = bounded_complement(a.eta_raw[x.g * a.hg + hl]);
          for (int c0 = 0; c0 < d; c0 += 32) {
            float v[32];
            tmem_ld32(lane_base + static_cast<uint32_t>(tb * a.cols + hl * d + c0), v);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int f = hl * d + c0 + 8 * q;
              uint4* p = reinterpret_cast<uint4*>(box_chunk(con + (f >> 6) * kBox, r, (f & 63) >> 3));
              const uint4 cv = *p;
              const float2 c01 = unpack_bf16(cv.x), c23 = unpack_bf16(cv.y), c45 = unpack_bf16(cv.z),
                           c67 = unpack_bf16(cv.w);
              float y[8] = {fmaf(eta, c01.x, v[8 * q]),     fmaf(eta, c01.y, v[8 * q + 1]),
                            fmaf(eta, c23.x, v[8 * q + 2]), fmaf(eta, c23.y, v[8 * q + 3]),
                            fmaf(eta, c45.x, v[8 * q + 4]), fmaf(eta, c45.y, v[8 * q + 5]),
                            fmaf(eta, c67.x, v[8 * q + 6]), fmaf(eta, c67.y, v[8 * q + 7])};
              *p = pack8_bf16(y);
            }
          }
        }
      }
      tc_fence_before();
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&sh.tempty[tb]));
        if (ok) mbar_arrive(smem_u32(&sh.edone[s]));
      }
    }
  } else {
    // ------------------------------------------------------------ storer
    if (lane == 0) {
      bool ok = true;
      ItemWalk w;
      w.start(a.groups, a.ntiles, a.rev, a.items);
      RingPos sp;
      for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots)) {
        const TileItem x = w.item();
        const int s = sp.s, u = sp.u;
        ok = twait(smem_u32(&sh.edone[s]), u & 1, abort_v, a.status);
        if (ok) {
          uint8_t* con = smem + static_cast<size_t>(s) * a.slot_bytes + a.off_val;
          for (int j = 0; j < a.nval; ++j)
            tma_store_3d(&tm_out, smem_u32(con + j * kBox), x.g * a.hg * d + j * 64, x.t * kTT, x.b);
          bulk_commit();
          bulk_wait_read<0>();
          mbar_arrive(smem_u32(&sh.sfree[s]));
        }
      }
      bulk_wait<0>();
    }
    __syncwarp();
  }
  tile_teardown(sh, a.slots, last_use, a.status);
}

// ============================================================================
// Gradient pass per (sample, head group, tile).  MMA per head (M = 128
// tokens, A operands K-major straight from the boxes):
//   dA' = dY B1y + C B1c + A' B1a   (N = R)     dC = A' B2   (N = d)
// Epilogue: dA' rotated back with the transposed Rank-Rotary map into the
// relation box, eta dY + dC into the content box (after the complement
// statistic sum(dY * C) is taken), both stored to the packed gradient.
// ============================================================================
template <int R>
__global__ void __launch_bounds__(kThreadsS, 1) grad_tile_kernel(const __grid_constant__ CUtensorMap tm_proj,
                                                                  const __grid_constant__ CUtensorMap tm_dy,
                                                                  const __grid_constant__ CUtensorMap tm_gproj,
                                                                  const TileArgs a) {
  pdl_wait();
  extern __shared__ uint8_t smem_raw[];
  __shared__ TileShared sh;
  volatile int* abort_v = &sh.abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int d = a.d;
  const int NC = R + d;
  uint8_t* smem = tile_setup(sh, smem_raw, a.slots, a.nbuf, 1, 1, kXWarps, kEWarps);
  const int nloc = (a.items - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                   static_cast<int>(gridDim.x);
  int last_use[kMaxSlots] = {-1, -1, -1, -1, -1, -1};
  // Operand matrices of the group's heads, each block contiguous per head.  B2
  // (d x R, K-major) is B1c (R x d, K-major canonical) read as an MN-major
  // operand: element (n, k) of B2 is element (k, n) of B1c, whose 8 x 8 core
  // matrices are n-adjacent at 128 bytes and k-adjacent at d * 16 bytes.
  const uint32_t sz_y = static_cast<uint32_t>(R * d * 2), sz_a = static_cast<uint32_t>(R * R * 2);
  const uint32_t off_y = 0, off_c = a.hg * sz_y, off_a = 2 * a.hg * sz_y;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tm_proj);
      prefetch_tmap(&tm_dy);
      prefetch_tmap(&tm_gproj);
    }
    bool ok = true;
    ItemWalk w;
    w.start(a.groups, a.ntiles, a.rev, a.items);
    RingPos sp;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots)) {
      const TileItem x = w.item();
      const int s = sp.s, u = sp.u;
      ok = twait(smem_u32(&sh.sfree[s]), (u & 1) ^ 1, abort_v, a.status);
      if (ok && lane == 0) {
        uint8_t* slot = smem + static_cast<size_t>(s) * a.slot_bytes;
        const uint32_t bar = smem_u32(&sh.full[s]);
        const int row = x.t * kTT;
        const uint32_t pb = phase16_bytes(row, a.N, R);
        mbar_arrive_expect_tx(bar, a.load_bytes + pb);
        const int64_t prow = a.pos_batched ? static_cast<int64_t>(x.b) * a.N : 0;
        bulk_load(smem_u32(slot + a.off_ph), a.phase16 + (prow + row) * (R / 2), pb, bar);
        for (int j = 0; j < a.nrel; ++j)
          tma_load_3d(smem_u32(slot + j * kBox), &tm_proj, x.g * a.hg * R + j * 64, row, x.b, bar);
        for (int j = 0; j < a.nval; ++j) {
          tma_load_3d(smem_u32(slot + a.off_val + j * kBox), &tm_proj, a.H * R + x.g * a.hg * d + j * 64, row, x.b,
                      bar);
          tma_load_3d(smem_u32(slot + a.off_aux + j * kBox), &tm_dy, x.g * a.hg * d + j * 64, row, x.b, bar);
        }
        const int64_t bh0 = static_cast<int64_t>(x.b) * a.H + x.g * a.hg;
        uint8_t* mat = slot + a.off_mat;
        bulk_load(smem_u32(mat + off_y), a.m0 + bh0 * R * d, a.hg * sz_y, bar);
        bulk_load(smem_u32(mat + off_c), a.m1 + bh0 * R * d, a.hg * sz_y, bar);
        bulk_load(smem_u32(mat + off_a), a.m2 + bh0 * R * R, a.hg * sz_a, bar);
        last_use[s] = u;
      }
      __syncwarp();
    }
  } else if (warp == 1) {
    const uint32_t idesc_r = make_idesc(128, R, false, false);
    const uint32_t idesc_d = make_idesc(128, d, false, true);
    bool ok = true;
    RingPos sp, bp;
    for (int i = 0; i < nloc && ok; ++i, sp.next(a.slots), bp.next(a.nbuf)) {
      const int s = sp.s, u = sp.u;
      const int tb = bp.s, tu = bp.u;
      ok = twait(smem_u32(&sh.xdone[s]), u & 1, abort_v, a.status);
      if (ok) ok = twait(smem_u32(&sh.tempty[tb]), (tu & 1) ^ 1, abort_v, a.status);
      tc_fence_after();
      if (ok && lane == 0) {
        const uint32_t slot = smem_u32(smem + static_cast<size_t>(s) * a.slot_bytes);
        const uint32_t mat = slot + a.off_mat;
        for (int hl = 0; hl < a.hg; ++hl) {
          const uint32_t da = sh.tmem + static_cast<uint32_t>(tb * a.cols + hl * NC);
          for (int ks = 0; ks < d / 16; ++ks) {
            const int f = hl * d + 16 * ks;
            const uint32_t fo = (f >> 6) * kBox + (f & 63) * 2;
            mma_bf16(da, make_desc_sw128(slot + a.off_aux + fo, 16, 1024),
                     make_desc(mat + off_y + hl * sz_y + ks * 256, 128, d * 16), idesc_r, ks > 0 ? 1u : 0u);
            mma_bf16(da, make_desc_sw128(slot + a.off_val + fo, 16, 1024),
                     make_desc(mat + off_c + hl * sz_y + ks * 256, 128, d * 16), idesc_r, 1u);
          }
#pragma unroll
          for (int ks = 0; ks < R / 16; ++ks) {
            const int f = hl * R + 16 * ks;
            const uint64_t ad = make_desc_sw128(slot + (f >> 6) * kBox + (f & 63) * 2, 16, 1024);
            mma_bf16(da, ad, make_desc(mat + off_a + hl * sz_a + ks * 256, 128, R * 16), idesc_r, 1u);
            mma_bf16(da + R, ad, make_desc(mat + off_c + hl * sz_y + ks * 32 * d, d * 16, 128), idesc_d,
                     ks > 0 ? 1u : 0u);
          }
        }
        mma_commit(smem_u32(&sh.tfull[tb]));
      }
      __syncwarp();
    }
  } else if (warp < kXWarp0 + kXWarps) {
    const int xt = threadIdx.x - kXWarp0 * 32;
    bool ok = true;
    ItemWalk w;
    w.start(a.groups, a.ntiles, a.rev, a.items);
    RingPos sp;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots)) {
      const TileItem x = w.item();
      const int s = sp.s, u = sp.u;
      ok = twait(smem_u32(&sh.full[s]), u & 1, abort_v, a.status);
      if (ok) {
        uint8_t* slot = smem + static_cast<size_t>(s) * a.slot_bytes;
        rotate_boxes16<R>(slot, a.nrel, slot + a.off_ph, x.t * kTT, a.N, xt);
        fence_proxy_async();
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(smem_u32(&sh.xdone[s]));
    }
  } else if (warp < kSWarp) {
    const int sub = warp & 3, half = (warp - kEWarp0) >> 2;
    const int r = 32 * sub + lane;
    const uint32_t lane_base = sh.tmem + (static_cast<uint32_t>(32 * sub) << 16);
    bool ok = true;
    ItemWalk w;
    w.start(a.groups, a.ntiles, a.rev, a.items);
    RingPos sp, bp;
    for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots), bp.next(a.nbuf)) {
      const TileItem x = w.item();
      const int s = sp.s;
      const int tb = bp.s, tu = bp.u;
      const int tok = x.t * kTT + r;
      // eta of this warp's first head, computed while the accumulator is still being produced
      const float eta_first = half < a.hg ? bounded_complement(a.eta_raw[x.g * a.hg + half]) : 0.0f;
      ok = twait_warp(smem_u32(&sh.tfull[tb]), tu & 1, abort_v, a.status);
      tc_fence_after();
      uint8_t* slot = smem + static_cast<size_t>(s) * a.slot_bytes;
      uint8_t* con = slot + a.off_val;
      uint8_t* dyb = slot + a.off_aux;
      const uint8_t* phs = slot + a.off_ph;
      if (ok) {
        for (int hl = half; hl < a.hg; hl += 2) {
          const uint32_t tcol = lane_base + static_cast<uint32_t>(tb * a.cols + hl * NC);
          // relation gradient: rotate dA' back and overwrite the relation box (features
          // in a box the group only partly owns, at R = 48, go straight to global memory)
          for (int r0 = 0; r0 < R; r0 += 32) {
            float gv[32];
            tmem_ld32(tcol + r0, gv);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if constexpr (R % 32 != 0) {
                if (r0 + 8 * q >= R) break;
              }
              const int f = hl * R + r0 + 8 * q;
              const Phase4 ph = phase_rows16(phs, r, tok, a.N, R, (r0 >> 3) + q);
              const float gi[8] = {gv[8 * q], gv[8 * q + 1], gv[8 * q + 2], gv[8 * q + 3],
                                   gv[8 * q + 4], gv[8 * q + 5], gv[8 * q + 6], gv[8 * q + 7]};
              float o[8];
              rotate8_transpose(gi, ph, o);
              const uint4 packed = pack8_bf16(o);
              if (R != 48 || (f >> 6) < a.rel_tma) {  // R = 16, 32, 64: every box wholly the group's
                *reinterpret_cast<uint4*>(box_chunk(slot + (f >> 6) * kBox, r, (f & 63) >> 3)) = packed;
              } else if (tok < a.N) {
                *reinterpret_cast<uint4*>(a.gproj + (static_cast<int64_t>(x.b) * a.N + tok) * a.W +
                                          x.g * a.hg * R + f) = packed;
              }
            }
          }
          // content gradient eta dY + dC, and the statistic sum(dY * C)
          const float eta = hl == half ? eta_first : bounded_complement(a.eta_raw[x.g * a.hg + hl]);
          float stat = 0.0f;
          for (int c0 = 0; c0 < d; c0 += 32) {
            float v[32];
            tmem_ld32(tcol + R + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int f = hl * d + c0 + 8 * q;
              const int bo = (f >> 6) * kBox;
              uint4* pc = reinterpret_cast<uint4*>(box_chunk(con + bo, r, (f & 63) >> 3));
              const uint4 yv = *reinterpret_cast<const uint4*>(box_chunk(dyb + bo, r, (f & 63) >> 3));
              const uint4 cv = *pc;
              const uint32_t yy[4] = {yv.x, yv.y, yv.z, yv.w}, cc[4] = {cv.x, cv.y, cv.z, cv.w};
              float o[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 y2 = unpack_bf16(yy[e]), c2 = unpack_bf16(cc[e]);
                stat = fmaf(y2.x, c2.x, stat);
                stat = fmaf(y2.y, c2.y, stat);
                o[2 * e] = fmaf(eta, y2.x, v[8 * q + 2 * e]);
                o[2 * e + 1] = fmaf(eta, y2.y, v[8 * q + 2 * e + 1]);
              }
              *pc = pack8_bf16(o);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) stat += __shfl_xor_sync(0xffffffffu, stat, o);
          if (lane == 0) sh.red[s][hl][sub] = stat;
        }
      }
      tc_fence_before();
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&sh.tempty[tb]));
        if (ok) mbar_arrive(smem_u32(&sh.edone[s]));
      }
    }
  } else {
    // ------------------------------------------------------------ storer
    if (lane == 0) {
      bool ok = true;
      ItemWalk w;
      w.start(a.groups, a.ntiles, a.rev, a.items);
      RingPos sp;
      for (int i = 0; i < nloc && ok; ++i, w.next(a.groups, a.ntiles, a.wdg, a.wdm, a.wdb), sp.next(a.slots)) {
        const TileItem x = w.item();
        const int s = sp.s, u = sp.u;
        ok = twait(smem_u32(&sh.edone[s]), u & 1, abort_v, a.status);
        if (ok) {
          uint8_t* slot = smem + static_cast<size_t>(s) * a.slot_bytes;
          uint8_t* con = slot + a.off_val;
          for (int j = 0; j < a.rel_tma; ++j)
            tma_store_3d(&tm_gproj, smem_u32(slot + j * kBox), x.g * a.hg * R + j * 64, x.t * kTT, x.b);
          for (int j = 0; j < a.nval; ++j)
            tma_store_3d(&tm_gproj, smem_u32(con + j * kBox), a.H * R + x.g * a.hg * d + j * 64, x.t * kTT, x.b);
          bulk_commit();
          for (int hl = 0; hl < a.hg; ++hl) {
            const int64_t bh = static_cast<int64_t>(x.b) * a.H + x.g * a.hg + hl;
            a.etastat[bh * a.ntiles + x.t] = (sh.red[s][hl][0] + sh.red[s][hl][1]) + (sh.red[s][hl][2] + sh.red[s][hl][3]);
          }
          bulk_wait_read<0>();
          mbar_arrive(smem_u32(&sh.sfree[s]));
        }
      }
      bulk_wait<0>();
    }
    __syncwarp();
  }
  tile_teardown(sh, a.slots, last_use, a.status);
}

// ---------------------------------------------------------------------------- host side
CUresult encode_boxes(PFN_cuTensorMapEncodeTiled_v12000 encode, CUtensorMap* map, const void* ptr, int64_t cols,
                      int64_t N, int64_t B) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 2), static_cast<cuuint64_t>(N * cols * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kTT), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Slot layout and counts shared by the launchers.  Returns false when fewer
// than two slots fit (the caller then uses the per-head kernels).
bool finish_args(TileArgs& a, uint32_t slot_bytes, int cols, int items, int sm_count, size_t* smem, int* grid,
                 uint32_t reserve = 0) {
  const int slots = static_cast<int>(
      std::min<int64_t>(kMaxSlots, (kTileSmemBudget - 1024 - static_cast<int64_t>(reserve)) / slot_bytes));
  if (slots < 2) return false;
  int pc = 32;
  while (pc < cols) pc *= 2;
  if (pc > 512) return false;
  a.nbuf = 512 / pc < 4 ? 512 / pc : 4;
  a.cols = cols;
  a.slots = slots;
  a.slot_bytes = slot_bytes;
  a.items = items;
  size_t bytes = reserve + static_cast<size_t>(slots) * slot_bytes + 1024;
  if (bytes < kSmemFloor) bytes = kSmemFloor;
  *smem = bytes;
  const int sms = sm_count > 0 ? sm_count : 148;
  *grid = items < sms ? items : sms;
  return items > 0;
}

// The item walk's stride: gridDim.x as (group, middle index, sample) steps.
void set_walk(TileArgs& a, int grid, int mids) {
  a.wdg = grid % a.groups;
  const int rest = grid / a.groups;
  a.wdm = rest % mids;
  a.wdb = rest / mids;
}

TileArgs base_args(const Plan& p, const __half2* phase16, const float* eta_raw, int* status) {
  TileArgs a{};
  a.phase16 = phase16;
  a.eta_raw = eta_raw;
  a.status = status;
  a.N = static_cast<int>(p.N);
  a.H = static_cast<int>(p.H);
  a.d = static_cast<int>(p.d);
  a.hg = p.hg;
  a.groups = p.groups;
  a.nrel = p.nrel;
  a.nval = p.nval;
  a.ntiles = static_cast<int>(ceil_div(p.N, kTT));
  a.ct = p.ct;
  a.nchunks = static_cast<int>(p.nchunks);
  a.pos_batched = p.pos_rows > 1 ? 1 : 0;
  a.W = static_cast<int>(p.W);
  a.rel_tma = static_cast<int>(p.hg * p.R / 64);
  return a;
}

}  // namespace

bool tiled_usable(const Plan& p, std::initializer_list<const void*> ptrs) {
  if (!p.tiled || tensor_map_encoder() == nullptr) return false;
  for (const void* q : ptrs)
    if (!aligned16(q)) return false;
  return true;
}

cudaError_t launch_moments_tiled(const Plan& p, bool bwd, const bf16* proj, const bf16* gout, const __half2* phase16,
                                 float* partial, int* status, int sm_count, cudaStream_t stream) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  CUtensorMap tm_rel{}, tm_val{};
  if (encode_boxes(encode, &tm_rel, proj, p.W, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (bwd) {
    if (encode_boxes(encode, &tm_val, gout, p.D, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  } else {
    tm_val = tm_rel;
  }
  TileArgs a = base_args(p, phase16, nullptr, status);
  a.partial = partial;
  // Traversal order (L2 reuse between consecutive passes): the forward moment
  // pass walks the projection backwards, from the rows the input projection
  // wrote last; the readout then walks forwards, from the rows the moment pass
  // read last.  The backward moment pass walks forwards from the rows the
  // output projection's input-gradient GEMM (reversed) wrote last, and the
  // gradient pass backwards from the rows the backward moment pass read last.
  a.rev = bwd ? 0 : 1;
  // One relation box per item: two heads at R = 32, one at R = 64, and the
  // value boxes holding those heads.  Slot: [relation box (hi in place) |
  // value boxes | the tile's FP16 phase rows]; the lo boxes, written by the
  // rotation warps and read by the MMA, come from a ring of two below the
  // slots, so the slots hold only loaded data.
  a.hg = static_cast<int>(64 / p.R);
  a.groups = static_cast<int>(p.H / a.hg);
  a.nrel = 1;
  a.nval = static_cast<int>(ceil_div(a.hg * p.d, 64));
  // lo ring of two boxes (measured: a ring of one, which leaves room for a fifth slot at r = d = 32,
  // serialises the rotation behind the MMA: moment passes 69 / 64 -> 85 / 80 us)
  a.loring = 2;
  a.off_slots = a.loring * kBox;
  a.off_rel = 0;
  a.off_val = kBox;
  a.load_bytes = (1 + a.nval) * kBox;
  const int cols = bwd ? 64 * a.nval : 64 + 64 * a.nval;
  const int items = static_cast<int>(p.B * a.groups * p.nchunks);
  size_t smem = 0;
  int grid = 0;
  a.off_ph = static_cast<uint32_t>((1 + a.nval) * kBox);
  const uint32_t slot = (a.off_ph + static_cast<uint32_t>(kTT * p.R * 2) + 1023u) & ~1023u;
  if (!finish_args(a, slot, cols, items, sm_count, &smem, &grid, a.loring * kBox)) return cudaErrorInvalidValue;
  set_walk(a, grid, a.nchunks);
  const void* fn = nullptr;
  switch (p.R) {
    case 16: fn = bwd ? reinterpret_cast<const void*>(&moments_tile_kernel<16, true>)
                      : reinterpret_cast<const void*>(&moments_tile_kernel<16, false>); break;
    case 32: fn = bwd ? reinterpret_cast<const void*>(&moments_tile_kernel<32, true>)
                      : reinterpret_cast<const void*>(&moments_tile_kernel<32, false>); break;
    case 48: fn = bwd ? reinterpret_cast<const void*>(&moments_tile_kernel<48, true>)
                      : reinterpret_cast<const void*>(&moments_tile_kernel<48, false>); break;
    case 64: fn = bwd ? reinterpret_cast<const void*>(&moments_tile_kernel<64, true>)
                      : reinterpret_cast<const void*>(&moments_tile_kernel<64, false>); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope(bwd ? "moments_bwd" : "moments_fwd", stream);
  if (p.R == 16) {
    if (bwd) launch_pdl(moments_tile_kernel<16, true>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
    else launch_pdl(moments_tile_kernel<16, false>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
  } else if (p.R == 32) {
    if (bwd) launch_pdl(moments_tile_kernel<32, true>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
    else launch_pdl(moments_tile_kernel<32, false>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
  } else if (p.R == 48) {
    if (bwd) launch_pdl(moments_tile_kernel<48, true>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
    else launch_pdl(moments_tile_kernel<48, false>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
  } else {
    if (bwd) launch_pdl(moments_tile_kernel<64, true>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
    else launch_pdl(moments_tile_kernel<64, false>, grid, kMThreads, smem, stream, tm_rel, tm_val, a);
  }
  return cudaGetLastError();
}

cudaError_t launch_readout_tiled(const Plan& p, const bf16* proj, const __half2* phase16, const bf16* rmat,
                                 const float* eta_raw, bf16* out, int* status, int sm_count, cudaStream_t stream) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  CUtensorMap tm_proj{}, tm_out{};
  if (encode_boxes(encode, &tm_proj, proj, p.W, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_boxes(encode, &tm_out, out, p.D, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  TileArgs a = base_args(p, phase16, eta_raw, status);
  a.rev = 0;  // forwards: the forward moment pass read the first rows last (see launch_moments_tiled)
  a.m0 = rmat;
  a.off_val = p.nrel * kBox;
  a.off_mat = (p.nrel + p.nval) * kBox;
  const uint32_t mat = static_cast<uint32_t>(p.hg * p.d * p.R * 2);
  a.off_ph = a.off_mat + mat;  // the tile's FP16 phase rows (mat is a multiple of 16 bytes)
  a.load_bytes = (p.nrel + p.nval) * kBox + mat;
  const int items = static_cast<int>(p.B * p.groups * ceil_div(p.N, kTT));
  size_t smem = 0;
  int grid = 0;
  const uint32_t slot = static_cast<uint32_t>(tile_slot_bytes(2, p.R, p.d, p.hg));
  if (!finish_args(a, slot, p.hg * static_cast<int>(p.d), items, sm_count, &smem, &grid)) return cudaErrorInvalidValue;
  set_walk(a, grid, a.ntiles);
  const void* fn = p.R == 16   ? reinterpret_cast<const void*>(&readout_tile_kernel<16>)
                   : p.R == 32 ? reinterpret_cast<const void*>(&readout_tile_kernel<32>)
                   : p.R == 48 ? reinterpret_cast<const void*>(&readout_tile_kernel<48>)
                               : reinterpret_cast<const void*>(&readout_tile_kernel<64>);
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope("readout", stream);
  if (p.R == 16) {
    launch_pdl(readout_tile_kernel<16>, grid, kThreadsS, smem, stream, tm_proj, tm_out, a);
  } else if (p.R == 32) {
    launch_pdl(readout_tile_kernel<32>, grid, kThreadsS, smem, stream, tm_proj, tm_out, a);
  } else if (p.R == 48) {
    launch_pdl(readout_tile_kernel<48>, grid, kThreadsS, smem, stream, tm_proj, tm_out, a);
  } else {
    launch_pdl(readout_tile_kernel<64>, grid, kThreadsS, smem, stream, tm_proj, tm_out, a);
  }
  return cudaGetLastError();
}

cudaError_t launch_grad_tiled(const Plan& p, const bf16* gout, const bf16* proj, const __half2* phase16, const bf16* b1y,
                              const bf16* b1c, const bf16* b1a, const float* eta_raw, bf16* gproj,
                              float* etastat, int* status, int sm_count, cudaStream_t stream) {
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  CUtensorMap tm_proj{}, tm_dy{}, tm_gproj{};
  if (encode_boxes(encode, &tm_proj, proj, p.W, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_boxes(encode, &tm_dy, gout, p.D, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_boxes(encode, &tm_gproj, gproj, p.W, p.N, p.B) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  TileArgs a = base_args(p, phase16, eta_raw, status);
  a.rev = 1;  // backwards: the backward moment pass read the last rows last
  a.m0 = b1y;
  a.m1 = b1c;
  a.m2 = b1a;
  a.etastat = etastat;
  a.gproj = gproj;
  a.off_val = p.nrel * kBox;
  a.off_aux = (p.nrel + p.nval) * kBox;
  a.off_ph = (p.nrel + 2 * p.nval) * kBox;
  a.off_mat = a.off_ph + static_cast<uint32_t>(kTT * p.R * 2);
  const uint32_t mat = static_cast<uint32_t>(p.hg * (2 * p.R * p.d + p.R * p.R) * 2);
  a.load_bytes = (p.nrel + 2 * p.nval) * kBox + mat;
  const int items = static_cast<int>(p.B * p.groups * ceil_div(p.N, kTT));
  size_t smem = 0;
  int grid = 0;
  const uint32_t slot = static_cast<uint32_t>(tile_slot_bytes(3, p.R, p.d, p.hg));
  if (!finish_args(a, slot, p.hg * static_cast<int>(p.R + p.d), items, sm_count, &smem, &grid))
    return cudaErrorInvalidValue;
  set_walk(a, grid, a.ntiles);
  const void* fn = p.R == 16   ? reinterpret_cast<const void*>(&grad_tile_kernel<16>)
                   : p.R == 32 ? reinterpret_cast<const void*>(&grad_tile_kernel<32>)
                   : p.R == 48 ? reinterpret_cast<const void*>(&grad_tile_kernel<48>)
                               : reinterpret_cast<const void*>(&grad_tile_kernel<64>);
  cudaError_t e = allow_smem(fn, smem);
  if (e != cudaSuccess) return e;
  LaunchScope scope("grad", stream);
  if (p.R == 16) {
    launch_pdl(grad_tile_kernel<16>, grid, kThreadsS, smem, stream, tm_proj, tm_dy, tm_gproj, a);
  } else if (p.R == 32) {
    launch_pdl(grad_tile_kernel<32>, grid, kThreadsS, smem, stream, tm_proj, tm_dy, tm_gproj, a);
  } else if (p.R == 48) {
    launch_pdl(grad_tile_kernel<48>, grid, kThreadsS, smem, stream, tm_proj, tm_dy, tm_gproj, a);
  } else {
    launch_pdl(grad_tile_kernel<64>, grid, kThreadsS, smem, stream, tm_proj, tm_dy, tm_gproj, a);
  }
  return cudaGetLastError();
}

}  // namespace lsso
