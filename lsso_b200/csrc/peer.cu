// One-shot all-reduce of the data-parallel gradient buffer over peer memory.
//
// Every rank (one process per GPU) owns an exchange region (peer.h): a small
// header of flags and the flat FP32 gradient buffer its backward writes.  The
// regions are mapped into every other rank's address space (CUDA IPC), so a
// kernel reads the peers' gradients straight over NVLink / NVSwitch.  One
// launch per exchange and rank:
//
//   arrive  CTA 0 tells every peer that this rank's buffer is complete (the
//           kernels that wrote it finished before this launch started);
//           every CTA waits until all peers have said the same;
//   reduce  each thread sums one 16-byte column of all ranks' buffers (the
//           values [first, first + count) of each region) in
//           rank order 0..world-1 (so every rank gets bit-identical values)
//           and writes sum * scale to its local output;
//   depart  the last CTA to finish tells every peer that this rank is done
//           reading, then waits until all peers are: only then may any rank's
//           next backward overwrite its buffer.
//
// Exchanges are numbered by a counter each rank keeps in its own header
// (advanced once per launch by the last CTA); the flags carry that number, so
// nothing is ever reset between exchanges and the launch can be replayed from
// a CUDA graph.  Every wait is bounded: when a peer does not come within the
// limit the kernel records kStatusPeerWaitTimeout in the status word and goes
// on (the output is then undefined), so a lost rank shows up as an error on
// the host instead of a hung GPU.  No TMA and no multicast: plain loads of
// peer memory and system-scope release / acquire flag operations.
#include "peer.h"
#include "tc.cuh"

namespace lsso {
namespace {

constexpr int kPeerThreads = 128;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[j] has reached `epoch` for every rank j other than `rank`
// (wrap-safe comparison).  False after `limit_ns` without that.
__device__ __forceinline__ bool wait_peers(const unsigned* flags, int world, int rank, unsigned epoch, unsigned long long limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int j = 0; j < world; ++j) {
    if (j == rank) continue;
    while (static_cast<int>(ld_acquire_sys(flags + j) - epoch) < 0) {
      if (globaltimer_ns() - t0 > limit_ns) return false;
      __nanosleep(100);
    }
  }
  return true;
}

// (Loops over the ranks are unrolled over W, and the kernel parameter is a
// __grid_constant__, so that its region array stays in parameter space.)
template <int W>
__device__ __forceinline__ void signal_peers(const PeerArgs& a, size_t offset, unsigned epoch) {
  __threadfence_system();
#pragma unroll
  for (int j = 0; j < W; ++j) {
    if (j != a.rank) st_release_sys(reinterpret_cast<unsigned*>(a.region[j] + offset) + a.rank, epoch);
  }
}

template <int W>
__global__ void __launch_bounds__(kPeerThreads, 8) peer_allreduce_kernel(const __grid_constant__ PeerArgs a) {
  char* mine = a.region[0];
#pragma unroll
  for (int j = 1; j < W; ++j) {
    if (j == a.rank) mine = a.region[j];
  }
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(mine + kPeerEpochOffset) + 1u;

  // arrive (thread 0's outcome reaches the CTA through the barrier itself: the
  // kernel uses no shared memory, so a CTA fits on an SM beside a projection
  // GEMM that leaves only the per-CTA reservation free)
  int ok = 0;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) signal_peers<W>(a, kPeerArriveOffset, epoch);
    ok = wait_peers(reinterpret_cast<const unsigned*>(mine + kPeerArriveOffset), W, a.rank, epoch, a.limit_ns);
    if (!ok) atomicExch(a.status, kStatusPeerWaitTimeout);
  }
  ok = __syncthreads_or(ok);

  // reduce
  if (ok) {
    const float4* src[W];
#pragma unroll
    for (int r = 0; r < W; ++r) {
      src[r] = reinterpret_cast<const float4*>(a.region[r] + kPeerDataOffset) + (a.first >> 2);
    }
    float4* out = reinterpret_cast<float4*>(a.out);
    const int64_t n4 = a.count >> 2;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kPeerThreads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * kPeerThreads + threadIdx.x; i < n4; i += stride) {
      float4 v[W];
#pragma unroll
      for (int r = 0; r < W; ++r) v[r] = __ldcg(src[r] + i);
      float4 s = v[0];
#pragma unroll
      for (int r = 1; r < W; ++r) {
        s.x += v[r].x;
        s.y += v[r].y;
        s.z += v[r].z;
        s.w += v[r].w;
      }
      s.x *= a.scale;
      s.y *= a.scale;
      s.z *= a.scale;
      s.w *= a.scale;
      out[i] = s;
    }
    const int64_t tail = n4 << 2;
    if (blockIdx.x == 0 && tail + threadIdx.x < a.count) {
      const int64_t i = tail + threadIdx.x;
      float v[W];
#pragma unroll
      for (int r = 0; r < W; ++r) {
        v[r] = __ldcg(reinterpret_cast<const float*>(a.region[r] + kPeerDataOffset) + a.first + i);
      }
      float s = v[0];
#pragma unroll
      for (int r = 1; r < W; ++r) s += v[r];
      a.out[i] = s * a.scale;
    }
  }

  // depart
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    unsigned* counter = reinterpret_cast<unsigned*>(mine + kPeerCounterOffset);
    if (atomicAdd(counter, 1u) == gridDim.x - 1) {
      atomicExch(counter, 0u);
      signal_peers<W>(a, kPeerDepartOffset, epoch);
      if (!wait_peers(reinterpret_cast<const unsigned*>(mine + kPeerDepartOffset), W, a.rank, epoch, a.limit_ns)) {
        atomicExch(a.status, kStatusPeerWaitTimeout);
      }
      *reinterpret_cast<volatile unsigned*>(mine + kPeerEpochOffset) = epoch;
    }
  }
}

template <int W>
cudaError_t launch_w(const PeerArgs& a, int grid, cudaStream_t stream) {
  peer_allreduce_kernel<W><<<grid, kPeerThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_peer_allreduce(const PeerArgs& a, int sm_count, cudaStream_t stream) {
  // One 16-byte column per thread; at most two CTAs per SM (the loop strides
  // over the rest).  At least one CTA, which carries the flags when count = 0.
  const int64_t n4 = (a.count + 3) >> 2;
  int64_t grid = (n4 + kPeerThreads - 1) / kPeerThreads;
  if (grid < 1) grid = 1;
  if (grid > 2 * static_cast<int64_t>(sm_count)) grid = 2 * static_cast<int64_t>(sm_count);
  const int g = static_cast<int>(grid);
  switch (a.world) {
    case 1: return launch_w<1>(a, g, stream);
    case 2: return launch_w<2>(a, g, stream);
    case 3: return launch_w<3>(a, g, stream);
    case 4: return launch_w<4>(a, g, stream);
    case 5: return launch_w<5>(a, g, stream);
    case 6: return launch_w<6>(a, g, stream);
    case 7: return launch_w<7>(a, g, stream);
    case 8: return launch_w<8>(a, g, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace lsso
