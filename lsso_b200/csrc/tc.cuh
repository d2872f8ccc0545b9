// Thin device-side wrappers for the sm_100a instructions the mixer uses:
// tcgen05 (TMEM allocation, BF16 MMA, commit, TMEM loads), mbarriers,
// cp.async and the proxy/thread-sync fences.  Every wait is bounded: a wait
// that runs out records an error code in a device flag and returns false so
// the caller can skip ahead to its TMEM release instead of spinning forever.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <utility>

namespace lsso {

// Error codes written to the device status word.
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusMmaWaitTimeout = 1,
  kStatusPeerWaitTimeout = 2,  // a peer rank did not reach the gradient exchange in time
};

// Time bound of a sleeping mbarrier wait: any legitimate wait inside one of
// these kernels takes microseconds, so one second means a broken schedule.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// The status word the kernels receive (`int* status`) is the first member of
// this per-device block.  `wait_limit_ns` bounds the pipeline waits (the
// waits that also watch an in-CTA abort flag); it is kWaitLimitNs unless a
// test shortens it (lsso_set_wait_limit_ns) to make those waits run out and
// exercise the abort path.  Drain waits of the abort path always keep
// kWaitLimitNs.
struct DeviceControl {
  int status;
  int reserved;
  unsigned long long wait_limit_ns;
};
// Suspend-time hint of one sleeping try_wait: the thread wakes when the phase
// completes or after this long, whichever comes first.
constexpr uint32_t kSuspendHintNs = 20000u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of the library is launched with programmatic stream
// serialisation (launch_pdl): the launch of its grid proceeds as the blocks of
// the previous kernel on the stream exit, instead of after that kernel's
// completion has been processed.  Each kernel therefore starts with
// pdl_wait(), which returns once the previous grid has completed and its
// memory operations are visible (immediately when there is no such
// dependency), and touches no global memory before it; since every kernel
// waits, the outputs of all earlier kernels on the stream are complete too.
// (Triggering the next launch explicitly at the start of each kernel was
// measured slower: the dependent grid's blocks then crowd the tail.)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- cp.async
// 16-byte global->shared copy; bytes beyond src_bytes (0 or 16) are zero-filled.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that lets the hardware suspend the thread until the phase
// completes (or the hint runs out) instead of returning at once, so waiting
// warps stop taking issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
// Bounded, sleeping wait on one phase of an mbarrier.  Gives up (returns
// false) when *abort_flag is set by another role, or after the time limit, in
// which case it sets *abort_flag and records a timeout in the status word.
// The limit is the control block's wait_limit_ns for a pipeline wait (one
// with an abort flag) and kWaitLimitNs otherwise; a limit below the sleep
// hint polls without sleeping, so it runs out as soon as the phase is late.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t limit = kWaitLimitNs;
  if (abort_flag != nullptr && status != nullptr) {
    // Through the read-only cache: the limit does not change while kernels of
    // the library run (the host sets it between calls), and a wait that
    // missed its first try re-checks the barrier only once this load returns,
    // so an L2 round trip here would delay every such wait.
    limit = __ldg(&reinterpret_cast<const DeviceControl*>(status)->wait_limit_ns);
  }
  const bool sleep = limit >= kSuspendHintNs;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (sleep ? mbar_try_wait_sleep(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (globaltimer_ns() - t0 > limit) break;
  }
  if (abort_flag != nullptr) *abort_flag = 1;
  if (status != nullptr) atomicExch(status, kStatusMmaWaitTimeout);
  return false;
}
// Bounded wait on one phase of an mbarrier.  On timeout, raises the status
// flag and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* status) {
  return mbar_wait_bounded(bar, parity, nullptr, status);
}

// Arrive once and announce `bytes` of transaction traffic (TMA / bulk copies).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------- TMA (no multicast)
// 2-D tiled tensor load into this CTA's shared memory, completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
// 2-D tiled tensor store from this CTA's shared memory (bulk-group completion).
// Rows/columns of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(tmap), "r"(src),
               "r"(c0), "r"(c1)
               : "memory");
}
// 3-D tiled tensor store from this CTA's shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const void* tmap, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];\n" ::"l"(tmap),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups are incomplete (writes performed).
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;\n" ::"n"(N) : "memory");
}
// 3-D tiled tensor load into this CTA's shared memory, completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, int c0, int c1, int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
// Contiguous global->shared bulk copy (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// Prefetch one 3-D tensor-map box into L2 (no shared memory, no completion):
// a later TMA load of the same box then hits L2.
__device__ __forceinline__ void tma_prefetch_3d(const void* tmap, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];\n" ::"l"(tmap), "r"(c0), "r"(c1),
               "r"(c2)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- fences
// Make generic-proxy shared-memory writes visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// ---------------------------------------------------------------- TMEM
// Warp-collective: allocate ncols (power of two >= 32) TMEM columns; the base
// address is written to shared memory at dst.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---------------------------------------------------------------- MMA
// Shared-memory matrix descriptor for the no-swizzle (interleaved) canonical
// layout.  The operand is a grid of 8x16-byte core matrices (128 contiguous
// bytes each); lbo is the byte distance between core matrices adjacent along
// K and sbo the distance between core matrices adjacent along M/N.
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  return d;                             // base offset 0, swizzle none
}

// Descriptor of the 128-byte-swizzled canonical layout (the layout a TMA box
// with a 128-byte inner dimension and CU_TENSOR_MAP_SWIZZLE_128B produces).
// K-major: 8-row atoms of 128-byte rows, sbo = atom stride (1024), lbo unused
// (16), a K-step of 16 elements advances the start address by 32 bytes.
// MN-major: 64-element rows, 8 K-rows per 1024-byte atom, sbo = K-atom
// stride, lbo = stride between 64-element MN groups.  Atoms are 1024-aligned.
__device__ __forceinline__ uint64_t make_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return make_desc(saddr, lbo, sbo) | (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16: BF16 A and B, FP32 D.
// a_mn / b_mn select the MN-major (transposed) operand layout.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A * B^T, one instruction of K = 16; issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier when every MMA issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}

// Teardown by the MMA-issuing thread: one more commit, to `bar` (an mbarrier
// of count 1 used for nothing else), tracks every tensor-core operation this
// thread issued; waiting on it (bounded by kWaitLimitNs) means none still
// writes TMEM or reads shared memory when the CTA frees its TMEM and exits --
// after an abort as much as after a normal run (then it returns at once).
__device__ __forceinline__ void mma_drain(uint32_t bar, int* status) {
  mma_commit(bar);
  mbar_wait_bounded(bar, 0, nullptr, status);
}

// Warp-collective TMEM load: 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// Warp-collective TMEM load: 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// Warp-collective TMEM load: 32 lanes x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// BF16 -> FP32 is exact: the BF16 bits are the high half of the FP32 bits.
// Integer ops keep the conversion off the (narrow) conversion pipe.
__device__ __forceinline__ float2 unpack_bf16(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
__host__ __device__ constexpr uint32_t tmem_cols_for(uint32_t n) {
  return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}

// Position (entry s, pass u) in a ring of n entries, advanced one step at a time.
struct RingPos {
  int s = 0, u = 0;
  __device__ __forceinline__ void next(int n) {
    if (++s == n) {
      s = 0;
      ++u;
    }
  }
};

}  // namespace lsso
