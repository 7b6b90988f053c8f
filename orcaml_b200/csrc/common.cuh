// common.cuh -- internals shared by the CUDA sources of liborca_cuda.so.
//
// Status plumbing for the C ABI (include/orca_cuda.h), the context/buffer
// structs, and the sm_100a device helpers: bounded mbarrier waits, TMA tile
// loads and the tcgen05 (5th-generation tensor core + tensor memory) PTX
// wrappers used by the GEMM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/orca_cuda.h"

namespace orca {

// ---------------------------------------------------------------- host status
void set_error(const char* fmt, ...);
orca_status fail(orca_status s, const char* fmt, ...);
// Gradient exchange over peer memory (comm.cu): the arena `base` (a cudaMalloc
// allocation of every rank, same layout) is mapped into every rank's process;
// peer_arena_allreduce_avg averages [offset, offset + n) of it across ranks,
// enqueued on `stream`; seq must grow by one per use of a slot on every rank.
struct PeerArena;
orca_status peer_arena_open(orca_comm* c, float* base, int n_slots, PeerArena** out);
orca_status peer_arena_allreduce_avg(PeerArena* pa, int slot, int64_t offset, int64_t n,
                                     uint32_t seq, cudaStream_t stream, int sms = 0);
void peer_arena_close(PeerArena* pa);
// Looks up, once per device, the device address of the fixed scratch array of
// orca_softmax_ce_fwd_bwd_noalloc (mlp.cu); the device must be current.
orca_status ce_scratch_setup(int device);

#define ORCA_CUDA_TRY(expr)                                                        \
  do {                                                                             \
    cudaError_t _e = (expr);                                                       \
    if (_e != cudaSuccess)                                                         \
      return ::orca::fail(ORCA_CUDA_ERROR, "%s failed: %s (%s:%d)", #expr,         \
                          cudaGetErrorString(_e), __FILE__, __LINE__);             \
  } while (0)

#define ORCA_TRY(expr)                                                             \
  do {                                                                             \
    orca_status _s = (expr);                                                       \
    if (_s != ORCA_OK) return _s;                                                  \
  } while (0)

// Device error word values (ctx->dev_err).
enum DeviceError : int {
  DEV_OK = 0,
  DEV_WAIT_TIMEOUT = 1,      // an mbarrier wait ran past its bound
  DEV_BAD_LAUNCH = 2,        // a kernel saw an impossible configuration
};

}  // namespace orca

struct orca_ctx {
  // Buffers, step runners and communicators each hold a reference; the
  // context is torn down when the last one is released (orca_ctx_destroy
  // drops the creator's reference), so no object outlives its streams.
  std::atomic<int> refs{1};
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;        // compute stream
  cudaStream_t comm_stream = nullptr;   // collectives
  int* dev_err = nullptr;               // device error word (DeviceError)
  int* tile_ctr = nullptr;              // tile counter of the persistent GEMM (reset per launch)
  double sync_timeout_s = 600.0;        // bound on every synchronising call
  cudaEvent_t sync_event = nullptr;
  std::mutex mu;
  std::atomic<uint64_t> launches{0};
};

struct orca_buf {
  orca_ctx* ctx = nullptr;
  void* ptr = nullptr;
  size_t n = 0;                // elements
  orca_dtype dtype = ORCA_F32;
  std::atomic<int> refs{1};
};

namespace orca {

size_t dtype_size(orca_dtype d);
orca_status check_ctx(orca_ctx* ctx);
orca_status new_buf(orca_ctx* ctx, size_t n, orca_dtype dtype, orca_buf** out);
void ctx_retain(orca_ctx* ctx);
void ctx_release(orca_ctx* ctx);
// Waits for a stream with a deadline (never blocks forever); ORCA_TIMEOUT
// when the deadline passes.  sync_stream uses the compute stream and the
// context's deadline.
orca_status sync_stream(orca_ctx* ctx);
orca_status sync_stream_for(orca_ctx* ctx, cudaStream_t stream, double timeout_s);
// Host wait for an event, polled up to timeout_s (ORCA_TIMEOUT after it).  An
// event never recorded counts as complete.
orca_status wait_event_for(cudaEvent_t event, double timeout_s);
// Device -> (pageable) host copy after the compute stream.  A copy into
// pageable memory blocks the calling thread until the stream reaches it, with
// no bound, so the stream is first drained with the deadline: a stream that
// never drains gives ORCA_TIMEOUT instead of a thread stuck in the copy.
orca_status copy_to_host(orca_ctx* ctx, void* dst, const void* src, size_t bytes);
// Reads and clears the device error word (synchronises the compute stream).
orca_status check_device_error(orca_ctx* ctx);
inline void count_launch(orca_ctx* ctx, uint64_t n = 1) { ctx->launches += n; }

__host__ __device__ inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------- numerics
// Split of an fp32 value into a TF32-exact high part (round to nearest, ties
// away, on the 10 explicit mantissa bits kept) and the exact fp32 residual:
// x == hi + lo bit-exactly.  Three TF32 products hi*hi + hi*lo + lo*hi give an
// fp32-accurate product.
__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u) return x;         // inf / nan unchanged
  uint32_t r = (u + 0x1000u) & 0xffffe000u;
  if ((r & 0x7f800000u) == 0x7f800000u) r = u & 0xffffe000u;  // would overflow: truncate
  return __uint_as_float(r);
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = tf32_hi(x);
  lo = __fsub_rn(x, hi);
}

// ---------------------------------------------------------------- time bound
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every device-side wait of this library gives up after this long and
// reports DEV_WAIT_TIMEOUT instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and
// raises *abort) when the bound runs out or another role already aborted.
// The clock and the abort flag are checked every 64 polls only; sleep_ns > 0
// backs off between polls (for waiters whose latency is not critical, so the
// issue slots stay with the MMA warp).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort, int* dev_err,
                                          unsigned sleep_ns = 0,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (sleep_ns) __nanosleep(sleep_ns);
    if ((it & 63u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > limit_ns) {
        *abort = 1;
        if (dev_err) atomicExch(dev_err, DEV_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
// 3-D tiled bulk tensor load global -> shared, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 4-D tiled load (an MN-major operand tile as one box: {32 mn, k, plane,
// 32-wide chunk}, see make_map4d in gemm.cu).
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cl, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cl), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

// The same load issued by the odd CTA of a pair, its completion counted on the
// even CTA's barrier (bar_cl: shared::cluster address); the bytes land in
// this CTA's own shared memory.
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cl, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cl), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// L2 eviction policies for cache-hinted loads and stores.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tma_load_3d / tma_load_4d with an L2 cache policy.
__device__ __forceinline__ void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int x, int y, int z,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
      "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_hint(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int x, int y, int z, int w,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w),
      "l"(policy)
      : "memory");
}

// 128-bit global store with an L2 cache policy.
__device__ __forceinline__ void st_global_v4_hint(void* p, float4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp TMEM allocation; the base address is written to *slot (smem).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, issued by one thread.
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- CTA pairs
// Helpers of the two-CTA (cluster of 2) tensor-core kernel.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Every thread of both CTAs: release this CTA's prior writes, acquire the
// other's (the cluster-wide counterpart of __syncthreads).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
               "memory");
}
// Arrive on an mbarrier of either CTA of the pair (default semantics,
// release at CTA scope: a cluster-scope release would put a full memory fence
// on every hand-off, and the data these barriers guard -- shared memory
// written by TMA, TMEM -- is ordered by the async-proxy completions and the
// tcgen05 fences, not by this thread's own writes).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
__device__ __forceinline__ void st_remote_u32(uint32_t cl_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cl_addr), "r"(v) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (both CTAs' TMEM, M = 256) (+)= A (128 rows from each CTA) * B (N/2
// columns from each CTA), issued by one thread of the even CTA.
__device__ __forceinline__ void tc_mma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at shared::cluster address cl_addr (either CTA
// of the pair) when the pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t cl_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   cl_addr)
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base lane + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace orca
