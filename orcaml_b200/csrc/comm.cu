// comm.cu -- the gradient exchange: NCCL all-reduce with averaging over NVLink.
//
// Replaces python/orca/distributed.py:161-256 (a TCP star through rank 0 that
// ships every gradient as big-endian f32 and averages in Python doubles) with
// one NCCL communicator per process/GPU.  The average is fused into the
// reduction (ncclAvg).  NCCL is resolved at run time with dlopen, so the
// library binds to whichever libnccl.so.2 the process already has loaded
// (PyTorch's, when torch is imported first) and loads without NCCL at all.
//
// Communicators are created non-blocking; initialisation and every
// collective are polled against a host deadline, and a communicator that
// misses it is aborted (ncclCommAbort) so the caller gets ORCA_TIMEOUT /
// ORCA_COMM_ERROR instead of a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"

struct orca_comm {
  orca_ctx* ctx = nullptr;
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  double timeout_s = 600.0;
  bool aborted = false;
  cudaEvent_t ev_in = nullptr;    // compute stream -> comm stream ordering
  cudaEvent_t ev_out = nullptr;   // comm stream -> compute stream ordering
};

namespace orca {
namespace {

struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = std::string("libnccl.so.2 not found: ") + dlerror();
      return;
    }
#define SYM(field, name)                                                        \
  a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name));                \
  if (!a.field) { a.why = std::string("missing NCCL symbol ") + name; return; }
    SYM(GetUniqueId, "ncclGetUniqueId");
    SYM(CommInitRankConfig, "ncclCommInitRankConfig");
    SYM(CommGetAsyncError, "ncclCommGetAsyncError");
    SYM(CommAbort, "ncclCommAbort");
    SYM(CommDestroy, "ncclCommDestroy");
    SYM(CommFinalize, "ncclCommFinalize");
    SYM(AllReduce, "ncclAllReduce");
    SYM(GetErrorString, "ncclGetErrorString");
#undef SYM
    a.ok = true;
  });
  return a;
}

orca_status nccl_fail(ncclResult_t r, const char* what) {
  NcclApi& a = api();
  return fail(ORCA_COMM_ERROR, "%s: %s", what, a.GetErrorString ? a.GetErrorString(r) : "nccl error");
}

// Poll a non-blocking communicator until its pending operation completes.
// The first ~50 us spin (a collective's enqueue usually finishes within
// microseconds, and a sleep here would stall the host's enqueue of the rest
// of the step); after that the poll backs off to 50 us sleeps.
orca_status wait_ready(orca_comm* c, const char* what) {
  NcclApi& a = api();
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = a.CommGetAsyncError(c->comm, &st);
    if (r != ncclSuccess) return nccl_fail(r, what);
    if (st == ncclSuccess) return ORCA_OK;
    if (st != ncclInProgress) return nccl_fail(st, what);
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > c->timeout_s) {
      a.CommAbort(c->comm);
      c->aborted = true;
      return fail(ORCA_TIMEOUT, "%s: no progress after %.1f s; communicator aborted", what,
                  c->timeout_s);
    }
    if (el < 50e-6) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

orca_status comm_allreduce_avg_stream(orca_comm* c, float* ptr, size_t n, cudaStream_t stream) {
  if (!c || c->aborted) return fail(ORCA_COMM_ERROR, "communicator unavailable");
  if (n == 0) return ORCA_OK;
  NcclApi& a = api();
  ncclResult_t r = a.AllReduce(ptr, ptr, n, ncclFloat32, ncclAvg, c->comm, stream);
  if (r == ncclInProgress) return wait_ready(c, "ncclAllReduce");
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return ORCA_OK;
}

// =============================================================== peer exchange
// The gradient all-reduce of the step runner as a kernel of its own over the
// ranks' gradient arenas, mapped into every process with CUDA IPC (plain
// peer loads and stores over NVLink; no multicast).  Why not NCCL: the
// persistent GEMMs hold every SM (one 320-thread CTA at 168 registers each,
// which leaves too few registers on the scheduler partitions for another
// block), so a collective overlaps them only on SMs the GEMM leaves free.
// The step runner therefore runs the first part of the dX GEMM on fewer CTAs
// and launches this kernel with a grid sized to the SMs left over: it moves
// a layer's gradients from a handful of SMs in about half the time NCCL's
// kernels took on the same SMs (268 MB at world 2 beside the configs[2] dX
// GEMM, 16 SMs: 0.87 ms against 1.4-2.1 ms).
//
// It also restates the reference's average exactly
// (python/orca/distributed.py:238-256): each element is summed in float64 in
// rank order, multiplied by 1/world in float64 and rounded once to float32 --
// bit for bit the reference's result at every world size (NCCL's ncclAvg
// differs from it in the last bits at world > 2).
//
// Protocol for one range [offset, offset + n) of the arena (one layer), on
// the comm stream after the range's gradients are complete:
//   1. peer_signal_kernel: ready[slot][rank] = seq on every rank;
//   2. peer_reduce_kernel: every block waits until ready[slot][r] >= seq for
//      all r (bounded), then reduces its part of this rank's chunk
//      (n / world floats): loads the chunk from every rank's arena, sums in
//      rank order and stores the average into every rank's arena; the last
//      block to finish sets done[slot][rank] = seq on every rank and waits
//      until done[slot][r] >= seq for all r -- when the kernel completes,
//      every rank's averaged chunk has landed in this rank's arena.
// seq grows by one per step on every rank.  All waits are bounded
// (limit_ns); a wait that runs out sets the device error word, skips the
// rest and signals nothing, so the peers' waits run out too and every rank's
// step reports ORCA_TIMEOUT.
constexpr int kMaxPeers = 8;
constexpr int kPeerThreads = 128;

struct PeerArgs {
  float* base[kMaxPeers];       // arena base on every rank (own pointer at [rank])
  uint32_t* flags[kMaxPeers];   // flag array on every rank: [slot][ready, done][src]
  int world = 1, rank = 0, slot = 0;
  uint32_t seq = 0;
  int64_t offset = 0, n = 0;    // the range, in floats from the arena base
  unsigned* counter = nullptr;  // this rank's finished-block counter of the slot
  int* dev_err = nullptr;
  uint64_t limit_ns = 0;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t* peer_flag(uint32_t* base, int slot, int phase, int src) {
  return base + ((size_t)slot * 2 + phase) * kMaxPeers + src;
}

// Waits until every rank's flag (slot, phase) in this rank's array reaches
// seq (wrap-safe); false after limit_ns, with the device error word set.
__device__ bool peer_wait_all(const PeerArgs& a, int phase) {
  const uint64_t t0 = global_ns();
  for (int r = 0; r < a.world; ++r) {
    const uint32_t* f = peer_flag(a.flags[a.rank], a.slot, phase, r);
    unsigned polls = 0;
    while ((int32_t)(ld_acquire_sys(f) - a.seq) < 0) {
      if ((++polls & 63u) == 0 && global_ns() - t0 > a.limit_ns) {
        atomicExch(a.dev_err, DEV_WAIT_TIMEOUT);
        return false;
      }
      __nanosleep(200);
    }
  }
  return true;
}

__global__ void peer_signal_kernel(PeerArgs a, int phase) {
  __threadfence_system();
  const int r = threadIdx.x;
  if (r < a.world) st_release_sys(peer_flag(a.flags[r], a.slot, phase, a.rank), a.seq);
}

// out = float32(((double)x[0] + x[1] + ... + x[world-1]) * inv_w)
__device__ __forceinline__ float peer_avg(const float (&x)[kMaxPeers], int world, double inv_w) {
  double s = (double)x[0];
#pragma unroll
  for (int r = 1; r < kMaxPeers; ++r)
    if (r < world) s = __dadd_rn(s, (double)x[r]);
  return __double2float_rn(__dmul_rn(s, inv_w));
}

// kU float4 vectors per thread and iteration: the loads of all kU x world
// vectors are issued before any is summed, so a thread keeps kU x world x 16
// bytes in flight (128 bytes at every world size: kU = 8 / world).
template <bool kVec, int kU>
__global__ void __launch_bounds__(kPeerThreads, 6) peer_reduce_kernel(PeerArgs a, double inv_w) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = peer_wait_all(a, 0) ? 1 : 0;
  __syncthreads();
  if (ok) {
    const int64_t per = (cdiv(a.n, (int64_t)a.world) + 3) & ~int64_t(3);
    const int64_t c0 = std::min<int64_t>(a.n, (int64_t)a.rank * per);
    const int64_t c1 = std::min<int64_t>(a.n, c0 + per);
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
    int64_t tail = c0;
    if (kVec) {
      constexpr int R = kMaxPeers / kU;   // ranks this instance can hold (world <= R)
      const int64_t nv = (c1 - c0) / 4;
      for (int64_t v0 = tid; v0 < nv; v0 += nthreads * kU) {
        float4 x[kU][R];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t v = v0 + (int64_t)u * nthreads;
#pragma unroll
          for (int r = 0; r < R; ++r)
            if (r < a.world && v < nv)
              x[u][r] = __ldcg(reinterpret_cast<const float4*>(a.base[r] + a.offset + c0 + 4 * v));
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t v = v0 + (int64_t)u * nthreads;
          if (v >= nv) break;
          float e[kMaxPeers];
          float4 o;
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) e[r] = (r < R && r < a.world) ? x[u][r < R ? r : 0].x : 0.0f;
          o.x = peer_avg(e, a.world, inv_w);
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) e[r] = (r < R && r < a.world) ? x[u][r < R ? r : 0].y : 0.0f;
          o.y = peer_avg(e, a.world, inv_w);
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) e[r] = (r < R && r < a.world) ? x[u][r < R ? r : 0].z : 0.0f;
          o.z = peer_avg(e, a.world, inv_w);
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) e[r] = (r < R && r < a.world) ? x[u][r < R ? r : 0].w : 0.0f;
          o.w = peer_avg(e, a.world, inv_w);
#pragma unroll
          for (int r = 0; r < R; ++r)
            if (r < a.world)
              __stcg(reinterpret_cast<float4*>(a.base[r] + a.offset + c0 + 4 * v), o);
        }
      }
      tail = c0 + 4 * nv;
    }
    for (int64_t j = tail + tid; j < c1; j += nthreads) {
      const int64_t i = a.offset + j;
      float e[kMaxPeers];
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r) e[r] = r < a.world ? __ldcg(a.base[r] + i) : 0.0f;
      const float o = peer_avg(e, a.world, inv_w);
#pragma unroll
      for (int r = 0; r < kMaxPeers; ++r)
        if (r < a.world) __stcg(a.base[r] + i, o);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(a.counter, 1u);
    if (prev == gridDim.x - 1) {
      *a.counter = 0;   // every block has counted: ready for the slot's next use
      if (atomicAdd(a.dev_err, 0) == DEV_OK) {
        __threadfence_system();
        for (int r = 0; r < a.world; ++r)
          st_release_sys(peer_flag(a.flags[r], a.slot, 1, a.rank), a.seq);
        peer_wait_all(a, 1);
      }
    }
  }
}

struct PeerArena {
  orca_comm* comm = nullptr;
  PeerArgs args;                 // base, flags, world, rank, dev_err, limit_ns
  int n_slots = 0;
  uint32_t* flags = nullptr;     // this rank's flag array (exported)
  unsigned* counters = nullptr;  // [n_slots], local
  std::vector<void*> opened;     // peers' mappings
};

void peer_arena_close(PeerArena* pa) {
  if (!pa) return;
  for (void* p : pa->opened) cudaIpcCloseMemHandle(p);
  if (pa->flags) cudaFree(pa->flags);
  if (pa->counters) cudaFree(pa->counters);
  delete pa;
}

orca_status peer_arena_open(orca_comm* c, float* base, int n_slots, PeerArena** out) {
  *out = nullptr;
  if (!c || c->aborted) return fail(ORCA_COMM_ERROR, "communicator unavailable");
  if (c->world < 2 || c->world > kMaxPeers)
    return fail(ORCA_INVALID_ARGUMENT, "peer exchange: world %d not in [2, %d]", c->world,
                kMaxPeers);
  if (n_slots < 1) return fail(ORCA_INVALID_ARGUMENT, "peer exchange: no slots");
  orca_ctx* ctx = c->ctx;
  NcclApi& nc = api();
  PeerArena* pa = new PeerArena();
  pa->comm = c;
  pa->n_slots = n_slots;
  struct Guard {
    PeerArena*& pa;
    ~Guard() { if (pa) peer_arena_close(pa); }
  } guard{pa};
  const size_t flag_bytes = (size_t)n_slots * 2 * kMaxPeers * sizeof(uint32_t);
  ORCA_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&pa->flags), flag_bytes));
  ORCA_CUDA_TRY(cudaMemset(pa->flags, 0, flag_bytes));
  ORCA_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&pa->counters), (size_t)n_slots * 4));
  ORCA_CUDA_TRY(cudaMemset(pa->counters, 0, (size_t)n_slots * 4));
  // Exchange the two IPC handles and the device UUID of every rank through
  // the communicator: a byte-wise sum over a buffer in which each rank fills
  // only its own slot.
  struct Entry {
    cudaIpcMemHandle_t h[2];
    cudaUUID_t uuid;
  } mine;
  ORCA_CUDA_TRY(cudaIpcGetMemHandle(&mine.h[0], base));
  ORCA_CUDA_TRY(cudaIpcGetMemHandle(&mine.h[1], pa->flags));
  cudaDeviceProp prop;
  ORCA_CUDA_TRY(cudaGetDeviceProperties(&prop, ctx->device));
  mine.uuid = prop.uuid;
  const size_t hb = sizeof(mine);
  std::vector<uint8_t> handles((size_t)c->world * hb, 0);
  memcpy(handles.data() + (size_t)c->rank * hb, &mine, hb);
  uint8_t* dbuf = nullptr;
  ORCA_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&dbuf), handles.size()));
  struct FreeBuf {
    uint8_t* p;
    ~FreeBuf() { cudaFree(p); }
  } free_buf{dbuf};
  ORCA_CUDA_TRY(cudaMemcpy(dbuf, handles.data(), handles.size(), cudaMemcpyHostToDevice));
  ncclResult_t r = nc.AllReduce(dbuf, dbuf, handles.size(), ncclUint8, ncclSum, c->comm,
                                ctx->comm_stream);
  if (r == ncclInProgress) ORCA_TRY(wait_ready(c, "ncclAllReduce (IPC handles)"));
  else if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce (IPC handles)");
  ORCA_TRY(sync_stream_for(ctx, ctx->comm_stream, c->timeout_s));
  ORCA_CUDA_TRY(cudaMemcpy(handles.data(), dbuf, handles.size(), cudaMemcpyDeviceToHost));
  // Every rank must own its GPU: the exchange kernels of different ranks
  // wait on one another, which only works when they run on different devices.
  for (int q = 0; q < c->world; ++q) {
    Entry e;
    memcpy(&e, handles.data() + (size_t)q * hb, hb);
    if (q != c->rank && memcmp(&e.uuid, &mine.uuid, sizeof(cudaUUID_t)) == 0)
      return fail(ORCA_INVALID_ARGUMENT, "peer exchange: ranks %d and %d share a GPU", c->rank, q);
  }
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank) {
      pa->args.base[q] = base;
      pa->args.flags[q] = pa->flags;
      continue;
    }
    Entry e;
    memcpy(&e, handles.data() + (size_t)q * hb, hb);
    void* pb = nullptr;
    void* pf = nullptr;
    ORCA_CUDA_TRY(cudaIpcOpenMemHandle(&pb, e.h[0], cudaIpcMemLazyEnablePeerAccess));
    pa->opened.push_back(pb);
    ORCA_CUDA_TRY(cudaIpcOpenMemHandle(&pf, e.h[1], cudaIpcMemLazyEnablePeerAccess));
    pa->opened.push_back(pf);
    pa->args.base[q] = static_cast<float*>(pb);
    pa->args.flags[q] = static_cast<uint32_t*>(pf);
  }
  pa->args.world = c->world;
  pa->args.rank = c->rank;
  pa->args.dev_err = ctx->dev_err;
  pa->args.limit_ns = (uint64_t)(std::min(c->timeout_s, 60.0) * 1e9);
  *out = pa;
  pa = nullptr;   // keep it
  return ORCA_OK;
}

template <bool kVec, int kU>
static int peer_blocks_per_sm() {
  static int v = 0;
  if (!v) {
    int b = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, peer_reduce_kernel<kVec, kU>,
                                                      kPeerThreads, 0) != cudaSuccess || b < 1)
      b = 1;
    v = b;
  }
  return v;
}

template <bool kVec, int kU>
static void launch_peer_reduce(const PeerArgs& a, int64_t per, int sms, double inv_w,
                               cudaStream_t stream) {
  const int64_t want = cdiv(per, 4 * kPeerThreads * kU);
  const int grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((int64_t)sms * peer_blocks_per_sm<kVec, kU>(), want));
  peer_reduce_kernel<kVec, kU><<<grid, kPeerThreads, 0, stream>>>(a, inv_w);
}

orca_status peer_arena_allreduce_avg(PeerArena* pa, int slot, int64_t offset, int64_t n,
                                     uint32_t seq, cudaStream_t stream, int sms) {
  if (!pa || slot < 0 || slot >= pa->n_slots || n < 0 || offset < 0)
    return fail(ORCA_INVALID_ARGUMENT, "peer exchange: bad range");
  if (n == 0) return ORCA_OK;
  PeerArgs a = pa->args;
  a.slot = slot;
  a.seq = seq;
  a.offset = offset;
  a.n = n;
  a.counter = pa->counters + slot;
  orca_ctx* ctx = pa->comm->ctx;
  peer_signal_kernel<<<1, 32, 0, stream>>>(a, 0);
  const int64_t per = (cdiv(n, (int64_t)a.world) + 3) & ~int64_t(3);
  const double inv_w = 1.0 / (double)a.world;
  // Grid: as many blocks as fit on `sms` SMs (the SMs the caller leaves free
  // next to its GEMMs), so that every block runs at once.
  sms = sms > 0 ? std::min(sms, ctx->sm_count) : ctx->sm_count;
  if ((offset & 3) != 0)
    launch_peer_reduce<false, 1>(a, per, sms, inv_w, stream);
  else if (a.world <= 2)
    launch_peer_reduce<true, 4>(a, per, sms, inv_w, stream);
  else if (a.world <= 4)
    launch_peer_reduce<true, 2>(a, per, sms, inv_w, stream);
  else
    launch_peer_reduce<true, 1>(a, per, sms, inv_w, stream);
  count_launch(ctx, 2);
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

}  // namespace orca

using namespace orca;

extern "C" {

orca_status orca_comm_get_unique_id(void* id_out) {
  if (!id_out) return fail(ORCA_INVALID_ARGUMENT, "null id");
  NcclApi& a = api();
  if (!a.ok) return fail(ORCA_COMM_ERROR, "%s", a.why.c_str());
  static_assert(sizeof(ncclUniqueId) == ORCA_COMM_ID_BYTES, "id size");
  ncclUniqueId id;
  ncclResult_t r = a.GetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id_out, &id, sizeof(id));
  return ORCA_OK;
}

orca_status orca_comm_init(orca_ctx* ctx, int rank, int world, const void* id, double timeout_s,
                           orca_comm** out) {
  ORCA_TRY(check_ctx(ctx));
  if (!id || !out) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  // Same validation as _validate_process_group (python/orca/distributed.py:30-40).
  if (world <= 0) return fail(ORCA_INVALID_ARGUMENT, "world_size must be positive");
  if (rank < 0 || rank >= world) return fail(ORCA_INVALID_ARGUMENT, "rank must be in [0, %d)", world);
  if (!(timeout_s > 0)) return fail(ORCA_INVALID_ARGUMENT, "timeout must be positive");
  NcclApi& a = api();
  if (!a.ok) return fail(ORCA_COMM_ERROR, "%s", a.why.c_str());
  orca_comm* c = new orca_comm();
  c->ctx = ctx;
  ctx_retain(ctx);
  c->rank = rank;
  c->world = world;
  c->timeout_s = timeout_s;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  // ORCA_NCCL_MAX_CTAS caps the CTAs (SMs) a collective may occupy: the
  // gradient all-reduce runs beside the next GEMM, which loses those SMs.
  if (const char* e = getenv("ORCA_NCCL_MAX_CTAS")) {
    const int v = atoi(e);
    if (v > 0) cfg.maxCTAs = v;
  }
  ncclResult_t r = a.CommInitRankConfig(&c->comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    ctx_release(ctx);
    delete c;
    return nccl_fail(r, "ncclCommInitRankConfig");
  }
  orca_status s = wait_ready(c, "ncclCommInitRankConfig");
  if (s == ORCA_OK &&
      (cudaEventCreateWithFlags(&c->ev_in, cudaEventDisableTiming) != cudaSuccess ||
       cudaEventCreateWithFlags(&c->ev_out, cudaEventDisableTiming) != cudaSuccess))
    s = fail(ORCA_CUDA_ERROR, "event creation failed");
  if (s != ORCA_OK) {
    if (!c->aborted && c->comm) a.CommAbort(c->comm);
    if (c->ev_in) cudaEventDestroy(c->ev_in);
    if (c->ev_out) cudaEventDestroy(c->ev_out);
    ctx_release(ctx);
    delete c;
    return s;
  }
  *out = c;
  return ORCA_OK;
}

orca_status orca_comm_destroy(orca_comm* c) {
  if (!c) return ORCA_OK;
  NcclApi& a = api();
  struct Release {
    orca_comm* c;
    ~Release() {
      if (c->ev_in) cudaEventDestroy(c->ev_in);
      if (c->ev_out) cudaEventDestroy(c->ev_out);
      ctx_release(c->ctx);
      delete c;
    }
  } release{c};
  if (!c->aborted && c->comm) {
    cudaSetDevice(c->ctx->device);
    // Bounded: a collective that a vanished peer never completes must not
    // hang teardown; the communicator is aborted instead.
    if (sync_stream_for(c->ctx, c->ctx->comm_stream, c->timeout_s) != ORCA_OK) {
      a.CommAbort(c->comm);
      c->aborted = true;
      return fail(ORCA_TIMEOUT, "comm destroy: collectives pending after %.1f s; aborted",
                  c->timeout_s);
    }
    ncclResult_t r = a.CommFinalize(c->comm);
    if (r != ncclSuccess && r != ncclInProgress) {
      a.CommAbort(c->comm);
      return nccl_fail(r, "ncclCommFinalize");
    }
    ORCA_TRY(wait_ready(c, "ncclCommFinalize"));   // aborts on timeout
    a.CommDestroy(c->comm);
  }
  return ORCA_OK;
}

orca_status orca_comm_abort(orca_comm* c) {
  if (!c) return ORCA_OK;
  NcclApi& a = api();
  if (!c->aborted && c->comm) a.CommAbort(c->comm);
  c->aborted = true;
  return ORCA_OK;
}

orca_status orca_comm_allreduce_avg(orca_comm* c, float* dev_ptr, size_t n) {
  if (!c) return fail(ORCA_INVALID_ARGUMENT, "null communicator");
  ORCA_TRY(check_ctx(c->ctx));
  std::lock_guard<std::mutex> lk(c->ctx->mu);
  ORCA_CUDA_TRY(cudaEventRecord(c->ev_in, c->ctx->stream));
  ORCA_CUDA_TRY(cudaStreamWaitEvent(c->ctx->comm_stream, c->ev_in, 0));
  orca_status s = comm_allreduce_avg_stream(c, dev_ptr, n, c->ctx->comm_stream);
  ORCA_CUDA_TRY(cudaEventRecord(c->ev_out, c->ctx->comm_stream));
  ORCA_CUDA_TRY(cudaStreamWaitEvent(c->ctx->stream, c->ev_out, 0));
  return s;
}

orca_status orca_comm_allreduce_avg_bufs(orca_comm* c, orca_buf* const* bufs, int nbufs,
                                         size_t bucket_bytes) {
  if (!c || (!bufs && nbufs)) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  for (int i = 0; i < nbufs; ++i) {
    if (!bufs[i] || bufs[i]->dtype != ORCA_F32)
      return fail(ORCA_UNSUPPORTED_DTYPE, "all-reduce: F32 buffers only");
    const size_t n = bufs[i]->n;
    const size_t chunk = bucket_bytes ? std::max<size_t>(bucket_bytes / 4, 1) : n;
    for (size_t off = 0; off < n; off += chunk)
      ORCA_TRY(orca_comm_allreduce_avg(c, (float*)bufs[i]->ptr + off, std::min(chunk, n - off)));
  }
  return ORCA_OK;
}

}  // extern "C"
