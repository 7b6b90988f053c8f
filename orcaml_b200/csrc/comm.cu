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
