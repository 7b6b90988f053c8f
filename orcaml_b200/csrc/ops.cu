// ops.cu -- context, buffers and the Backend-trait primitive ops of the C ABI.
//
// Each op restates the semantics of the reference CPU backend
// (orca-backend-cpu/src/backend.rs) on the device: element-wise ops are one
// IEEE f32 rounding per element (no contraction), and the shape reductions
// (sum_to_shape, max_to_shape) visit each output's inputs in ascending linear
// input order, which is the reference's serial order, so they are bit-exact.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace orca {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

orca_status fail(orca_status s, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

size_t dtype_size(orca_dtype d) {
  switch (d) {
    case ORCA_F32: case ORCA_I32: return 4;
    case ORCA_F64: case ORCA_I64: return 8;
    case ORCA_F16: case ORCA_BF16: return 2;
    case ORCA_U8: case ORCA_BOOL: return 1;
  }
  return 0;
}

orca_status check_ctx(orca_ctx* ctx) {
  if (!ctx) return fail(ORCA_INVALID_ARGUMENT, "null context");
  ORCA_CUDA_TRY(cudaSetDevice(ctx->device));
  return ORCA_OK;
}

void ctx_retain(orca_ctx* ctx) { ctx->refs++; }

void ctx_release(orca_ctx* ctx) {
  if (--ctx->refs != 0) return;
  cudaSetDevice(ctx->device);
  // Bounded: a stream that never drains (a peer gone mid-collective whose
  // communicator was not aborted) must not hang the caller's teardown.
  sync_stream_for(ctx, ctx->stream, ctx->sync_timeout_s);
  sync_stream_for(ctx, ctx->comm_stream, ctx->sync_timeout_s);
  cudaFree(ctx->dev_err);
  cudaFree(ctx->tile_ctr);
  if (ctx->sync_event) cudaEventDestroy(ctx->sync_event);
  cudaStreamDestroy(ctx->stream);
  cudaStreamDestroy(ctx->comm_stream);
  delete ctx;
}

orca_status new_buf(orca_ctx* ctx, size_t n, orca_dtype dtype, orca_buf** out) {
  if (!out) return fail(ORCA_INVALID_ARGUMENT, "null output pointer");
  size_t es = dtype_size(dtype);
  if (!es) return fail(ORCA_UNSUPPORTED_DTYPE, "unknown dtype %d", (int)dtype);
  orca_buf* b = new orca_buf();
  b->ctx = ctx;
  b->n = n;
  b->dtype = dtype;
  if (n) {
    cudaError_t e = cudaMallocAsync(&b->ptr, n * es, ctx->stream);
    if (e != cudaSuccess) {
      delete b;
      return fail(ORCA_CUDA_ERROR, "device allocation of %zu bytes failed: %s", n * es,
                  cudaGetErrorString(e));
    }
  }
  ctx_retain(ctx);
  *out = b;
  return ORCA_OK;
}

orca_status sync_stream(orca_ctx* ctx) {
  return sync_stream_for(ctx, ctx->stream, ctx->sync_timeout_s);
}

orca_status sync_stream_for(orca_ctx* ctx, cudaStream_t stream, double timeout_s) {
  ORCA_CUDA_TRY(cudaEventRecord(ctx->sync_event, stream));
  return wait_event_for(ctx->sync_event, timeout_s);
}

orca_status wait_event_for(cudaEvent_t event, double timeout_s) {
  const auto t0 = std::chrono::steady_clock::now();
  for (int it = 0;; ++it) {
    const cudaError_t e = cudaEventQuery(event);
    if (e == cudaSuccess) return ORCA_OK;
    if (e != cudaErrorNotReady)
      return fail(ORCA_CUDA_ERROR, "stream error: %s", cudaGetErrorString(e));
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s)
      return fail(ORCA_TIMEOUT, "device work still pending after %.1f s", timeout_s);
    if (it > 1000) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

orca_status copy_to_host(orca_ctx* ctx, void* dst, const void* src, size_t bytes) {
  ORCA_TRY(sync_stream(ctx));
  if (!bytes) return ORCA_OK;
  ORCA_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  return sync_stream(ctx);
}

orca_status check_device_error(orca_ctx* ctx) {
  int h = 0;
  ORCA_TRY(copy_to_host(ctx, &h, ctx->dev_err, sizeof(int)));
  if (h != DEV_OK) {
    ORCA_CUDA_TRY(cudaMemsetAsync(ctx->dev_err, 0, sizeof(int), ctx->stream));
    if (h == DEV_WAIT_TIMEOUT)
      return fail(ORCA_TIMEOUT, "a device-side wait ran past its bound (results discarded)");
    return fail(ORCA_INTERNAL, "device error word %d", h);
  }
  return ORCA_OK;
}

// ---------------------------------------------------------------- shapes
struct ShapeInfo {
  static constexpr int MAXR = 8;
  int rank = 0;
  int64_t d[MAXR] = {};
};

static orca_status to_shape(const int64_t* dims, int rank, ShapeInfo& s, int64_t* numel) {
  if (rank < 0 || rank > ShapeInfo::MAXR) return fail(ORCA_INVALID_ARGUMENT, "rank %d", rank);
  if (rank > 0 && !dims) return fail(ORCA_INVALID_ARGUMENT, "null dims");
  s.rank = rank;
  int64_t n = 1;
  for (int i = 0; i < rank; ++i) {
    if (dims[i] < 0) return fail(ORCA_INVALID_ARGUMENT, "negative dim");
    s.d[i] = dims[i];
    n *= dims[i];
  }
  *numel = n;
  return ORCA_OK;
}

// pad_shape_left (backend.rs:17-26)
static ShapeInfo pad_left(const ShapeInfo& s, int target) {
  ShapeInfo p;
  p.rank = target;
  for (int i = 0; i < target; ++i) p.d[i] = 1;
  if (s.rank <= target)
    for (int i = 0; i < s.rank; ++i) p.d[target - s.rank + i] = s.d[i];
  return p;
}

static orca_status need(const orca_buf* b, size_t n, const char* what) {
  if (!b) return fail(ORCA_INVALID_ARGUMENT, "%s: null buffer", what);
  if (b->n < n)
    return fail(ORCA_SHAPE_MISMATCH, "%s: buffer holds %zu elements, shape needs %zu", what, b->n, n);
  return ORCA_OK;
}

static orca_status need_f32(orca_dtype d, const char* what) {
  if (d != ORCA_F32)
    return fail(ORCA_UNSUPPORTED_DTYPE, "%s: the CUDA backend computes in F32 only (got %d)", what,
                (int)d);
  return ORCA_OK;
}

static int grid_for(orca_ctx* ctx, int64_t n, int threads = 256) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, threads), (int64_t)ctx->sm_count * 16));
}

// ---------------------------------------------------------------- kernels
enum BinOp : int { B_ADD, B_SUB, B_MUL, B_DIV, B_RELU_BW, B_SIGMOID_BW, B_EXP_BW, B_LOG_BW,
                   B_SQRT_BW, B_DIV_BW_LHS };
enum UnOp : int { U_RELU, U_SIGMOID, U_EXP, U_LOG, U_SQRT, U_MULS };

__global__ void binary_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                              float* __restrict__ o, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float x = a[i], y = b[i], r;
    switch (op) {
      case B_ADD: r = __fadd_rn(x, y); break;
      case B_SUB: r = __fsub_rn(x, y); break;
      case B_MUL: r = __fmul_rn(x, y); break;
      case B_DIV: r = __fdiv_rn(x, y); break;
      case B_RELU_BW: r = y > 0.0f ? x : 0.0f; break;                    // backend.rs:432-434
      case B_SIGMOID_BW: r = __fmul_rn(__fmul_rn(x, y), __fsub_rn(1.0f, y)); break;  // :458-460
      case B_EXP_BW: r = __fmul_rn(x, y); break;                         // :603
      case B_LOG_BW: r = __fdiv_rn(x, y); break;                         // :629 (no clamp)
      case B_SQRT_BW: r = __fdiv_rn(x, __fmul_rn(2.0f, y)); break;       // :755
      default: r = __fdiv_rn(x, y); break;                               // div_backward_lhs
    }
    o[i] = r;
  }
}

__global__ void div_bw_rhs_kernel(const float* g, const float* l, const float* r, float* o,
                                  int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    o[i] = __fmul_rn(g[i], __fdiv_rn(-l[i], __fmul_rn(r[i], r[i])));   // backend.rs:727
}

__global__ void unary_kernel(int op, const float* __restrict__ a, float* __restrict__ o, int64_t n,
                             float s) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float x = a[i], r;
    switch (op) {
      case U_RELU: r = x > 0.0f ? x : 0.0f; break;                                   // :384-386
      case U_SIGMOID: r = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); break;        // :406-408
      case U_EXP: r = expf(x); break;
      case U_LOG: r = logf(fmaxf(x, 1e-7f)); break;                                  // :577
      case U_SQRT: r = __fsqrt_rn(x); break;
      default: r = __fmul_rn(x, s); break;
    }
    o[i] = r;
  }
}

// out[i] = in[map(i)] over the broadcast (expand, backend.rs:466-497).
__global__ void expand_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n,
                              ShapeInfo out_s, ShapeInfo padded_in) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, idx = 0, st = 1;
    for (int d = out_s.rank - 1; d >= 0; --d) {
      int64_t c = rem % out_s.d[d];
      rem /= out_s.d[d];
      if (padded_in.d[d] != 1) idx += c * st;
      st *= padded_in.d[d];
    }
    out[i] = in[idx];
  }
}

// One thread per output; inputs visited in ascending linear order (mode 0 sum
// from 0.0, mode 1 max from -FLT_MAX with strict >).
__global__ void reduce_to_shape_kernel(int mode, const float* __restrict__ in,
                                       float* __restrict__ out, int64_t n_out, ShapeInfo in_s,
                                       ShapeInfo padded_out) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < n_out;
       o += (int64_t)gridDim.x * blockDim.x) {
    // Decode o in the padded output shape; kept coordinates are fixed.
    int64_t coord[ShapeInfo::MAXR];
    int64_t rem = o;
    for (int d = in_s.rank - 1; d >= 0; --d) {
      coord[d] = rem % padded_out.d[d];
      rem /= padded_out.d[d];
    }
    int64_t red_total = 1;
    for (int d = 0; d < in_s.rank; ++d)
      if (padded_out.d[d] == 1) red_total *= in_s.d[d];
    float acc = mode == 0 ? 0.0f : -3.402823466e38f;
    for (int64_t r = 0; r < red_total; ++r) {
      // r enumerates the reduced coordinates in row-major order.
      int64_t rr = r, idx = 0, st = 1;
      for (int d = in_s.rank - 1; d >= 0; --d) {
        int64_t c;
        if (padded_out.d[d] == 1) { c = rr % in_s.d[d]; rr /= in_s.d[d]; }
        else c = coord[d];
        idx += c * st;
        st *= in_s.d[d];
      }
      float v = in[idx];
      if (mode == 0) acc = __fadd_rn(acc, v);
      else if (v > acc) acc = v;
    }
    out[o] = acc;
  }
}

// max_to_shape_backward (backend.rs:1383-1435): 0 + g where in == max.
__global__ void max_bw_kernel(const float* __restrict__ g, const float* __restrict__ ip,
                              const float* __restrict__ op, float* __restrict__ out, int64_t n,
                              ShapeInfo in_s, ShapeInfo padded_out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = i, idx = 0, st = 1;
    for (int d = in_s.rank - 1; d >= 0; --d) {
      int64_t c = rem % in_s.d[d];
      rem /= in_s.d[d];
      if (padded_out.d[d] != 1) idx += c * st;
      st *= padded_out.d[d];
    }
    out[i] = ip[i] == op[idx] ? __fadd_rn(0.0f, g[idx]) : 0.0f;
  }
}

__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out, int64_t n,
                                 ShapeInfo in_s, ShapeInfo out_s, int d0, int d1) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < n;
       o += (int64_t)gridDim.x * blockDim.x) {
    int64_t rem = o;
    int64_t c[ShapeInfo::MAXR];
    for (int d = out_s.rank - 1; d >= 0; --d) {
      c[d] = rem % out_s.d[d];
      rem /= out_s.d[d];
    }
    int64_t idx = 0, st = 1;
    for (int d = in_s.rank - 1; d >= 0; --d) {
      int od = d == d0 ? d1 : (d == d1 ? d0 : d);
      idx += c[od] * st;
      st *= in_s.d[d];
    }
    out[o] = in[idx];
  }
}

template <typename S, typename D>
__device__ __forceinline__ D conv(S v) { return static_cast<D>(v); }
template <> __device__ __forceinline__ float conv<__half, float>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ __half conv<float, __half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ float conv<__nv_bfloat16, float>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ __nv_bfloat16 conv<float, __nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename S, typename D>
__global__ void cast_kernel(const S* in, D* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = conv<S, D>(in[i]);
}

__global__ void nonfinite_kernel(const float* in, int64_t n, int* flag) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    if (!isfinite(in[i])) { atomicExch(flag, 1); return; }
}

// Waits on an mbarrier that nothing arrives at, with a bound of limit_ns: the
// wait must run out, record DEV_WAIT_TIMEOUT and return -- the same bounded
// wait the GEMM's roles use, exercised without any fault.
__global__ void selftest_wait_kernel(int* dev_err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, dev_err, 100, limit_ns);
  __syncthreads();
}

}  // namespace orca

using namespace orca;

// =============================================================== C ABI
extern "C" {

const char* orca_last_error(void) { return g_last_error.c_str(); }

const char* orca_status_string(orca_status s) {
  switch (s) {
    case ORCA_OK: return "ok";
    case ORCA_SHAPE_MISMATCH: return "shape mismatch";
    case ORCA_DEVICE_MISMATCH: return "device mismatch";
    case ORCA_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case ORCA_DTYPE_MISMATCH: return "dtype mismatch";
    case ORCA_INTERNAL: return "internal error";
    case ORCA_TIMEOUT: return "timeout";
    case ORCA_INVALID_ARGUMENT: return "invalid argument";
    case ORCA_NOT_IMPLEMENTED: return "not implemented";
    case ORCA_CUDA_ERROR: return "cuda error";
    case ORCA_COMM_ERROR: return "communicator error";
  }
  return "unknown status";
}

uint32_t orca_version(void) { return 0x000100u; }

orca_status orca_ctx_create(int device, orca_ctx** out) {
  if (!out) return fail(ORCA_INVALID_ARGUMENT, "null output pointer");
  int count = 0;
  ORCA_CUDA_TRY(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count)
    return fail(ORCA_INVALID_ARGUMENT, "device %d out of range (%d devices)", device, count);
  ORCA_CUDA_TRY(cudaSetDevice(device));
  cudaDeviceProp prop;
  ORCA_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(ORCA_UNSUPPORTED_DTYPE, "device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  orca_ctx* c = new orca_ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  ORCA_CUDA_TRY(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  // Collectives get the highest stream priority: when a GEMM CTA retires, a
  // waiting all-reduce takes the SM before more GEMM CTAs do (the GEMM's
  // dynamic tile scheduler lets the CTAs that start later take fewer tiles).
  int prio_low = 0, prio_high = 0;
  ORCA_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high));
  ORCA_CUDA_TRY(cudaStreamCreateWithPriority(&c->comm_stream, cudaStreamNonBlocking, prio_high));
  ORCA_CUDA_TRY(cudaEventCreateWithFlags(&c->sync_event, cudaEventDisableTiming));
  ORCA_CUDA_TRY(cudaMalloc(&c->dev_err, sizeof(int)));
  ORCA_CUDA_TRY(cudaMemset(c->dev_err, 0, sizeof(int)));
  ORCA_CUDA_TRY(cudaMalloc(&c->tile_ctr, sizeof(int)));
  ORCA_CUDA_TRY(cudaMemset(c->tile_ctr, 0, sizeof(int)));
  // Device address of the no-allocation CE entry point's fixed scratch,
  // looked up now with the device current (allocates nothing).  A failure
  // here only disables that entry point, which then reports it.
  if (ce_scratch_setup(device) != ORCA_OK) set_error("");
  // Keep freed stream-ordered allocations in the pool instead of returning
  // them to the driver at every synchronisation.
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t thr = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
  }
  *out = c;
  return ORCA_OK;
}

orca_status orca_ctx_destroy(orca_ctx* ctx) {
  if (!ctx) return ORCA_OK;
  ctx_release(ctx);   // freed once every buffer / runner / communicator is released too
  return ORCA_OK;
}

orca_status orca_ctx_sync(orca_ctx* ctx, double timeout_s) {
  ORCA_TRY(check_ctx(ctx));
  if (timeout_s <= 0) timeout_s = ctx->sync_timeout_s;
  std::lock_guard<std::mutex> lk(ctx->mu);
  ORCA_TRY(sync_stream_for(ctx, ctx->stream, timeout_s));
  return check_device_error(ctx);
}

orca_status orca_ctx_set_timeout(orca_ctx* ctx, double seconds) {
  if (!ctx || !(seconds > 0)) return fail(ORCA_INVALID_ARGUMENT, "timeout must be positive");
  ctx->sync_timeout_s = seconds;
  return ORCA_OK;
}

orca_status orca_ctx_selftest_wait_timeout(orca_ctx* ctx, double limit_s) {
  ORCA_TRY(check_ctx(ctx));
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!(limit_s > 0) || limit_s > 10.0)
    return fail(ORCA_INVALID_ARGUMENT, "limit must be in (0, 10] seconds");
  selftest_wait_kernel<<<1, 32, 0, ctx->stream>>>(ctx->dev_err, (uint64_t)(limit_s * 1e9));
  count_launch(ctx);
  ORCA_CUDA_TRY(cudaGetLastError());
  return check_device_error(ctx);   // ORCA_TIMEOUT when the wait ran out, as it must
}

orca_status orca_ctx_device(const orca_ctx* ctx, int* device) {
  if (!ctx || !device) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  *device = ctx->device;
  return ORCA_OK;
}

void* orca_ctx_stream(orca_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

orca_status orca_host_alloc(size_t bytes, void** out) {
  if (!out || !bytes) return fail(ORCA_INVALID_ARGUMENT, "host_alloc: null output or zero size");
  *out = nullptr;
  const cudaError_t e = cudaHostAlloc(out, bytes, cudaHostAllocPortable);
  if (e != cudaSuccess) {
    *out = nullptr;
    return fail(ORCA_CUDA_ERROR, "page-locked allocation of %zu bytes failed: %s", bytes,
                cudaGetErrorString(e));
  }
  return ORCA_OK;
}

orca_status orca_host_free(void* ptr) {
  if (!ptr) return ORCA_OK;
  const cudaError_t e = cudaFreeHost(ptr);
  if (e != cudaSuccess) return fail(ORCA_CUDA_ERROR, "host_free: %s", cudaGetErrorString(e));
  return ORCA_OK;
}

uint64_t orca_ctx_launch_count(const orca_ctx* ctx) { return ctx ? ctx->launches.load() : 0; }

orca_status orca_buf_retain(orca_buf* buf) {
  if (!buf) return fail(ORCA_INVALID_ARGUMENT, "null buffer");
  buf->refs++;
  return ORCA_OK;
}

orca_status orca_buf_release(orca_buf* buf) {
  if (!buf) return ORCA_OK;
  if (--buf->refs == 0) {
    orca_ctx* ctx = buf->ctx;
    if (buf->ptr) {
      cudaSetDevice(ctx->device);
      cudaFreeAsync(buf->ptr, ctx->stream);
    }
    delete buf;
    ctx_release(ctx);
  }
  return ORCA_OK;
}

size_t orca_buf_len(const orca_buf* buf) { return buf ? buf->n : 0; }
orca_dtype orca_buf_dtype(const orca_buf* buf) { return buf ? buf->dtype : ORCA_F32; }
void* orca_buf_device_ptr(const orca_buf* buf) { return buf ? buf->ptr : nullptr; }

#define LOCK(ctx) std::lock_guard<std::mutex> _lk((ctx)->mu)

orca_status orca_zeros(orca_ctx* ctx, const int64_t* dims, int rank, orca_dtype dtype,
                       orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  ORCA_TRY(new_buf(ctx, (size_t)n, dtype, out));
  if (n) ORCA_CUDA_TRY(cudaMemsetAsync((*out)->ptr, 0, (size_t)n * dtype_size(dtype), ctx->stream));
  return ORCA_OK;
}

orca_status orca_from_f32_slice(orca_ctx* ctx, const int64_t* dims, int rank, const float* data,
                                orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  if (n && !data) return fail(ORCA_INVALID_ARGUMENT, "null host data");
  ORCA_TRY(new_buf(ctx, (size_t)n, ORCA_F32, out));
  if (n) {
    ORCA_CUDA_TRY(cudaMemcpyAsync((*out)->ptr, data, (size_t)n * 4, cudaMemcpyHostToDevice,
                                  ctx->stream));
    ORCA_TRY(sync_stream(ctx));   // host memory may be freed on return
  }
  return ORCA_OK;
}

orca_status orca_to_f32_vec(orca_ctx* ctx, const orca_buf* buf, float* dst, size_t n_elems) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  if (!buf || (!dst && n_elems)) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (buf->dtype != ORCA_F32) return fail(ORCA_DTYPE_MISMATCH, "to_f32_vec on a non-F32 buffer");
  if (n_elems != buf->n)
    return fail(ORCA_SHAPE_MISMATCH, "to_f32_vec: buffer has %zu elements, dst %zu", buf->n, n_elems);
  ORCA_TRY(copy_to_host(ctx, dst, buf->ptr, n_elems * 4));
  return check_device_error(ctx);
}

orca_status orca_from_bytes(orca_ctx* ctx, const int64_t* dims, int rank, const void* bytes,
                            size_t n_bytes, orca_dtype dtype, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  if ((size_t)n * dtype_size(dtype) != n_bytes)
    return fail(ORCA_SHAPE_MISMATCH, "from_bytes: %zu bytes for %lld elements", n_bytes,
                (long long)n);
  ORCA_TRY(new_buf(ctx, (size_t)n, dtype, out));
  if (n_bytes) {
    ORCA_CUDA_TRY(cudaMemcpyAsync((*out)->ptr, bytes, n_bytes, cudaMemcpyHostToDevice, ctx->stream));
    ORCA_TRY(sync_stream(ctx));
  }
  return ORCA_OK;
}

orca_status orca_to_bytes(orca_ctx* ctx, const orca_buf* buf, void* dst, size_t n_bytes) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  if (!buf) return fail(ORCA_INVALID_ARGUMENT, "null buffer");
  if (n_bytes != buf->n * dtype_size(buf->dtype))
    return fail(ORCA_SHAPE_MISMATCH, "to_bytes: size mismatch");
  ORCA_TRY(copy_to_host(ctx, dst, buf->ptr, n_bytes));
  return check_device_error(ctx);
}

static orca_status binary(orca_ctx* ctx, int op, const orca_buf* a, const orca_buf* b,
                          const int64_t* dims, int rank, orca_dtype dtype, orca_buf** out,
                          const char* name) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, name));
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  ORCA_TRY(need(a, (size_t)n, name));
  ORCA_TRY(need(b, (size_t)n, name));
  if (a->ctx != ctx || b->ctx != ctx)
    return fail(ORCA_DEVICE_MISMATCH, "%s: operands belong to another context", name);
  ORCA_TRY(new_buf(ctx, (size_t)n, ORCA_F32, out));
  if (n) {
    binary_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(op, (const float*)a->ptr,
                                                             (const float*)b->ptr,
                                                             (float*)(*out)->ptr, n);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

static orca_status unary(orca_ctx* ctx, int op, const orca_buf* a, float s_, const int64_t* dims,
                         int rank, orca_dtype dtype, orca_buf** out, const char* name) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, name));
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  ORCA_TRY(need(a, (size_t)n, name));
  ORCA_TRY(new_buf(ctx, (size_t)n, ORCA_F32, out));
  if (n) {
    unary_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(op, (const float*)a->ptr,
                                                            (float*)(*out)->ptr, n, s_);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

orca_status orca_add(orca_ctx* c, const orca_buf* l, const orca_buf* r, const int64_t* d, int k,
                     orca_dtype t, orca_buf** o) { return binary(c, B_ADD, l, r, d, k, t, o, "add"); }
orca_status orca_sub(orca_ctx* c, const orca_buf* l, const orca_buf* r, const int64_t* d, int k,
                     orca_dtype t, orca_buf** o) { return binary(c, B_SUB, l, r, d, k, t, o, "sub"); }
orca_status orca_mul(orca_ctx* c, const orca_buf* l, const orca_buf* r, const int64_t* d, int k,
                     orca_dtype t, orca_buf** o) { return binary(c, B_MUL, l, r, d, k, t, o, "mul"); }
orca_status orca_div(orca_ctx* c, const orca_buf* l, const orca_buf* r, const int64_t* d, int k,
                     orca_dtype t, orca_buf** o) { return binary(c, B_DIV, l, r, d, k, t, o, "div"); }
orca_status orca_relu_backward(orca_ctx* c, const orca_buf* g, const orca_buf* x, const int64_t* d,
                               int k, orca_dtype t, orca_buf** o) {
  return binary(c, B_RELU_BW, g, x, d, k, t, o, "relu_backward");
}
orca_status orca_sigmoid_backward(orca_ctx* c, const orca_buf* g, const orca_buf* y,
                                  const int64_t* d, int k, orca_dtype t, orca_buf** o) {
  return binary(c, B_SIGMOID_BW, g, y, d, k, t, o, "sigmoid_backward");
}
orca_status orca_exp_backward(orca_ctx* c, const orca_buf* g, const orca_buf* y, const int64_t* d,
                              int k, orca_dtype t, orca_buf** o) {
  return binary(c, B_EXP_BW, g, y, d, k, t, o, "exp_backward");
}
orca_status orca_log_backward(orca_ctx* c, const orca_buf* g, const orca_buf* x, const int64_t* d,
                              int k, orca_dtype t, orca_buf** o) {
  return binary(c, B_LOG_BW, g, x, d, k, t, o, "log_backward");
}
orca_status orca_sqrt_backward(orca_ctx* c, const orca_buf* g, const orca_buf* y, const int64_t* d,
                               int k, orca_dtype t, orca_buf** o) {
  return binary(c, B_SQRT_BW, g, y, d, k, t, o, "sqrt_backward");
}
orca_status orca_div_backward_lhs(orca_ctx* c, const orca_buf* g, const orca_buf* r,
                                  const int64_t* d, int k, orca_dtype t, orca_buf** o) {
  return binary(c, B_DIV_BW_LHS, g, r, d, k, t, o, "div_backward_lhs");
}
orca_status orca_accumulate_grad(orca_ctx* c, const orca_buf* l, const orca_buf* r, orca_buf** o) {
  if (!l || !r) return fail(ORCA_INVALID_ARGUMENT, "accumulate_grad: null buffer");
  if (l->n != r->n) return fail(ORCA_SHAPE_MISMATCH, "accumulate_grad: %zu vs %zu", l->n, r->n);
  int64_t d = (int64_t)l->n;
  return binary(c, B_ADD, l, r, &d, 1, l->dtype, o, "accumulate_grad");
}

orca_status orca_div_backward_rhs(orca_ctx* ctx, const orca_buf* g, const orca_buf* l,
                                  const orca_buf* r, const int64_t* dims, int rank,
                                  orca_dtype dtype, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, "div_backward_rhs"));
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  ORCA_TRY(need(g, (size_t)n, "div_backward_rhs"));
  ORCA_TRY(need(l, (size_t)n, "div_backward_rhs"));
  ORCA_TRY(need(r, (size_t)n, "div_backward_rhs"));
  ORCA_TRY(new_buf(ctx, (size_t)n, ORCA_F32, out));
  if (n) {
    div_bw_rhs_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(
        (const float*)g->ptr, (const float*)l->ptr, (const float*)r->ptr, (float*)(*out)->ptr, n);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

orca_status orca_relu(orca_ctx* c, const orca_buf* x, const int64_t* d, int k, orca_dtype t,
                      orca_buf** o) { return unary(c, U_RELU, x, 0.f, d, k, t, o, "relu"); }
orca_status orca_sigmoid(orca_ctx* c, const orca_buf* x, const int64_t* d, int k, orca_dtype t,
                         orca_buf** o) { return unary(c, U_SIGMOID, x, 0.f, d, k, t, o, "sigmoid"); }
orca_status orca_exp(orca_ctx* c, const orca_buf* x, const int64_t* d, int k, orca_dtype t,
                     orca_buf** o) { return unary(c, U_EXP, x, 0.f, d, k, t, o, "exp"); }
orca_status orca_log(orca_ctx* c, const orca_buf* x, const int64_t* d, int k, orca_dtype t,
                     orca_buf** o) { return unary(c, U_LOG, x, 0.f, d, k, t, o, "log"); }
orca_status orca_sqrt(orca_ctx* c, const orca_buf* x, const int64_t* d, int k, orca_dtype t,
                      orca_buf** o) { return unary(c, U_SQRT, x, 0.f, d, k, t, o, "sqrt"); }
orca_status orca_mul_scalar(orca_ctx* c, const orca_buf* x, float s, const int64_t* d, int k,
                            orca_dtype t, orca_buf** o) {
  return unary(c, U_MULS, x, s, d, k, t, o, "mul_scalar");
}

orca_status orca_expand(orca_ctx* ctx, const orca_buf* x, const int64_t* in_dims, int in_rank,
                        const int64_t* out_dims, int out_rank, orca_dtype dtype, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, "expand"));
  ShapeInfo si, so;
  int64_t ni = 0, no = 0;
  ORCA_TRY(to_shape(in_dims, in_rank, si, &ni));
  ORCA_TRY(to_shape(out_dims, out_rank, so, &no));
  ORCA_TRY(need(x, (size_t)ni, "expand"));
  if (in_rank > out_rank) return fail(ORCA_SHAPE_MISMATCH, "expand: rank %d -> %d", in_rank, out_rank);
  ShapeInfo pi = pad_left(si, out_rank);
  for (int d = 0; d < out_rank; ++d)
    if (pi.d[d] != 1 && pi.d[d] != so.d[d])
      return fail(ORCA_SHAPE_MISMATCH, "expand: dim %d is %lld, target %lld", d,
                  (long long)pi.d[d], (long long)so.d[d]);
  ORCA_TRY(new_buf(ctx, (size_t)no, ORCA_F32, out));
  if (no) {
    expand_kernel<<<grid_for(ctx, no), 256, 0, ctx->stream>>>((const float*)x->ptr,
                                                              (float*)(*out)->ptr, no, so, pi);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

static orca_status reduce_to(orca_ctx* ctx, int mode, const orca_buf* x, const int64_t* in_dims,
                             int in_rank, const int64_t* out_dims, int out_rank, orca_dtype dtype,
                             orca_buf** out, const char* name) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, name));
  ShapeInfo si, so;
  int64_t ni = 0, no = 0;
  ORCA_TRY(to_shape(in_dims, in_rank, si, &ni));
  ORCA_TRY(to_shape(out_dims, out_rank, so, &no));
  ORCA_TRY(need(x, (size_t)ni, name));
  if (out_rank > in_rank) return fail(ORCA_SHAPE_MISMATCH, "%s: rank %d -> %d", name, in_rank, out_rank);
  ShapeInfo po = pad_left(so, in_rank);
  for (int d = 0; d < in_rank; ++d)
    if (po.d[d] != 1 && po.d[d] != si.d[d])
      return fail(ORCA_SHAPE_MISMATCH, "%s: dim %d is %lld, input %lld", name, d,
                  (long long)po.d[d], (long long)si.d[d]);
  ORCA_TRY(new_buf(ctx, (size_t)no, ORCA_F32, out));
  if (no) {
    reduce_to_shape_kernel<<<grid_for(ctx, no), 256, 0, ctx->stream>>>(
        mode, (const float*)x->ptr, (float*)(*out)->ptr, no, si, po);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

orca_status orca_sum_to_shape(orca_ctx* c, const orca_buf* x, const int64_t* id, int ir,
                              const int64_t* od, int orank, orca_dtype t, orca_buf** o) {
  return reduce_to(c, 0, x, id, ir, od, orank, t, o, "sum_to_shape");
}
orca_status orca_max_to_shape(orca_ctx* c, const orca_buf* x, const int64_t* id, int ir,
                              const int64_t* od, int orank, orca_dtype t, orca_buf** o) {
  return reduce_to(c, 1, x, id, ir, od, orank, t, o, "max_to_shape");
}

orca_status orca_max_to_shape_backward(orca_ctx* ctx, const orca_buf* g, const orca_buf* ip,
                                       const orca_buf* op, const int64_t* in_dims, int in_rank,
                                       const int64_t* out_dims, int out_rank, orca_dtype dtype,
                                       orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, "max_to_shape_backward"));
  ShapeInfo si, so;
  int64_t ni = 0, no = 0;
  ORCA_TRY(to_shape(in_dims, in_rank, si, &ni));
  ORCA_TRY(to_shape(out_dims, out_rank, so, &no));
  ORCA_TRY(need(g, (size_t)no, "max_to_shape_backward"));
  ORCA_TRY(need(op, (size_t)no, "max_to_shape_backward"));
  ORCA_TRY(need(ip, (size_t)ni, "max_to_shape_backward"));
  if (out_rank > in_rank) return fail(ORCA_SHAPE_MISMATCH, "max_to_shape_backward: rank");
  ShapeInfo po = pad_left(so, in_rank);
  ORCA_TRY(new_buf(ctx, (size_t)ni, ORCA_F32, out));
  if (ni) {
    max_bw_kernel<<<grid_for(ctx, ni), 256, 0, ctx->stream>>>(
        (const float*)g->ptr, (const float*)ip->ptr, (const float*)op->ptr, (float*)(*out)->ptr,
        ni, si, po);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

orca_status orca_reshape(orca_ctx* ctx, const orca_buf* x, const int64_t* in_dims, int in_rank,
                         const int64_t* out_dims, int out_rank, orca_dtype dtype, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ShapeInfo si, so;
  int64_t ni = 0, no = 0;
  ORCA_TRY(to_shape(in_dims, in_rank, si, &ni));
  ORCA_TRY(to_shape(out_dims, out_rank, so, &no));
  if (ni != no)   // backend.rs:539-545
    return fail(ORCA_SHAPE_MISMATCH, "reshape: %lld elements vs %lld", (long long)ni, (long long)no);
  ORCA_TRY(need(x, (size_t)ni, "reshape"));
  if (!out) return fail(ORCA_INVALID_ARGUMENT, "null output");
  (void)dtype;
  // Contiguous storage: the result shares the buffer, as the CPU backend's
  // storage.clone() does (backend.rs:546).
  orca_buf* b = const_cast<orca_buf*>(x);
  b->refs++;
  *out = b;
  return ORCA_OK;
}

orca_status orca_transpose(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                           int dim0, int dim1, orca_dtype dtype, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, "transpose"));
  ShapeInfo si;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, si, &n));
  if (dim0 < 0 || dim1 < 0 || dim0 >= rank || dim1 >= rank)   // backend.rs:238-242
    return fail(ORCA_INTERNAL, "Invalid transpose dimensions");
  ORCA_TRY(need(x, (size_t)n, "transpose"));
  ShapeInfo so = si;
  std::swap(so.d[dim0], so.d[dim1]);
  ORCA_TRY(new_buf(ctx, (size_t)n, ORCA_F32, out));
  if (n) {
    transpose_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>((const float*)x->ptr,
                                                                (float*)(*out)->ptr, n, si, so,
                                                                dim0, dim1);
    count_launch(ctx);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

// matmul (backend.rs:130-221): batched, same rank, row-major, FP32.
orca_status orca_matmul(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                        const int64_t* ld, int lr, const int64_t* rd, int rr, orca_dtype dtype,
                        orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, "matmul"));
  ShapeInfo sl, sr;
  int64_t nl = 0, nr = 0;
  ORCA_TRY(to_shape(ld, lr, sl, &nl));
  ORCA_TRY(to_shape(rd, rr, sr, &nr));
  if (lr < 2 || rr < 2)
    return fail(ORCA_SHAPE_MISMATCH, "matmul: expected >= 2D tensors, got %dD and %dD", lr, rr);
  if (lr != rr) return fail(ORCA_SHAPE_MISMATCH, "matmul: same rank required (%d vs %d)", lr, rr);
  int64_t batch = 1;
  for (int i = 0; i < lr - 2; ++i) {
    if (sl.d[i] != sr.d[i]) return fail(ORCA_SHAPE_MISMATCH, "matmul: batch dims differ");
    batch *= sl.d[i];
  }
  const int64_t M = sl.d[lr - 2], K = sl.d[lr - 1], N = sr.d[rr - 1];
  if (sr.d[rr - 2] != K)
    return fail(ORCA_SHAPE_MISMATCH, "matmul: inner dimensions %lld != %lld", (long long)K,
                (long long)sr.d[rr - 2]);
  ORCA_TRY(need(lhs, (size_t)nl, "matmul"));
  ORCA_TRY(need(rhs, (size_t)nr, "matmul"));
  ORCA_TRY(new_buf(ctx, (size_t)(batch * M * N), ORCA_F32, out));
  if (batch * M * N == 0) return ORCA_OK;
  const float* A = (const float*)lhs->ptr;
  const float* B = (const float*)rhs->ptr;
  float* C = (float*)(*out)->ptr;
  // The tensor-core path takes (hi, lo) plane pairs: split both operands once.
  Epilogue ep;
  ep.mode = EPI_STORE;
  ep.ldc = N;
  float* scratch = nullptr;
  // Same shape rule as the GEMM dispatcher; the 16-byte TMA stride rule needs
  // K and N to be multiples of 4 f32 elements.
  const bool use_tc = M >= 64 && N >= 64 && K >= 16 && (K & 3) == 0 && (N & 3) == 0;
  if (use_tc) {
    const size_t elems = 2 * (size_t)(batch * M * K) + 2 * (size_t)(batch * K * N);
    ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), elems * 4, ctx->stream));
    float* a_hi = scratch;
    float* a_lo = a_hi + batch * M * K;
    float* b_hi = a_lo + batch * M * K;
    float* b_lo = b_hi + batch * K * N;
    ORCA_TRY(split_planes(ctx, A, a_hi, a_lo, batch * M * K));
    ORCA_TRY(split_planes(ctx, B, b_hi, b_lo, batch * K * N));
    for (int64_t b = 0; b < batch; ++b) {
      // Each batch's planes: hi block then lo block of the same per-batch size
      // would be needed for the 3-D map; use per-batch views with the plane
      // stride of the whole split buffer.
      Operand oa, ob;
      oa.hi = a_hi + b * M * K; oa.lo = a_lo + b * M * K; oa.ld = K; oa.mn_major = false;
      ob.hi = b_hi + b * K * N; ob.lo = b_lo + b * K * N; ob.ld = N; ob.mn_major = true;
      Epilogue e2 = ep;
      e2.out = C + b * M * N;
      orca_status st = gemm(ctx, M, N, K, oa, ob, e2, GEMM_AUTO);
      if (st != ORCA_OK) { cudaFreeAsync(scratch, ctx->stream); return st; }
    }
    cudaFreeAsync(scratch, ctx->stream);
    return ORCA_OK;
  }
  for (int64_t b = 0; b < batch; ++b) {
    Operand oa, ob;
    oa.hi = A + b * M * K; oa.ld = K;
    ob.hi = B + b * K * N; ob.ld = N; ob.mn_major = true;
    Epilogue e2 = ep;
    e2.out = C + b * M * N;
    ORCA_TRY(gemm(ctx, M, N, K, oa, ob, e2, GEMM_SIMT));
  }
  return ORCA_OK;
}

orca_status orca_gemm_ex(orca_ctx* ctx, int64_t M, int64_t N, int64_t K, const orca_buf* a,
                         int a_mn, const orca_buf* b, int b_mn, int path, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  if (!a || !b || !out) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (M < 0 || N < 0 || K < 0 || path < 0 || path > 4)
    return fail(ORCA_INVALID_ARGUMENT, "gemm_ex: bad arguments");
  ORCA_TRY(need(a, (size_t)(M * K), "gemm_ex"));
  ORCA_TRY(need(b, (size_t)(K * N), "gemm_ex"));
  ORCA_TRY(need_f32(a->dtype, "gemm_ex"));
  ORCA_TRY(need_f32(b->dtype, "gemm_ex"));
  ORCA_TRY(new_buf(ctx, (size_t)(M * N), ORCA_F32, out));
  if (M * N == 0) return ORCA_OK;
  float* scratch = nullptr;
  const size_t elems = 2 * (size_t)(M * K) + 2 * (size_t)(K * N) + 8;
  ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), elems * 4, ctx->stream));
  float* ah = scratch;
  float* bh = scratch + ((2 * M * K + 3) & ~int64_t(3));
  ORCA_TRY(split_planes(ctx, (const float*)a->ptr, ah, ah + M * K, M * K));
  ORCA_TRY(split_planes(ctx, (const float*)b->ptr, bh, bh + K * N, K * N));
  Operand oa, ob;
  oa.hi = ah; oa.lo = ah + M * K; oa.ld = a_mn ? M : K; oa.mn_major = a_mn != 0;
  ob.hi = bh; ob.lo = bh + K * N; ob.ld = b_mn ? N : K; ob.mn_major = b_mn != 0;
  Epilogue ep;
  ep.mode = EPI_STORE;
  ep.out = (float*)(*out)->ptr;
  ep.ldc = N;
  if (gemm_path_is_tc(path) && !gemm_tc_eligible(M, N, K, oa, ob)) {
    cudaFreeAsync(scratch, ctx->stream);
    orca_buf_release(*out);
    *out = nullptr;
    return fail(ORCA_INVALID_ARGUMENT, "gemm_ex: shape/operands not eligible for the tcgen05 path");
  }
  orca_status st = gemm(ctx, M, N, K, oa, ob, ep, path);
  cudaFreeAsync(scratch, ctx->stream);
  if (st != ORCA_OK) {
    orca_buf_release(*out);
    *out = nullptr;
  }
  return st;
}

orca_status orca_cast(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                      orca_dtype cur, orca_dtype tgt, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ShapeInfo s;
  int64_t n = 0;
  ORCA_TRY(to_shape(dims, rank, s, &n));
  ORCA_TRY(need(x, (size_t)n, "cast"));
  if (x->dtype != cur) return fail(ORCA_DTYPE_MISMATCH, "cast: buffer dtype %d, stated %d",
                                   (int)x->dtype, (int)cur);
  ORCA_TRY(new_buf(ctx, (size_t)n, tgt, out));
  if (!n) return ORCA_OK;
  const int g = grid_for(ctx, n);
  if (cur == tgt) {
    ORCA_CUDA_TRY(cudaMemcpyAsync((*out)->ptr, x->ptr, (size_t)n * dtype_size(cur),
                                  cudaMemcpyDeviceToDevice, ctx->stream));
    return ORCA_OK;
  }
  const void* i = x->ptr;
  void* o = (*out)->ptr;
#define CAST(S, D) cast_kernel<S, D><<<g, 256, 0, ctx->stream>>>((const S*)i, (D*)o, n)
  if (cur == ORCA_F32 && tgt == ORCA_F64) CAST(float, double);
  else if (cur == ORCA_F64 && tgt == ORCA_F32) CAST(double, float);
  else if (cur == ORCA_F32 && tgt == ORCA_F16) CAST(float, __half);
  else if (cur == ORCA_F16 && tgt == ORCA_F32) CAST(__half, float);
  else if (cur == ORCA_F32 && tgt == ORCA_BF16) CAST(float, __nv_bfloat16);
  else if (cur == ORCA_BF16 && tgt == ORCA_F32) CAST(__nv_bfloat16, float);
  else if (cur == ORCA_F32 && tgt == ORCA_I32) CAST(float, int32_t);
  else if (cur == ORCA_I32 && tgt == ORCA_F32) CAST(int32_t, float);
  else if (cur == ORCA_F32 && tgt == ORCA_I64) CAST(float, int64_t);
  else if (cur == ORCA_I64 && tgt == ORCA_F32) CAST(int64_t, float);
  else {
    orca_buf_release(*out);
    *out = nullptr;
    return fail(ORCA_UNSUPPORTED_DTYPE, "cast %d -> %d is outside the F32 path", (int)cur, (int)tgt);
  }
#undef CAST
  count_launch(ctx);
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

orca_status orca_has_nan_or_inf(orca_ctx* ctx, const orca_buf* x, orca_dtype dtype, int* result) {
  ORCA_TRY(check_ctx(ctx));
  LOCK(ctx);
  ORCA_TRY(need_f32(dtype, "has_nan_or_inf"));
  if (!x || !result) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  int* flag = nullptr;
  ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&flag), sizeof(int), ctx->stream));
  ORCA_CUDA_TRY(cudaMemsetAsync(flag, 0, sizeof(int), ctx->stream));
  if (x->n) {
    nonfinite_kernel<<<grid_for(ctx, (int64_t)x->n), 256, 0, ctx->stream>>>((const float*)x->ptr,
                                                                            (int64_t)x->n, flag);
    count_launch(ctx);
  }
  int h = 0;
  const orca_status st = copy_to_host(ctx, &h, flag, sizeof(int));
  cudaFreeAsync(flag, ctx->stream);
  ORCA_TRY(st);
  *result = h;
  return ORCA_OK;
}

orca_status orca_conv2d(orca_ctx*, const orca_buf*, const orca_buf*, const orca_buf*,
                        const int64_t*, int, const int64_t*, int, int64_t, int64_t, int64_t,
                        int64_t, orca_dtype, orca_buf**) {
  return fail(ORCA_NOT_IMPLEMENTED, "conv2d is outside the MLP path of the CUDA backend");
}
orca_status orca_gather(orca_ctx*, const orca_buf*, int64_t, const orca_buf*, const int64_t*, int,
                        const int64_t*, int, orca_dtype, orca_buf**) {
  return fail(ORCA_NOT_IMPLEMENTED, "gather is outside the MLP path of the CUDA backend");
}
orca_status orca_scatter(orca_ctx*, const orca_buf*, int64_t, const orca_buf*, const orca_buf*,
                         const int64_t*, int, const int64_t*, int, orca_dtype, orca_buf**) {
  return fail(ORCA_NOT_IMPLEMENTED, "scatter is outside the MLP path of the CUDA backend");
}

}  // extern "C"
