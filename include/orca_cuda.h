/*
 * orca_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for Orca's FP32
 * MLP data-parallel training path.
 *
 * This is the drop-in boundary.  In the reference (cowoksoftspoken/orcaml) the
 * plugin interface is the Rust trait `Backend` (orca-tensor/src/backend.rs:
 * 19-315), implemented by `CpuBackend` (orca-backend-cpu/src/backend.rs) and
 * `GpuBackend` (orca-backend-gpu, wgpu), wrapped by `Autodiff<B>` and exposed
 * to Python by the PyO3 module `orca.orca_python` (orca-python/src/lib.rs).
 * A Rust `orca-backend-cuda` crate implements `Backend` by calling the
 * `orca_*` functions below one-to-one (each storage an Arc'd handle whose
 * Drop calls orca_buf_release); the Python host layer of this repository
 * (orcaml_b200) binds the same symbols through ctypes.
 *
 * Conventions
 *  - Every function returns an orca_status; ORCA_OK is 0.  The message of
 *    the last failure on the calling thread is orca_last_error().  The
 *    statuses map one-to-one onto the reference's OrcaError variants
 *    (orca-core/src/error.rs:5-31); PyO3 raises ValueError for all of them
 *    except backend-construction failures (RuntimeError, lib.rs:23-33).
 *  - Shapes are (const int64_t* dims, int rank), row-major, contiguous, as
 *    `Shape` (orca-core/src/shape.rs).  dtype values follow orca-core's
 *    `DType` order (orca-core/src/dtype.rs:5-22).
 *  - Ops are functional like the trait: each allocates and returns a NEW
 *    buffer through an out-parameter (refcount 1); inputs are never modified.
 *  - All kernels of a context run on its compute stream in call order; a call
 *    returns once its work is enqueued, except the *_to_host/_to_f32_vec
 *    reads, which are synchronous like `to_f32_vec` (trait line 35).
 *  - Device-side waits inside the library's kernels are bounded; a wait that
 *    runs out sets a device error word and the next synchronising call
 *    returns ORCA_TIMEOUT instead of hanging.
 *  - One context per device; calls on one context are serialised by an
 *    internal mutex, so a context may be shared across host threads.
 */
#ifndef ORCA_CUDA_H
#define ORCA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  ORCA_OK = 0,
  ORCA_SHAPE_MISMATCH = 1,      /* OrcaError::ShapeMismatch (error.rs:7-12) */
  ORCA_DEVICE_MISMATCH = 2,     /* OrcaError::DeviceMismatch (error.rs:14) */
  ORCA_UNSUPPORTED_DTYPE = 3,   /* OrcaError::UnsupportedDType (error.rs:17-21) */
  ORCA_DTYPE_MISMATCH = 4,      /* OrcaError::DTypeMismatch (error.rs:23-28) */
  ORCA_INTERNAL = 5,            /* OrcaError::InternalError (error.rs:30) */
  ORCA_TIMEOUT = 6,             /* a bounded device or host wait ran out */
  ORCA_INVALID_ARGUMENT = 7,    /* null pointer, bad rank, bad hyper-parameter */
  ORCA_NOT_IMPLEMENTED = 8,     /* trait method outside the MLP path (conv, gather, ...) */
  ORCA_CUDA_ERROR = 9,          /* CUDA runtime/driver failure, message in orca_last_error */
  ORCA_COMM_ERROR = 10          /* NCCL failure or abort */
} orca_status;

typedef enum {                   /* orca-core/src/dtype.rs:5-22 */
  ORCA_F32 = 0, ORCA_F64 = 1, ORCA_F16 = 2, ORCA_BF16 = 3,
  ORCA_I32 = 4, ORCA_I64 = 5, ORCA_U8 = 6, ORCA_BOOL = 7
} orca_dtype;

typedef struct orca_ctx orca_ctx;
typedef struct orca_buf orca_buf;
typedef struct orca_mlp orca_mlp;
typedef struct orca_comm orca_comm;

/* ---- library / errors ---------------------------------------------------- */
const char* orca_last_error(void);
const char* orca_status_string(orca_status s);
/* Packed version 0xMMmmpp of this library. */
uint32_t orca_version(void);

/* ---- context: one per device (GpuBackend::new, orca-backend-gpu/src/backend.rs:53-80) */
orca_status orca_ctx_create(int device, orca_ctx** out);
orca_status orca_ctx_destroy(orca_ctx* ctx);
/* Wait for all enqueued work; ORCA_TIMEOUT after timeout_s seconds (<=0: 600 s). */
orca_status orca_ctx_sync(orca_ctx* ctx, double timeout_s);
/* Backend::device (trait :24). */
orca_status orca_ctx_device(const orca_ctx* ctx, int* device);
/* Deadline in seconds for every call that waits on the device (default 600).
 * A wait past it returns ORCA_TIMEOUT instead of blocking; a trainer with a
 * communicator attached then aborts the communicator (a peer has gone). */
orca_status orca_ctx_set_timeout(orca_ctx* ctx, double seconds);
/* Runs a one-warp kernel whose mbarrier wait nothing completes, bounded by
 * limit_s (0 < limit_s <= 10): the wait runs out, the kernel records the
 * timeout and returns, and this call returns ORCA_TIMEOUT with the context
 * still usable.  Exercises the bounded-wait path of the device code without
 * any fault. */
orca_status orca_ctx_selftest_wait_timeout(orca_ctx* ctx, double limit_s);
/* The compute stream (a cudaStream_t), for callers that interoperate. */
void* orca_ctx_stream(orca_ctx* ctx);
/* Number of this library's kernels launched on ctx so far. */
uint64_t orca_ctx_launch_count(const orca_ctx* ctx);

/* ---- buffers: Storage (trait :7-15) = refcounted device allocation -------- */
orca_status orca_buf_retain(orca_buf* buf);
orca_status orca_buf_release(orca_buf* buf);
size_t orca_buf_len(const orca_buf* buf);           /* Storage::len, elements */
orca_dtype orca_buf_dtype(const orca_buf* buf);
void* orca_buf_device_ptr(const orca_buf* buf);

/* ---- Backend trait methods (orca-tensor/src/backend.rs) -------------------- */
orca_status orca_zeros(orca_ctx* ctx, const int64_t* dims, int rank, orca_dtype dtype,
                       orca_buf** out);                                       /* :27 */
orca_status orca_from_f32_slice(orca_ctx* ctx, const int64_t* dims, int rank,
                                const float* data, orca_buf** out);           /* :31 */
orca_status orca_to_f32_vec(orca_ctx* ctx, const orca_buf* buf, float* dst,
                            size_t n_elems);                                  /* :34 */
orca_status orca_from_bytes(orca_ctx* ctx, const int64_t* dims, int rank,
                            const void* bytes, size_t n_bytes, orca_dtype dtype,
                            orca_buf** out);                                  /* :296 */
orca_status orca_to_bytes(orca_ctx* ctx, const orca_buf* buf, void* dst,
                          size_t n_bytes);                                    /* :297 */
orca_status orca_matmul(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                        const int64_t* lhs_dims, int lhs_rank,
                        const int64_t* rhs_dims, int rhs_rank, orca_dtype dtype,
                        orca_buf** out);                                      /* :38-45 */
orca_status orca_transpose(orca_ctx* ctx, const orca_buf* x, const int64_t* dims,
                           int rank, int dim0, int dim1, orca_dtype dtype,
                           orca_buf** out);                                   /* :48-55 */
orca_status orca_add(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                     const int64_t* dims, int rank, orca_dtype dtype, orca_buf** out);  /* :57-63 */
orca_status orca_sub(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                     const int64_t* dims, int rank, orca_dtype dtype, orca_buf** out);  /* :64-70 */
orca_status orca_mul_scalar(orca_ctx* ctx, const orca_buf* x, float scalar,
                            const int64_t* dims, int rank, orca_dtype dtype,
                            orca_buf** out);                                  /* :71-77 */
orca_status orca_mul(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                     const int64_t* dims, int rank, orca_dtype dtype, orca_buf** out);  /* :80-86 */
orca_status orca_relu(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                      orca_dtype dtype, orca_buf** out);                      /* :87 */
orca_status orca_sigmoid(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                         orca_dtype dtype, orca_buf** out);                   /* :88-93 */
orca_status orca_relu_backward(orca_ctx* ctx, const orca_buf* grad_out,
                               const orca_buf* in_primal, const int64_t* dims, int rank,
                               orca_dtype dtype, orca_buf** out);             /* :96-102 */
orca_status orca_sigmoid_backward(orca_ctx* ctx, const orca_buf* grad_out,
                                  const orca_buf* out_primal, const int64_t* dims,
                                  int rank, orca_dtype dtype, orca_buf** out);/* :103-109 */
orca_status orca_expand(orca_ctx* ctx, const orca_buf* x, const int64_t* in_dims,
                        int in_rank, const int64_t* out_dims, int out_rank,
                        orca_dtype dtype, orca_buf** out);                    /* :112-118 */
orca_status orca_sum_to_shape(orca_ctx* ctx, const orca_buf* x, const int64_t* in_dims,
                              int in_rank, const int64_t* out_dims, int out_rank,
                              orca_dtype dtype, orca_buf** out);              /* :119-125 */
orca_status orca_reshape(orca_ctx* ctx, const orca_buf* x, const int64_t* in_dims,
                         int in_rank, const int64_t* out_dims, int out_rank,
                         orca_dtype dtype, orca_buf** out);                   /* :128-134 */
orca_status orca_exp(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                     orca_dtype dtype, orca_buf** out);                       /* :135 */
orca_status orca_log(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                     orca_dtype dtype, orca_buf** out);                       /* :136 */
orca_status orca_exp_backward(orca_ctx* ctx, const orca_buf* grad_out,
                              const orca_buf* out_primal, const int64_t* dims, int rank,
                              orca_dtype dtype, orca_buf** out);              /* :137-143 */
orca_status orca_log_backward(orca_ctx* ctx, const orca_buf* grad_out,
                              const orca_buf* in_primal, const int64_t* dims, int rank,
                              orca_dtype dtype, orca_buf** out);              /* :144-150 */
orca_status orca_div(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                     const int64_t* dims, int rank, orca_dtype dtype, orca_buf** out);  /* :153-159 */
orca_status orca_sqrt(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                      orca_dtype dtype, orca_buf** out);                      /* :160 */
orca_status orca_div_backward_lhs(orca_ctx* ctx, const orca_buf* grad_out,
                                  const orca_buf* rhs_primal, const int64_t* dims,
                                  int rank, orca_dtype dtype, orca_buf** out);/* :161-167 */
orca_status orca_div_backward_rhs(orca_ctx* ctx, const orca_buf* grad_out,
                                  const orca_buf* lhs_primal, const orca_buf* rhs_primal,
                                  const int64_t* dims, int rank, orca_dtype dtype,
                                  orca_buf** out);                            /* :168-174 */
orca_status orca_sqrt_backward(orca_ctx* ctx, const orca_buf* grad_out,
                               const orca_buf* out_primal, const int64_t* dims, int rank,
                               orca_dtype dtype, orca_buf** out);             /* :176-182 */
orca_status orca_accumulate_grad(orca_ctx* ctx, const orca_buf* lhs, const orca_buf* rhs,
                                 orca_buf** out);                             /* :185 */
orca_status orca_cast(orca_ctx* ctx, const orca_buf* x, const int64_t* dims, int rank,
                      orca_dtype current, orca_dtype target, orca_buf** out); /* :239-246 */
orca_status orca_has_nan_or_inf(orca_ctx* ctx, const orca_buf* x, orca_dtype dtype,
                                int* result);                                 /* :298 */
orca_status orca_max_to_shape(orca_ctx* ctx, const orca_buf* x, const int64_t* in_dims,
                              int in_rank, const int64_t* out_dims, int out_rank,
                              orca_dtype dtype, orca_buf** out);              /* :299-305 */
orca_status orca_max_to_shape_backward(orca_ctx* ctx, const orca_buf* grad_out,
                                       const orca_buf* in_primal, const orca_buf* out_primal,
                                       const int64_t* in_dims, int in_rank,
                                       const int64_t* out_dims, int out_rank,
                                       orca_dtype dtype, orca_buf** out);     /* :306-314 */
/* Trait methods outside the MLP path (conv2d :189-237, scatter/gather :248-293):
 * exported so the Rust binding is total; they return ORCA_NOT_IMPLEMENTED. */
orca_status orca_conv2d(orca_ctx* ctx, const orca_buf* input, const orca_buf* weight,
                        const orca_buf* bias, const int64_t* in_dims, int in_rank,
                        const int64_t* w_dims, int w_rank, int64_t padding, int64_t stride,
                        int64_t dilation, int64_t groups, orca_dtype dtype, orca_buf** out);
orca_status orca_gather(orca_ctx* ctx, const orca_buf* x, int64_t dim, const orca_buf* index,
                        const int64_t* dims, int rank, const int64_t* index_dims,
                        int index_rank, orca_dtype dtype, orca_buf** out);
orca_status orca_scatter(orca_ctx* ctx, const orca_buf* x, int64_t dim, const orca_buf* index,
                         const orca_buf* src, const int64_t* dims, int rank,
                         const int64_t* index_dims, int index_rank, orca_dtype dtype,
                         orca_buf** out);

/* ---- fused ops (not in the trait; inherent methods of the CUDA backend) ---- */
/* out = relu?(x @ w + b), x [m,k], w [k,n] ([in,out], python/orca/nn/linear.py:29),
 * b [1,n] (nullable).  One GEMM with the bias and ReLU in its epilogue. */
orca_status orca_linear_fwd(orca_ctx* ctx, const orca_buf* x, const orca_buf* w,
                            const orca_buf* b, int64_t m, int64_t k, int64_t n, int relu,
                            orca_buf** out);
/* Backward of out = x @ w + b, fused (MatMulBackward + ExpandBackward,
 * orca-autograd/src/backend.rs:1448-1499 and 1675-1698): dW = x^T dy [k,n],
 * db = the row sum of dy [1,n], and, when dx is not null, dX = dy w^T [m,k]
 * masked by (mask > 0) when mask is given — the ReluBackward of the layer
 * below (backend.rs:1624-1646; mask = that layer's pre-activation or
 * activation).  x [m,k], w [k,n] ([in,out]), dy [m,n]; F32 only. */
orca_status orca_linear_bwd(orca_ctx* ctx, const orca_buf* x, const orca_buf* w,
                            const orca_buf* dy, const orca_buf* mask, int64_t m, int64_t k,
                            int64_t n, orca_buf** dx, orca_buf** dw, orca_buf** db);
/* C[m,n] = op(A) @ op(B) on plain f32 buffers, FP32-accurate.  a_mn_major /
 * b_mn_major select the storage of A ([k,m] instead of [m,k]) and B ([k,n]
 * row-major, the reference's [in,out] layout, vs [n,k]), i.e. X@W, dY@W^T and
 * X^T@dY without materialised transposes (orca-autograd/src/backend.rs:
 * 1448-1499 transposes explicitly).  path: 0 auto, 1 SIMT FFMA, 2 tcgen05
 * (ORCA_INVALID_ARGUMENT when the shape/alignment does not allow it), 3 / 4
 * tcgen05 with the single-CTA / CTA-pair (256 x 256 tiles on two SMs) kernel. */
orca_status orca_gemm_ex(orca_ctx* ctx, int64_t m, int64_t n, int64_t k, const orca_buf* a,
                         int a_mn_major, const orca_buf* b, int b_mn_major, int path,
                         orca_buf** out);
/* Softmax cross-entropy forward + backward in one kernel
 * (python/orca/nn/loss.py:59-100, mean reduction).  loss [1], dP [b,c]. */
orca_status orca_softmax_ce_fwd_bwd(orca_ctx* ctx, const orca_buf* logits,
                                    const orca_buf* target, int64_t batch, int64_t classes,
                                    orca_buf** loss, orca_buf** dlogits);
/* Softmax cross-entropy forward + backward that allocates nothing.  No
 * counterpart in the reference: an addition for callers that cannot call
 * cudaMalloc at this point -- code whose device memory is owned by another
 * allocator (a framework's caching pool, a preallocated arena) and
 * latency-bound loops, where a device allocation can synchronise the GPU or
 * fragment the caller's pool.  The caller passes device pointers for every
 * input and output: logits and target [batch, classes], loss [1], dlogits
 * [batch, classes] (NULL for forward only).  The per-row scratch is a fixed
 * device array of 2^20 rows (4 MiB, resident on every GPU that loads the
 * library); larger batches are rejected with ORCA_INVALID_ARGUMENT.  The
 * array's device address is looked up once per device by orca_ctx_create
 * (with that device current), so the call itself does no set-up.  All calls
 * share the one array: calls that overlap on the GPU (other streams, other
 * host threads with their own contexts on the same device) race on it. */
orca_status orca_softmax_ce_fwd_bwd_noalloc(orca_ctx* ctx, const float* logits,
                                            const float* target, int64_t batch, int64_t classes,
                                            float* loss, float* dlogits);
/* In-place optimizer updates with the reference's per-op f32 rounding
 * (python/orca/optim/sgd.py:55-79, adamw.py:75-99).  v / m may be NULL when
 * unused; first != 0 is SGD's first momentum step. */
orca_status orca_sgd_step(orca_ctx* ctx, orca_buf* p, const orca_buf* g, orca_buf* v,
                          double lr, double momentum, double dampening,
                          double weight_decay, int first);
orca_status orca_adamw_step(orca_ctx* ctx, orca_buf* p, const orca_buf* g, orca_buf* m,
                            orca_buf* v, double lr, double beta1, double beta2, double eps,
                            double weight_decay, int64_t t);

/* ---- data-parallel step runner -------------------------------------------------
 * Sequential(Linear, ReLU, ..., Linear) + CrossEntropyLoss + SGD/AdamW on
 * device-resident parameters (python/orca/nn/model.py:546-552 step), with
 * an optional communicator for DistributedDataParallel.all_reduce_gradients
 * (python/orca/distributed.py:222-256). */
typedef enum { ORCA_OPT_SGD = 0, ORCA_OPT_ADAMW = 1 } orca_optimizer;

typedef struct {
  int n_layers;              /* number of Linear layers */
  const int64_t* dims;       /* n_layers + 1 feature sizes */
  int64_t batch;             /* per-rank batch */
  orca_optimizer optimizer;
  double lr, momentum, dampening, weight_decay;   /* SGD (sgd.py:30-44) */
  double beta1, beta2, eps;                       /* AdamW (adamw.py:24-38) */
  int gemm_path;             /* 0 auto (tcgen05 where shapes allow and the output has
                                enough tiles), 1 SIMT FFMA only, 2 tcgen05 wherever allowed;
                                3 / 4 as 2 with the single-CTA / CTA-pair tcgen05 kernel */
} orca_mlp_config;

orca_status orca_mlp_create(orca_ctx* ctx, const orca_mlp_config* cfg, orca_mlp** out);
orca_status orca_mlp_destroy(orca_mlp* mlp);
/* Parameters in Module.parameters() order: 2*l = W_l [in,out], 2*l+1 = b_l [1,out]. */
orca_status orca_mlp_num_params(const orca_mlp* mlp, int* count);
orca_status orca_mlp_param_numel(const orca_mlp* mlp, int index, int64_t* numel);
orca_status orca_mlp_set_param(orca_mlp* mlp, int index, const float* host, int64_t numel);
orca_status orca_mlp_get_param(orca_mlp* mlp, int index, float* host, int64_t numel);
/* Gradient of the last backward (after the all-reduce when a comm is attached). */
orca_status orca_mlp_get_grad(orca_mlp* mlp, int index, float* host, int64_t numel);
/* Inspection (no counterpart in the reference, which keeps activations in
 * its tape): the input of Linear `layer` (1..n_layers-1) in the last forward,
 * i.e. the ReLU output of the layer below, [batch, dims[layer]].  Parity
 * tests read the ReLU masks the step used from it. */
orca_status orca_mlp_get_activation(orca_mlp* mlp, int layer, float* host, int64_t numel);
/* Optimizer state of parameter `index` for checkpoints (the reference's
 * optimizers keep it in Python objects and never save it, optim/sgd.py:46-79,
 * adamw.py:48-99): slot 0 = SGD velocity / AdamW first moment m, slot 1 =
 * AdamW second moment v.  *numel = 0 when the optimizer has no such slot. */
orca_status orca_mlp_state_numel(const orca_mlp* mlp, int slot, int index, int64_t* numel);
orca_status orca_mlp_get_state(orca_mlp* mlp, int slot, int index, float* host, int64_t numel);
orca_status orca_mlp_set_state(orca_mlp* mlp, int slot, int index, const float* host,
                               int64_t numel);
/* Step counters: AdamW's t (bias correction) and whether SGD's velocity holds a
 * value (the first momentum step sets v = g, sgd.py:67-71). */
orca_status orca_mlp_get_step(const orca_mlp* mlp, int64_t* t, int* velocity_started);
orca_status orca_mlp_set_step(orca_mlp* mlp, int64_t t, int velocity_started);
/* Attach (or detach with NULL) the communicator used by every later step.
 * Collective when the peer exchange is chosen (every rank must call it). */
orca_status orca_mlp_attach_comm(orca_mlp* mlp, orca_comm* comm, size_t bucket_bytes);
/* How the step averages gradients across ranks (set before attaching; same
 * on every rank).  NCCL: ncclAllReduce with ncclAvg per bucket.  PEER: the
 * ranks' gradient arenas are mapped into each other with CUDA IPC and one
 * kernel per layer sums every element in float64 in rank order and scales
 * by 1/world -- the reference's average (python/orca/distributed.py:238-256)
 * bit for bit at every world size -- running on the SMs beside the GEMMs of
 * the rest of the backward pass.  AUTO: PEER when the mapping can be set up
 * (world 2..8, CUDA IPC available), else NCCL. */
typedef enum { ORCA_XCHG_AUTO = 0, ORCA_XCHG_NCCL = 1, ORCA_XCHG_PEER = 2 } orca_exchange;
orca_status orca_mlp_set_exchange(orca_mlp* mlp, int mode);
/* The exchange in use: 0 none (no communicator), ORCA_XCHG_NCCL or ORCA_XCHG_PEER. */
orca_status orca_mlp_exchange_kind(const orca_mlp* mlp, int* kind);
/* The gradient exchange plan a runner with these dims and bucket size uses
 * (host only; no device needed), replacing the per-parameter loop of
 * DistributedDataParallel.all_reduce_gradients (python/orca/distributed.py:
 * 222-256).  The gradient arena holds the parameters in Module.parameters()
 * order (python/orca/nn/module.py:32-44); bucket i covers floats
 * [offsets[i], offsets[i] + counts[i]) of it and belongs to layer layers[i].
 * Buckets come in exchange order: last layer first, each layer's (dW, db)
 * range in pieces of at most bucket_bytes (0 = whole layer).  With all three
 * arrays NULL only *n_buckets is set. */
orca_status orca_mlp_bucket_plan(int n_layers, const int64_t* dims, size_t bucket_bytes,
                                 int capacity, int64_t* offsets, int64_t* counts, int* layers,
                                 int* n_buckets);
/* One training step with host inputs: x [batch, dims[0]] and the one-hot (or
 * soft) target t [batch, dims[n_layers]] are copied to the device inside the
 * call; *loss (host, nullable) receives this rank's loss (read back). */
orca_status orca_mlp_step(orca_mlp* mlp, const float* x, const float* t, float* loss);
/* Same step with device-resident inputs (device pointers, f32, row-major).
 * loss_dev (device, nullable) receives the loss; nothing is synchronised. */
orca_status orca_mlp_step_device(orca_mlp* mlp, const float* x_dev, const float* t_dev,
                                 float* loss_dev);
/* Input pipeline (the device side of DataLoader._collate,
 * python/orca/data/dataloader.py:309-350): a batch is staged into one of
 * ORCA_MLP_STAGE_SLOTS device slots by a host->device copy on the trainer's
 * own copy stream, so the copy of batch k+1 runs while step k computes.
 * _stage_batch returns at once when x and t are page-locked (cudaHostAlloc /
 * orca_host_alloc / cudaHostRegister); the host memory must then stay
 * unchanged until the step that consumes the slot has returned with its loss.
 * Pageable sources are copied after a bounded host wait for the slot (the
 * call returns once the data has left the host buffer).  Device pointers are
 * refused.  _step_staged runs orca_mlp_step on the slot's batch, ordered
 * after its copy; *loss (nullable) is read back as orca_mlp_step does.  A slot
 * is consumed by one step; stepping on a slot with nothing staged is
 * ORCA_INVALID_ARGUMENT. */
#define ORCA_MLP_STAGE_SLOTS 2
orca_status orca_mlp_stage_batch(orca_mlp* mlp, int slot, const float* x, const float* t);
orca_status orca_mlp_step_staged(orca_mlp* mlp, int slot, float* loss);
/* Page-locked host memory for staged batches (cudaHostAlloc, portable). */
orca_status orca_host_alloc(size_t bytes, void** out);
orca_status orca_host_free(void* ptr);
/* Forward + loss only (no update): logits_host [batch, classes] and *loss. */
orca_status orca_mlp_forward(orca_mlp* mlp, const float* x, const float* t, float* logits,
                             float* loss);
/* Number of this library's kernels the last step launched. */
orca_status orca_mlp_launches_per_step(const orca_mlp* mlp, int* count);
/* CUDA-graph form of orca_mlp_step_device for fixed device buffers: _capture
 * records one step (it runs one ordinary step first if the optimizer has not
 * stepped yet), _replay launches the recorded step -- one launch for the
 * whole step, for models whose steps are launch-bound.  SGD only (AdamW's
 * bias corrections change every step: ORCA_NOT_IMPLEMENTED), no communicator,
 * not while profiling.  Parameters and optimizer state live in the trainer,
 * so replays continue training exactly as ordinary steps would. */
orca_status orca_mlp_graph_capture(orca_mlp* mlp, const float* x_dev, const float* t_dev,
                                   float* loss_dev);
orca_status orca_mlp_graph_replay(orca_mlp* mlp);
orca_status orca_mlp_graph_release(orca_mlp* mlp);
/* Per-kernel-group timing of later steps: CUDA events recorded on the compute
 * stream around each GEMM / CE / column-sum / optimizer group.  _end
 * synchronises and aggregates; _site reads one group (name, total ms over
 * the profiled steps, launches, algorithmic FLOPs and bytes per launch, and
 * the GEMM path taken: 1 SIMT, 2 tcgen05, -1 not a GEMM). */
orca_status orca_mlp_profile_begin(orca_mlp* mlp);
orca_status orca_mlp_profile_end(orca_mlp* mlp, int* n_sites);
orca_status orca_mlp_profile_site(const orca_mlp* mlp, int index, const char** name,
                                  double* ms_total, int* launches, double* flops_per_launch,
                                  double* bytes_per_launch, int* gemm_path);

/* ---- communicator: NCCL over NVLink (replaces the TCP star of
 * python/orca/distributed.py:161-256) ---------------------------------------- */
#define ORCA_COMM_ID_BYTES 128
/* Rank 0 creates the id and ships it to the others out of band. */
orca_status orca_comm_get_unique_id(void* id_out /* ORCA_COMM_ID_BYTES */);
orca_status orca_comm_init(orca_ctx* ctx, int rank, int world, const void* id,
                           double timeout_s, orca_comm** out);
orca_status orca_comm_destroy(orca_comm* comm);
/* Abort a communicator (ncclCommAbort); pending collectives end with errors. */
orca_status orca_comm_abort(orca_comm* comm);
/* In-place all-reduce average of n f32 values at dev_ptr on the comm stream,
 * ordered after the ctx compute stream; bounded by the comm's timeout. */
orca_status orca_comm_allreduce_avg(orca_comm* comm, float* dev_ptr, size_t n);
/* Same on library buffers, in buckets of bucket_bytes (0 = one call per buffer). */
orca_status orca_comm_allreduce_avg_bufs(orca_comm* comm, orca_buf* const* bufs, int nbufs,
                                         size_t bucket_bytes);

#ifdef __cplusplus
}
#endif
#endif /* ORCA_CUDA_H */
