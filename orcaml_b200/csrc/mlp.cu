// mlp.cu -- the data-parallel MLP training step on device-resident state.
//
// One step = python/orca/nn/model.py:546-552 (zero_grad, forward, loss,
// backward, all_reduce_gradients, optimizer.step) for
// Sequential(Linear, ReLU, ..., Linear) + CrossEntropyLoss + SGD/AdamW:
//
//   forward   Z = X @ W (+ b, ReLU) ........ tcgen05 GEMM, bias+ReLU+split epilogue;
//             the classifier layer (C <= 16) inside the last hidden GEMM's
//             epilogue, reduced over column slices by head_logits
//   loss      softmax-CE fwd+bwd ........... ce_kernel (one thread per row)
//   backward  classifier dW, dX (masked) and the bias gradient of the layer
//             below ........................ head_backward, one pass
//             dW = X^T @ dZ ................ GEMM (CTA-pair kernel), MN-major A and
//                                            B (no transposes); for layer 0 the
//                                            input's column of ones adds db0
//             dX = dZ @ W^T, * (X > 0) ..... GEMM, K-major B, ReLU-mask+split epilogue
//             db of the classifier ......... colsum kernels
//   exchange  all-reduce average of each layer's (dW, db) on the comm stream,
//             started as soon as that layer's gradients exist
//   update    SGD / SGD-momentum / AdamW kernels with the reference's per-op
//             f32 rounding, writing the weights back as (hi, lo) planes; with a
//             communicator each layer waits only for its own all-reduce.
//
// GEMM operands live as (hi, lo) plane pairs (gemm.cuh); the reference's
// [in, out] weight layout (python/orca/nn/linear.py:29) is kept.
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"

namespace orca {
orca_status comm_allreduce_avg_stream(orca_comm* comm, float* ptr, size_t n, cudaStream_t stream);
}  // namespace orca

namespace orca {

// ---------------------------------------------------------------- kernels
// Softmax cross-entropy forward + backward for one row per thread, restating
// python/orca/nn/loss.py:83-100 and the reverse sweep of the tape nodes it
// records (orca-autograd/src/backend.rs:1380-1793, node by node).  row_loss[b]
// gets sum_c -(t*ls); the mean is taken by ce_loss_kernel.
__global__ void ce_kernel(const float* __restrict__ P, const float* __restrict__ T, int64_t B,
                          int64_t C, float inv_b, float* __restrict__ dP,
                          float* __restrict__ row_loss) {
  const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const float* p = P + b * C;
  const float* t = T + b * C;
  float m = -3.402823466e38f;
  for (int64_t c = 0; c < C; ++c) m = p[c] > m ? p[c] : m;
  float s = 0.0f;
  for (int64_t c = 0; c < C; ++c) s = __fadd_rn(s, expf(__fsub_rn(p[c], m)));
  const float lse = __fadd_rn(m, logf(fmaxf(s, 1e-7f)));
  float per = 0.0f;
  for (int64_t c = 0; c < C; ++c) {
    const float ls = __fsub_rn(p[c], lse);
    per = __fadd_rn(per, __fmul_rn(__fmul_rn(t[c], ls), -1.0f));
  }
  row_loss[b] = per;
  if (!dP) return;
  float* d = dP + b * C;
  const float g_tl = __fmul_rn(inv_b, -1.0f);
  float g_s0 = 0.0f;
  for (int64_t c = 0; c < C; ++c) {
    const float g_ls = __fadd_rn(0.0f, __fmul_rn(g_tl, t[c]));
    const float g_lse = __fadd_rn(0.0f, __fmul_rn(g_ls, -1.0f));
    g_s0 = __fadd_rn(g_s0, __fdiv_rn(__fadd_rn(0.0f, g_lse), s));
  }
  float g_m0 = 0.0f;
  for (int64_t c = 0; c < C; ++c) {
    const float g_ls = __fadd_rn(0.0f, __fmul_rn(g_tl, t[c]));
    const float g_lse = __fadd_rn(0.0f, __fmul_rn(g_ls, -1.0f));
    const float e = expf(__fsub_rn(p[c], m));
    const float g_s = __fmul_rn(g_s0, e);
    g_m0 = __fadd_rn(g_m0, __fadd_rn(__fadd_rn(0.0f, g_lse), __fadd_rn(0.0f, __fmul_rn(g_s, -1.0f))));
    d[c] = __fadd_rn(__fadd_rn(0.0f, g_ls), __fadd_rn(0.0f, g_s));
  }
  for (int64_t c = 0; c < C; ++c) {
    const float gi = p[c] == m ? __fadd_rn(0.0f, g_m0) : 0.0f;
    d[c] = __fadd_rn(d[c], gi);
  }
}

// The same computation with one warp per row, for wide rows (C > 32; the
// thread-per-row form would read C-float rows strided across a warp and run
// few threads, e.g. 2048 rows of C = 1000).  The row is staged in shared
// memory with coalesced loads; every per-element term is computed by all
// lanes in parallel, and each of the reference's serial sums runs on one
// lane in ascending c over the staged terms, so the result is bit-identical
// to ce_kernel.  Shared memory per warp: 5 * C floats.
constexpr int CE_WIDE_MIN_C = 33, CE_WIDE_MAX_C = 8192;
__global__ void ce_wide_kernel(const float* __restrict__ P, const float* __restrict__ T, int64_t B,
                               int C, float inv_b, float* __restrict__ dP,
                               float* __restrict__ row_loss) {
  extern __shared__ float ce_sm[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t b = (int64_t)blockIdx.x * (blockDim.x / 32) + warp;
  if (b >= B) return;   // whole warps leave together
  float* sp = ce_sm + (size_t)warp * 5 * C;
  float* st = sp + C;
  float* se = st + C;
  float* sq = se + C;
  float* sr = sq + C;
  const float* p = P + b * C;
  const float* t = T + b * C;
  float m = -3.402823466e38f;
  for (int c = lane; c < C; c += 32) {
    const float pv = p[c];
    sp[c] = pv;
    st[c] = t[c];
    m = pv > m ? pv : m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float q = __shfl_xor_sync(0xffffffffu, m, o);
    m = q > m ? q : m;
  }
  for (int c = lane; c < C; c += 32) se[c] = expf(__fsub_rn(sp[c], m));
  __syncwarp();
  float s = 0.0f;
  if (lane == 0)
    for (int c = 0; c < C; ++c) s = __fadd_rn(s, se[c]);
  s = __shfl_sync(0xffffffffu, s, 0);
  const float lse = __fadd_rn(m, logf(fmaxf(s, 1e-7f)));
  const float g_tl = __fmul_rn(inv_b, -1.0f);
  for (int c = lane; c < C; c += 32) {
    const float ls = __fsub_rn(sp[c], lse);
    sq[c] = __fmul_rn(__fmul_rn(st[c], ls), -1.0f);
    const float g_ls = __fadd_rn(0.0f, __fmul_rn(g_tl, st[c]));
    const float g_lse = __fadd_rn(0.0f, __fmul_rn(g_ls, -1.0f));
    sr[c] = __fdiv_rn(__fadd_rn(0.0f, g_lse), s);
  }
  __syncwarp();
  // Lane 0: the loss sum; lane 1: g_s0 -- the same loop over different arrays.
  float acc = 0.0f;
  if (lane < 2) {
    const float* arr = lane == 0 ? sq : sr;
    for (int c = 0; c < C; ++c) acc = __fadd_rn(acc, arr[c]);
  }
  const float per = __shfl_sync(0xffffffffu, acc, 0);
  const float g_s0 = __shfl_sync(0xffffffffu, acc, 1);
  if (lane == 0) row_loss[b] = per;
  if (!dP) return;
  __syncwarp();
  for (int c = lane; c < C; c += 32) {
    const float g_ls = __fadd_rn(0.0f, __fmul_rn(g_tl, st[c]));
    const float g_lse = __fadd_rn(0.0f, __fmul_rn(g_ls, -1.0f));
    const float g_s = __fmul_rn(g_s0, se[c]);
    sq[c] = __fadd_rn(__fadd_rn(0.0f, g_lse), __fadd_rn(0.0f, __fmul_rn(g_s, -1.0f)));
    sr[c] = __fadd_rn(__fadd_rn(0.0f, g_ls), __fadd_rn(0.0f, g_s));
  }
  __syncwarp();
  float g_m0 = 0.0f;
  if (lane == 0)
    for (int c = 0; c < C; ++c) g_m0 = __fadd_rn(g_m0, sq[c]);
  g_m0 = __shfl_sync(0xffffffffu, g_m0, 0);
  float* d = dP + b * C;
  for (int c = lane; c < C; c += 32) {
    const float gi = sp[c] == m ? __fadd_rn(0.0f, g_m0) : 0.0f;
    d[c] = __fadd_rn(sr[c], gi);
  }
}

// loss = (sum_b row_loss[b]) * f32(1/B) with the sum taken serially in
// ascending b, as the reference's mean does (sum_to_shape's serial loop,
// orca-backend-cpu/src/backend.rs:519-527, then the multiply of
// orca-python/src/lib.rs:664-669).  The rows are staged in shared memory by
// the whole block (coalesced), one thread runs the chain (about 4 cycles per
// row: ~9 us at B = 4096).
constexpr int CE_LOSS_THREADS = 1024, CE_LOSS_TILE = 8192;
__global__ void __launch_bounds__(CE_LOSS_THREADS)
ce_loss_kernel(const float* __restrict__ row_loss, int64_t B, float inv_b,
               float* __restrict__ loss) {
  __shared__ float tile[CE_LOSS_TILE];
  float acc = 0.0f;
  for (int64_t b0 = 0; b0 < B; b0 += CE_LOSS_TILE) {
    const int n = (int)(B - b0 < CE_LOSS_TILE ? B - b0 : CE_LOSS_TILE);
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) tile[i] = row_loss[b0 + i];
    __syncthreads();
    if (threadIdx.x == 0) {
      int i = 0;
      for (; i + 8 <= n; i += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = tile[i + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, v[j]);
      }
      for (; i < n; ++i) acc = __fadd_rn(acc, tile[i]);
    }
  }
  if (threadIdx.x == 0) loss[0] = __fmul_rn(acc, inv_b);
}

// db[n] = sum_b g[b, n]: partial sums over row chunks (grid.y), then an
// ordered sum of the partials -- deterministic for a given shape.
constexpr int COLSUM_ROWS = 256;
__global__ void colsum_partial_kernel(const float* __restrict__ hi, const float* __restrict__ lo,
                                      int64_t B, int64_t N, int64_t ld, float* __restrict__ part) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int64_t b0 = (int64_t)blockIdx.y * COLSUM_ROWS;
  const int64_t b1 = b0 + COLSUM_ROWS < B ? b0 + COLSUM_ROWS : B;
  float acc = 0.0f;
  for (int64_t b = b0; b < b1; ++b) {
    float v = hi[b * ld + n];
    if (lo) v = __fadd_rn(v, lo[b * ld + n]);
    acc = __fadd_rn(acc, v);
  }
  part[(int64_t)blockIdx.y * N + n] = acc;
}

__global__ void colsum_final_kernel(const float* __restrict__ part, int chunks, int64_t N,
                                    float* __restrict__ out) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float acc = 0.0f;
  for (int c = 0; c < chunks; ++c) acc = __fadd_rn(acc, part[(int64_t)c * N + n]);
  out[n] = acc;
}

// Row losses of a softmax-CE batch (ce_kernel or, for wide rows, ce_wide_kernel).
static void launch_ce_rows(cudaStream_t stream, const float* P, const float* T, int64_t B,
                           int64_t C, float inv_b, float* dP, float* rows) {
  if (C >= CE_WIDE_MIN_C && C <= CE_WIDE_MAX_C) {
    // Warps per block so that 5*C floats per warp stay within 96 KB a block
    // (one warp of 160 KB at the widest rows).
    const int wpb = (int)std::max<int64_t>(1, std::min<int64_t>(8, (96 * 1024) / (20 * C)));
    const size_t smem = (size_t)wpb * 20 * (size_t)C;
    static std::once_flag attr_once[128];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(attr_once[dev & 127], [] {
      cudaFuncSetAttribute(ce_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           20 * CE_WIDE_MAX_C);
    });
    ce_wide_kernel<<<(unsigned)cdiv(B, wpb), 32 * wpb, smem, stream>>>(P, T, B, (int)C, inv_b, dP,
                                                                     rows);
  } else {
    ce_kernel<<<(unsigned)cdiv(B, 128), 128, 0, stream>>>(P, T, B, C, inv_b, dP, rows);
  }
}

struct SgdArgs {
  float lr, wd, mom, one_minus_damp;
  int use_wd, use_mom, use_damp, first;
};

// SGD.step (python/orca/optim/sgd.py:55-79) of one parameter, one rounding per
// reference op.  v (the velocity) is read only after the first momentum step
// and written whenever momentum is on.
__device__ __forceinline__ float sgd_elem(float p, float gi, float& v, const SgdArgs& a) {
  if (a.use_wd) gi = __fadd_rn(gi, __fmul_rn(p, a.wd));
  if (a.use_mom) {
    if (a.first) v = gi;
    else if (a.use_damp) v = __fadd_rn(__fmul_rn(v, a.mom), __fmul_rn(gi, a.one_minus_damp));
    else v = __fadd_rn(__fmul_rn(v, a.mom), gi);
    gi = v;
  }
  return __fsub_rn(p, __fmul_rn(gi, a.lr));
}

struct AdamArgs {
  float decay, b1, one_minus_b1, b2, one_minus_b2, bc1, bc2, eps, lr;
};

// AdamW.step (python/orca/optim/adamw.py:75-99) of one parameter, one rounding
// per reference op; m and v are updated in place.
__device__ __forceinline__ float adamw_elem(float p, float gi, float& m, float& v,
                                            const AdamArgs& a) {
  const float decayed = __fmul_rn(p, a.decay);
  m = __fadd_rn(__fmul_rn(m, a.b1), __fmul_rn(gi, a.one_minus_b1));
  v = __fadd_rn(__fmul_rn(v, a.b2), __fmul_rn(__fmul_rn(gi, gi), a.one_minus_b2));
  const float mh = __fmul_rn(m, a.bc1);
  const float vh = __fmul_rn(v, a.bc2);
  const float denom = __fadd_rn(__fsqrt_rn(vh), a.eps);
  return __fsub_rn(decayed, __fmul_rn(__fdiv_rn(mh, denom), a.lr));
}

// p is (hi, lo) planes when kPlanes, else plain fp32 in hi.
template <bool kPlanes>
__device__ __forceinline__ float load_param(const float* hi, const float* lo, int64_t i) {
  return kPlanes ? __fadd_rn(hi[i], lo[i]) : hi[i];
}

template <bool kPlanes>
__device__ __forceinline__ void store_param(float* hi, float* lo, int64_t i, float p) {
  if (kPlanes) {
    float h, l;
    split_tf32(p, h, l);
    hi[i] = h;
    lo[i] = l;
  } else {
    hi[i] = p;
  }
}

// Four consecutive parameters per thread and iteration as 128-bit accesses
// (every array 16-byte aligned); the n % 4 tail goes element by element.
template <bool kPlanes>
__device__ __forceinline__ void load_param4(const float* hi, const float* lo, int64_t q,
                                            float (&p)[4]) {
  const float4 h = reinterpret_cast<const float4*>(hi)[q];
  p[0] = h.x; p[1] = h.y; p[2] = h.z; p[3] = h.w;
  if (kPlanes) {
    const float4 l = reinterpret_cast<const float4*>(lo)[q];
    p[0] = __fadd_rn(p[0], l.x); p[1] = __fadd_rn(p[1], l.y);
    p[2] = __fadd_rn(p[2], l.z); p[3] = __fadd_rn(p[3], l.w);
  }
}

template <bool kPlanes>
__device__ __forceinline__ void store_param4(float* hi, float* lo, int64_t q, const float (&p)[4]) {
  if (kPlanes) {
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split_tf32(p[j], h[j], l[j]);
    reinterpret_cast<float4*>(hi)[q] = make_float4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<float4*>(lo)[q] = make_float4(l[0], l[1], l[2], l[3]);
  } else {
    reinterpret_cast<float4*>(hi)[q] = make_float4(p[0], p[1], p[2], p[3]);
  }
}

__device__ __forceinline__ void to4(const float4 v, float (&o)[4]) {
  o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
}

template <bool kPlanes, bool kVec>
__global__ void sgd_kernel(float* __restrict__ hi, float* __restrict__ lo,
                           const float* __restrict__ g, float* __restrict__ v, int64_t n,
                           SgdArgs a) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool read_v = a.use_mom && !a.first;
  int64_t tail = 0;
  if (kVec) {
    const int64_t n4 = n >> 2;
    for (int64_t q = t0; q < n4; q += stride) {
      float p[4], gv[4], vv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      load_param4<kPlanes>(hi, lo, q, p);
      to4(reinterpret_cast<const float4*>(g)[q], gv);
      if (read_v) to4(reinterpret_cast<const float4*>(v)[q], vv);
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = sgd_elem(p[j], gv[j], vv[j], a);
      if (a.use_mom) reinterpret_cast<float4*>(v)[q] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      store_param4<kPlanes>(hi, lo, q, p);
    }
    tail = n4 << 2;
  }
  for (int64_t i = tail + t0; i < n; i += stride) {
    float vi = read_v ? v[i] : 0.0f;
    const float p = sgd_elem(load_param<kPlanes>(hi, lo, i), g[i], vi, a);
    if (a.use_mom) v[i] = vi;
    store_param<kPlanes>(hi, lo, i, p);
  }
}

template <bool kPlanes, bool kVec>
__global__ void adamw_kernel(float* __restrict__ hi, float* __restrict__ lo,
                             const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, int64_t n, AdamArgs a) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t tail = 0;
  if (kVec) {
    const int64_t n4 = n >> 2;
    for (int64_t q = t0; q < n4; q += stride) {
      float p[4], gv[4], mv[4], vv[4];
      load_param4<kPlanes>(hi, lo, q, p);
      to4(reinterpret_cast<const float4*>(g)[q], gv);
      to4(reinterpret_cast<const float4*>(m)[q], mv);
      to4(reinterpret_cast<const float4*>(v)[q], vv);
#pragma unroll
      for (int j = 0; j < 4; ++j) p[j] = adamw_elem(p[j], gv[j], mv[j], vv[j], a);
      reinterpret_cast<float4*>(m)[q] = make_float4(mv[0], mv[1], mv[2], mv[3]);
      reinterpret_cast<float4*>(v)[q] = make_float4(vv[0], vv[1], vv[2], vv[3]);
      store_param4<kPlanes>(hi, lo, q, p);
    }
    tail = n4 << 2;
  }
  for (int64_t i = tail + t0; i < n; i += stride) {
    float mi = m[i], vi = v[i];
    const float p = adamw_elem(load_param<kPlanes>(hi, lo, i), g[i], mi, vi, a);
    m[i] = mi;
    v[i] = vi;
    store_param<kPlanes>(hi, lo, i, p);
  }
}

__global__ void merge_planes_kernel(const float* __restrict__ hi, const float* __restrict__ lo,
                                    float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(hi[i], lo[i]);
}

static SgdArgs sgd_args(double lr, double mom, double damp, double wd, int first) {
  SgdArgs a;
  a.lr = (float)lr;
  a.wd = (float)wd;
  a.mom = (float)mom;
  a.one_minus_damp = (float)(1.0 - damp);
  a.use_wd = wd != 0.0;
  a.use_mom = mom != 0.0;
  a.use_damp = damp != 0.0;
  a.first = first;
  return a;
}

static AdamArgs adam_args(double lr, double b1, double b2, double eps, double wd, int64_t t) {
  AdamArgs a;
  a.decay = (float)(1.0 - lr * wd);
  a.b1 = (float)b1;
  a.one_minus_b1 = (float)(1.0 - b1);
  a.b2 = (float)b2;
  a.one_minus_b2 = (float)(1.0 - b2);
  a.bc1 = (float)(1.0 / (1.0 - std::pow(b1, (double)t)));
  a.bc2 = (float)(1.0 / (1.0 - std::pow(b2, (double)t)));
  a.eps = (float)eps;
  a.lr = (float)lr;
  return a;
}

static int ew_grid(orca_ctx* ctx, int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), (int64_t)ctx->sm_count * 8));
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The optimizer kernels take the 128-bit form when every array they touch is
// 16-byte aligned (parameters, gradients and state of the step runner are,
// except after a parameter whose size is not a multiple of 4).
// Resident 256-thread blocks per SM of a kernel (its register use decides).
template <typename Kernel>
static int blocks_per_sm(Kernel kernel) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  return per_sm;
}

// Grid of a grid-stride kernel: one wave of resident blocks, fewer for small
// n.  A second, partial wave would leave SMs idle while it runs.
static int resident_grid(orca_ctx* ctx, int per_sm, int64_t items) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(cdiv(items, 256),
                                                     (int64_t)ctx->sm_count * per_sm));
}

template <bool kPlanes, bool kVec>
static void launch_sgd_as(orca_ctx* ctx, float* hi, float* lo, const float* g, float* v, int64_t n,
                          const SgdArgs& a) {
  static const int per_sm = blocks_per_sm(sgd_kernel<kPlanes, kVec>);
  const int grid = resident_grid(ctx, per_sm, kVec ? cdiv(n, 4) : n);
  sgd_kernel<kPlanes, kVec><<<grid, 256, 0, ctx->stream>>>(hi, lo, g, v, n, a);
}

template <bool kPlanes, bool kVec>
static void launch_adamw_as(orca_ctx* ctx, float* hi, float* lo, const float* g, float* m,
                            float* v, int64_t n, const AdamArgs& a) {
  static const int per_sm = blocks_per_sm(adamw_kernel<kPlanes, kVec>);
  const int grid = resident_grid(ctx, per_sm, kVec ? cdiv(n, 4) : n);
  adamw_kernel<kPlanes, kVec><<<grid, 256, 0, ctx->stream>>>(hi, lo, g, m, v, n, a);
}

static void launch_sgd(orca_ctx* ctx, float* hi, float* lo, const float* g, float* v, int64_t n,
                       const SgdArgs& a) {
  const bool vec = aligned16(hi) && (!lo || aligned16(lo)) && aligned16(g) &&
                   (!v || aligned16(v));
  if (lo) {
    if (vec) launch_sgd_as<true, true>(ctx, hi, lo, g, v, n, a);
    else launch_sgd_as<true, false>(ctx, hi, lo, g, v, n, a);
  } else {
    if (vec) launch_sgd_as<false, true>(ctx, hi, lo, g, v, n, a);
    else launch_sgd_as<false, false>(ctx, hi, lo, g, v, n, a);
  }
  count_launch(ctx);
}

static void launch_adamw(orca_ctx* ctx, float* hi, float* lo, const float* g, float* m, float* v,
                         int64_t n, const AdamArgs& a) {
  const bool vec = aligned16(hi) && (!lo || aligned16(lo)) && aligned16(g) && aligned16(m) &&
                   aligned16(v);
  if (lo) {
    if (vec) launch_adamw_as<true, true>(ctx, hi, lo, g, m, v, n, a);
    else launch_adamw_as<true, false>(ctx, hi, lo, g, m, v, n, a);
  } else {
    if (vec) launch_adamw_as<false, true>(ctx, hi, lo, g, m, v, n, a);
    else launch_adamw_as<false, false>(ctx, hi, lo, g, m, v, n, a);
  }
  count_launch(ctx);
}

// g[i] = mask[i] > 0 ? g[i] : 0 (one comparison, no arithmetic: bit-exact).
__global__ void mask_kernel(float* __restrict__ g, const float* __restrict__ mask, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    if (!(mask[i] > 0.0f)) g[i] = 0.0f;
}

orca_status colsum(orca_ctx* ctx, const float* hi, const float* lo, int64_t B, int64_t N,
                   int64_t ld, float* out, float* part) {
  const int chunks = (int)cdiv(B, COLSUM_ROWS);
  dim3 g1((unsigned)cdiv(N, 256), (unsigned)chunks);
  colsum_partial_kernel<<<g1, 256, 0, ctx->stream>>>(hi, lo, B, N, ld, part);
  colsum_final_kernel<<<(unsigned)cdiv(N, 256), 256, 0, ctx->stream>>>(part, chunks, N, out);
  count_launch(ctx, 2);
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

}  // namespace orca

using namespace orca;

// The gradient exchange plan.  The arena holds the gradients in
// Module.parameters() order (python/orca/nn/module.py:32-44: W0, b0, W1, b1,
// ...), so each layer's (dW, db) is one contiguous range; the layers are
// exchanged last layer first (the order the backward pass finishes them in),
// each in buckets of at most bucket_bytes (0: the whole layer).  The
// reference averages every parameter independently
// (python/orca/distributed.py:238-256), so neither the order nor the bucket
// boundaries change any result.
struct Bucket {
  int64_t offset, count;
  int layer;
};
static void bucket_plan(int L, const int64_t* dims, size_t bucket_bytes, std::vector<Bucket>& out) {
  std::vector<int64_t> layer_off(L);
  int64_t off = 0;
  for (int l = 0; l < L; ++l) {
    layer_off[l] = off;
    off += dims[l] * dims[l + 1] + dims[l + 1];
  }
  for (int l = L - 1; l >= 0; --l) {
    const int64_t n = dims[l] * dims[l + 1] + dims[l + 1];
    const int64_t chunk = bucket_bytes ? std::max<int64_t>((int64_t)(bucket_bytes / 4), 1) : n;
    for (int64_t o = 0; o < n; o += chunk) out.push_back({layer_off[l] + o, std::min(chunk, n - o), l});
  }
}

// =============================================================== step runner
struct orca_mlp {
  orca_ctx* ctx = nullptr;
  int L = 0;
  std::vector<int64_t> dims;
  int64_t B = 0;
  orca_optimizer opt = ORCA_OPT_SGD;
  double lr = 0, mom = 0, damp = 0, wd = 0, b1 = 0.9, b2 = 0.999, eps = 1e-8;
  int gemm_path = GEMM_AUTO;
  int64_t t = 0;                     // AdamW step count
  bool vel_init = false;             // SGD momentum buffers hold a value
  // parameters
  std::vector<float*> w_hi, w_lo, bias;   // w_lo = w_hi + K*N (one allocation per weight)
  std::vector<int64_t> p_off;        // offset of each parameter in the gradient arena
  int64_t n_params = 0;
  float* grads = nullptr;            // gradient arena, Module.parameters() order
  float* state0 = nullptr;           // SGD velocity / AdamW m (same layout as grads)
  float* state1 = nullptr;           // AdamW v
  // activations
  float* x_planes = nullptr;         // [2][B][x_ld]: input planes + a column of ones
  int64_t x_ld = 0;                  // dims[0] + 1 rounded up to a multiple of 4
  std::vector<float*> act_planes;    // act_planes[l] = [2][B][dims[l]], l = 1..L-1
  // ReLU decisions of act[l] as bits ([B][ceil(dims[l] / 32)] words), written by
  // the forward GEMM's epilogue and read by the dX GEMM's mask epilogue when
  // both run on the tensor cores; relu_bits_ok[l]: this step's forward wrote them.
  std::vector<uint32_t*> relu_bits;
  std::vector<char> relu_bits_ok;
  float* t_buf = nullptr;            // one-hot target [B][C]
  float* x_stage = nullptr;          // raw input [B][dims[0]]
  float* logits = nullptr;           // [B][C]
  float* dlogits = nullptr;          // [B][C]
  float* dlogit_planes = nullptr;    // [2][B][C]: dlogits split for the classifier's products
                                     // when they run as GEMMs (no classifier fusion)
  float* row_loss = nullptr;         // [B]
  float* loss = nullptr;             // [1]
  float* dz[2] = {nullptr, nullptr}; // ping-pong (hi, lo) planes of hidden-layer dZ
  int64_t dz_plane = 0;              // elements per plane in dz buffers
  float* colsum_part = nullptr;
  // Classifier-layer fusion (C <= HEAD_MAX_CLASSES, at least one hidden
  // layer, tensor-core path allowed): logits from the last hidden GEMM's
  // epilogue, dW and dX of the classifier layer in one pass (head_* kernels).
  bool use_head = false;
  float* host_stage = nullptr;       // pinned: [0] loss, [1] device error word
  float* head_part = nullptr;        // dot slices [S][B][head_ldp] or dW row-block partials
  float* head_w = nullptr;           // classifier weights packed [H][16] for the dot
  int64_t head_ldp = 0;
  float* workspace = nullptr;
  size_t workspace_bytes = 0;
  std::vector<void*> allocs;
  // data parallel
  orca_comm* comm = nullptr;
  size_t bucket_bytes = 0;
  int xchg_mode = ORCA_XCHG_AUTO;   // requested exchange (orca_mlp_set_exchange)
  PeerArena* pex = nullptr;         // peer exchange of the gradient arena, when in use
  uint32_t pex_seq = 0;             // steps exchanged through pex (same on every rank)
  cudaEvent_t ev_layer[64];         // layer's gradients ready (compute stream)
  cudaEvent_t ev_reduced[64];       // layer's gradients averaged (comm stream)
  int last_launches = 0;
  // Input staging (orca_mlp_stage_batch / _step_staged): batches copied
  // host->device on the trainer's own stream into one of the slots while the
  // previous step computes; allocated on first use.
  cudaStream_t copy_stream = nullptr;
  float* slot_x[ORCA_MLP_STAGE_SLOTS] = {};
  float* slot_t[ORCA_MLP_STAGE_SLOTS] = {};
  cudaEvent_t ev_staged[ORCA_MLP_STAGE_SLOTS] = {};     // slot's copy done (copy stream)
  cudaEvent_t ev_consumed[ORCA_MLP_STAGE_SLOTS] = {};   // slot read by its step (compute stream)
  bool slot_ready[ORCA_MLP_STAGE_SLOTS] = {};
  // Captured step (orca_mlp_graph_*).
  cudaGraphExec_t graph_exec = nullptr;
  int graph_launches = 0;
  // Optional per-kernel-group timing: CUDA events recorded on the compute
  // stream around each group of a step while profiling is on.
  struct ProfSite { std::string name; double flops = 0, bytes = 0; double ms = 0; int count = 0;
                    int gemm_path = -1; };
  struct ProfRec { int site; cudaEvent_t a, b; cudaStream_t stream; };
  bool profiling = false;
  std::vector<ProfSite> sites;
  std::vector<ProfRec> recs;
  std::vector<cudaEvent_t> event_pool;
};

static cudaEvent_t pool_event(orca_mlp* m) {
  if (!m->event_pool.empty()) {
    cudaEvent_t e = m->event_pool.back();
    m->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Opens a timed group; returns a record index (or -1 when not profiling).
static int prof_open(orca_mlp* m, const std::string& name, double flops, double bytes,
                     int gemm_path = -1, cudaStream_t stream = nullptr) {
  if (!m->profiling) return -1;
  int site = -1;
  for (size_t i = 0; i < m->sites.size(); ++i)
    if (m->sites[i].name == name) { site = (int)i; break; }
  if (site < 0) {
    orca_mlp::ProfSite ps;
    ps.name = name;
    ps.flops = flops;
    ps.bytes = bytes;
    ps.gemm_path = gemm_path;
    m->sites.push_back(ps);
    site = (int)m->sites.size() - 1;
  }
  orca_mlp::ProfRec r;
  r.site = site;
  r.a = pool_event(m);
  r.b = pool_event(m);
  r.stream = stream ? stream : m->ctx->stream;
  cudaEventRecord(r.a, r.stream);
  m->recs.push_back(r);
  return (int)m->recs.size() - 1;
}

static void prof_close(orca_mlp* m, int rec) {
  if (rec < 0) return;
  cudaEventRecord(m->recs[rec].b, m->recs[rec].stream);
}

static orca_status mlp_alloc(orca_mlp* m, void** p, size_t bytes) {
  ORCA_CUDA_TRY(cudaMalloc(p, bytes));
  m->allocs.push_back(*p);
  return ORCA_OK;
}

static orca_status mlp_forward_impl(orca_mlp* m, bool with_loss_grad);

// Input planes: x [B][D] -> hi, lo [B][x_ld] with column D = 1 (hi) / 0 (lo)
// and zeros after it (see the dW product of layer 0).
__global__ void split_input_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                   float* __restrict__ lo, int64_t B, int64_t D, int64_t ld) {
  const int64_t n = B * ld;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / ld, c = i % ld;
    float h = c == D ? 1.0f : 0.0f, l = 0.0f;
    if (c < D) split_tf32(x[r * D + c], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

static orca_status split_input(orca_mlp* m, const float* x) {
  const int64_t n = m->B * m->x_ld;
  const int blocks = (int)std::min<int64_t>(cdiv(n, 256), (int64_t)m->ctx->sm_count * 8);
  split_input_kernel<<<blocks, 256, 0, m->ctx->stream>>>(x, m->x_planes, m->x_planes + n, m->B,
                                                         m->dims[0], m->x_ld);
  count_launch(m->ctx);
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}
static orca_status mlp_backward_impl(orca_mlp* m);
static orca_status mlp_update_impl(orca_mlp* m);

// Waits for the step's work with the context's deadline.  A deadline that
// passes while a communicator is attached means a peer stopped taking part
// (the compute stream waits on the gradient all-reduce): the communicator is
// aborted, which ends its pending collective, the streams drain (bounded) and
// the caller gets ORCA_TIMEOUT.  The trainer is then detached from the
// communicator; its parameters are those of the last completed step or a
// partially updated state and must be reloaded before further use.
static orca_status finish_sync(orca_mlp* m) {
  const orca_status s = sync_stream(m->ctx);
  if (s != ORCA_TIMEOUT || !m->comm) return s;
  const std::string why = orca_last_error();
  orca_comm_abort(m->comm);
  m->comm = nullptr;
  sync_stream_for(m->ctx, m->ctx->comm_stream, 30.0);
  sync_stream_for(m->ctx, m->ctx->stream, 30.0);
  return fail(ORCA_TIMEOUT, "%s; communicator aborted (a peer stopped responding)", why.c_str());
}

extern "C" {

orca_status orca_mlp_create(orca_ctx* ctx, const orca_mlp_config* cfg, orca_mlp** out) {
  ORCA_TRY(check_ctx(ctx));
  if (!cfg || !out || !cfg->dims) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (cfg->n_layers < 1 || cfg->n_layers > 60) return fail(ORCA_INVALID_ARGUMENT, "n_layers");
  if (cfg->gemm_path < GEMM_AUTO || cfg->gemm_path > GEMM_TC_PAIR)
    return fail(ORCA_INVALID_ARGUMENT, "gemm_path must be in [0, 4]");
  if (cfg->batch < 1) return fail(ORCA_INVALID_ARGUMENT, "batch must be positive");
  for (int i = 0; i <= cfg->n_layers; ++i)
    if (cfg->dims[i] < 1) return fail(ORCA_INVALID_ARGUMENT, "dims must be positive");
  // Hyper-parameter validation as the reference's optimizers do
  // (python/orca/optim/optimizer.py:6-66, sgd.py:40-44, adamw.py:31-34).
  auto finite_nonneg = [](double v) { return std::isfinite(v) && v >= 0.0; };
  if (!finite_nonneg(cfg->lr)) return fail(ORCA_INVALID_ARGUMENT, "lr must be non-negative");
  if (cfg->optimizer == ORCA_OPT_SGD) {
    if (!finite_nonneg(cfg->momentum) || !finite_nonneg(cfg->weight_decay) ||
        !finite_nonneg(cfg->dampening) || cfg->dampening > 1.0)
      return fail(ORCA_INVALID_ARGUMENT, "invalid SGD hyper-parameters");
  } else if (cfg->optimizer == ORCA_OPT_ADAMW) {
    if (!(cfg->beta1 >= 0.0 && cfg->beta1 < 1.0) || !(cfg->beta2 >= 0.0 && cfg->beta2 < 1.0) ||
        !(std::isfinite(cfg->eps) && cfg->eps > 0.0) || !finite_nonneg(cfg->weight_decay))
      return fail(ORCA_INVALID_ARGUMENT, "invalid AdamW hyper-parameters");
  } else {
    return fail(ORCA_INVALID_ARGUMENT, "unknown optimizer %d", (int)cfg->optimizer);
  }
  orca_mlp* m = new orca_mlp();
  m->ctx = ctx;
  ctx_retain(ctx);
  m->L = cfg->n_layers;
  m->dims.assign(cfg->dims, cfg->dims + cfg->n_layers + 1);
  m->B = cfg->batch;
  m->opt = cfg->optimizer;
  m->lr = cfg->lr;
  m->mom = cfg->momentum;
  m->damp = cfg->dampening;
  m->wd = cfg->weight_decay;
  m->b1 = cfg->beta1;
  m->b2 = cfg->beta2;
  m->eps = cfg->eps;
  m->gemm_path = cfg->gemm_path;
  const int L = m->L;
  const int64_t B = m->B, C = m->dims[L];
  auto cleanup = [&](orca_status s) {
    orca_mlp_destroy(m);
    return s;
  };
  int64_t off = 0;
  m->w_hi.resize(L);
  m->w_lo.resize(L);
  m->bias.resize(L);
  for (int l = 0; l < L; ++l) {
    const int64_t K = m->dims[l], N = m->dims[l + 1];
    void* p;
    orca_status s = mlp_alloc(m, &p, (size_t)(2 * K * N) * 4);
    if (s != ORCA_OK) return cleanup(s);
    m->w_hi[l] = (float*)p;
    m->w_lo[l] = (float*)p + K * N;
    s = mlp_alloc(m, &p, (size_t)N * 4);
    if (s != ORCA_OK) return cleanup(s);
    m->bias[l] = (float*)p;
    m->p_off.push_back(off);
    off += K * N;
    m->p_off.push_back(off);
    off += N;
  }
  m->n_params = off;
  void* p;
  const size_t pbytes = (size_t)off * 4;
#define ALLOC(field, bytes)                               \
  do {                                                    \
    orca_status _s = mlp_alloc(m, &p, (bytes));           \
    if (_s != ORCA_OK) return cleanup(_s);                \
    m->field = (float*)p;                                 \
  } while (0)
  ALLOC(grads, pbytes);
  if (m->opt == ORCA_OPT_ADAMW || m->mom != 0.0) ALLOC(state0, pbytes);
  if (m->opt == ORCA_OPT_ADAMW) ALLOC(state1, pbytes);
  if (m->state0) cudaMemset(m->state0, 0, pbytes);
  if (m->state1) cudaMemset(m->state1, 0, pbytes);
  m->x_ld = (m->dims[0] + 1 + 3) / 4 * 4;
  ALLOC(x_planes, (size_t)(2 * B * m->x_ld) * 4);
  ALLOC(x_stage, (size_t)(B * m->dims[0]) * 4);
  ALLOC(t_buf, (size_t)(B * C) * 4);
  ALLOC(logits, (size_t)(B * C) * 4);
  ALLOC(dlogits, (size_t)(B * C) * 4);
  ALLOC(row_loss, (size_t)B * 4);
  ALLOC(loss, 64);
  m->act_planes.assign(L, nullptr);
  m->relu_bits.assign(L, nullptr);
  m->relu_bits_ok.assign(L, 0);
  int64_t maxh = 1;
  for (int l = 1; l < L; ++l) {
    ALLOC(act_planes[l], (size_t)(2 * B * m->dims[l]) * 4);
    void* pb = nullptr;
    orca_status sb = mlp_alloc(m, &pb, (size_t)(B * cdiv(m->dims[l], 32)) * 4);
    if (sb != ORCA_OK) return cleanup(sb);
    m->relu_bits[l] = static_cast<uint32_t*>(pb);
    maxh = std::max(maxh, m->dims[l]);
  }
  m->dz_plane = B * maxh;
  ALLOC(dz[0], (size_t)(2 * m->dz_plane) * 4);
  ALLOC(dz[1], (size_t)(2 * m->dz_plane) * 4);
  int64_t maxn = C;
  for (int l = 0; l <= L; ++l) maxn = std::max(maxn, m->dims[l]);
  ALLOC(colsum_part, (size_t)(cdiv(B, COLSUM_ROWS) * maxn) * 4);
  m->workspace_bytes = (size_t)64 * (size_t)maxn * 16 * 4;
  ALLOC(workspace, m->workspace_bytes);
  if (cudaMallocHost(reinterpret_cast<void**>(&m->host_stage), 2 * sizeof(float)) != cudaSuccess)
    return cleanup(fail(ORCA_CUDA_ERROR, "pinned host allocation failed"));
  m->use_head = L >= 2 && C <= HEAD_MAX_CLASSES && m->gemm_path != GEMM_SIMT;
  // Without the fused classifier pass, the classifier's dW and dX products
  // take dlogits as an operand; split into planes they can run on the tensor
  // cores (plain fp32 would send them to the FFMA kernels).
  if (!m->use_head) ALLOC(dlogit_planes, (size_t)(2 * B * C) * 4);
  if (m->use_head) {
    const int64_t H = m->dims[L - 1];
    m->head_ldp = (C + 3) / 4 * 4;
    const int64_t fwd = cdiv(H, DOT_SLICE) * B * m->head_ldp;
    const int64_t bwd = head_part_floats(B, H, (int)C);
    ALLOC(head_part, (size_t)std::max(fwd, bwd) * 4);
    ALLOC(head_w, (size_t)H * 16 * 4);
  }
#undef ALLOC
  for (int l = 0; l < 64; ++l) m->ev_layer[l] = m->ev_reduced[l] = nullptr;
  for (int l = 0; l < L; ++l)
    if (cudaEventCreateWithFlags(&m->ev_layer[l], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&m->ev_reduced[l], cudaEventDisableTiming) != cudaSuccess)
      return cleanup(fail(ORCA_CUDA_ERROR, "event creation failed"));
  if (sync_stream(ctx) != ORCA_OK) return cleanup(ORCA_CUDA_ERROR);
  *out = m;
  return ORCA_OK;
}

orca_status orca_mlp_destroy(orca_mlp* m) {
  if (!m) return ORCA_OK;
  cudaSetDevice(m->ctx->device);
  sync_stream_for(m->ctx, m->ctx->stream, m->ctx->sync_timeout_s);
  sync_stream_for(m->ctx, m->ctx->comm_stream, m->ctx->sync_timeout_s);
  if (m->copy_stream) {
    sync_stream_for(m->ctx, m->copy_stream, m->ctx->sync_timeout_s);
    cudaStreamDestroy(m->copy_stream);
  }
  for (int i = 0; i < ORCA_MLP_STAGE_SLOTS; ++i) {
    if (m->ev_staged[i]) cudaEventDestroy(m->ev_staged[i]);
    if (m->ev_consumed[i]) cudaEventDestroy(m->ev_consumed[i]);
  }
  if (m->graph_exec) cudaGraphExecDestroy(m->graph_exec);
  if (m->pex) peer_arena_close(m->pex);   // before the arena it maps is freed
  for (void* p : m->allocs) cudaFree(p);
  if (m->host_stage) cudaFreeHost(m->host_stage);
  for (int l = 0; l < 64; ++l)
    if (m->ev_layer[l]) cudaEventDestroy(m->ev_layer[l]);
  for (int l = 0; l < 64; ++l)
    if (m->ev_reduced[l]) cudaEventDestroy(m->ev_reduced[l]);
  for (auto& r : m->recs) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
  for (auto e : m->event_pool) cudaEventDestroy(e);
  orca_ctx* ctx = m->ctx;
  delete m;
  ctx_release(ctx);
  return ORCA_OK;
}

orca_status orca_mlp_num_params(const orca_mlp* m, int* count) {
  if (!m || !count) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  *count = 2 * m->L;
  return ORCA_OK;
}

orca_status orca_mlp_param_numel(const orca_mlp* m, int index, int64_t* numel) {
  if (!m || !numel || index < 0 || index >= 2 * m->L)
    return fail(ORCA_INVALID_ARGUMENT, "bad parameter index");
  const int l = index / 2;
  *numel = (index % 2 == 0) ? m->dims[l] * m->dims[l + 1] : m->dims[l + 1];
  return ORCA_OK;
}

orca_status orca_mlp_set_param(orca_mlp* m, int index, const float* host, int64_t numel) {
  int64_t n;
  ORCA_TRY(orca_mlp_param_numel(m, index, &n));
  if (n != numel || !host) return fail(ORCA_SHAPE_MISMATCH, "set_param: %lld elements expected",
                                       (long long)n);
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  const int l = index / 2;
  if (index % 2 == 0) {
    // Stage through the gradient arena slot of this parameter, then split.
    ORCA_CUDA_TRY(cudaMemcpyAsync(m->grads + m->p_off[index], host, (size_t)n * 4,
                                  cudaMemcpyHostToDevice, m->ctx->stream));
    ORCA_TRY(split_planes(m->ctx, m->grads + m->p_off[index], m->w_hi[l], m->w_lo[l], n));
  } else {
    ORCA_CUDA_TRY(cudaMemcpyAsync(m->bias[l], host, (size_t)n * 4, cudaMemcpyHostToDevice,
                                  m->ctx->stream));
  }
  ORCA_TRY(finish_sync(m));
  return ORCA_OK;
}

orca_status orca_mlp_get_param(orca_mlp* m, int index, float* host, int64_t numel) {
  int64_t n;
  ORCA_TRY(orca_mlp_param_numel(m, index, &n));
  if (n != numel || !host) return fail(ORCA_SHAPE_MISMATCH, "get_param: %lld elements expected",
                                       (long long)n);
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  const int l = index / 2;
  if (index % 2 == 0) {
    float* tmp = nullptr;
    ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&tmp), (size_t)n * 4, m->ctx->stream));
    merge_planes_kernel<<<ew_grid(m->ctx, n), 256, 0, m->ctx->stream>>>(m->w_hi[l], m->w_lo[l],
                                                                        tmp, n);
    count_launch(m->ctx);
    orca_status st = finish_sync(m);
    if (st == ORCA_OK) st = copy_to_host(m->ctx, host, tmp, (size_t)n * 4);
    cudaFreeAsync(tmp, m->ctx->stream);
    ORCA_TRY(st);
  } else {
    ORCA_TRY(finish_sync(m));
    ORCA_TRY(copy_to_host(m->ctx, host, m->bias[l], (size_t)n * 4));
  }
  return check_device_error(m->ctx);
}

orca_status orca_mlp_get_activation(orca_mlp* m, int layer, float* host, int64_t numel) {
  if (!m || !host) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (layer < 1 || layer >= m->L)
    return fail(ORCA_INVALID_ARGUMENT, "layer %d: hidden activations are layers 1..%d", layer,
                m->L - 1);
  const int64_t n = m->B * m->dims[layer];
  if (numel != n)
    return fail(ORCA_SHAPE_MISMATCH, "get_activation: %lld elements expected", (long long)n);
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  float* tmp = nullptr;
  ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&tmp), (size_t)n * 4, m->ctx->stream));
  merge_planes_kernel<<<ew_grid(m->ctx, n), 256, 0, m->ctx->stream>>>(
      m->act_planes[layer], m->act_planes[layer] + n, tmp, n);
  count_launch(m->ctx);
  orca_status st = finish_sync(m);
  if (st == ORCA_OK) st = copy_to_host(m->ctx, host, tmp, (size_t)n * 4);
  cudaFreeAsync(tmp, m->ctx->stream);
  ORCA_TRY(st);
  return check_device_error(m->ctx);
}

orca_status orca_mlp_get_grad(orca_mlp* m, int index, float* host, int64_t numel) {
  int64_t n;
  ORCA_TRY(orca_mlp_param_numel(m, index, &n));
  if (n != numel || !host) return fail(ORCA_SHAPE_MISMATCH, "get_grad: size");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  ORCA_TRY(finish_sync(m));
  ORCA_TRY(copy_to_host(m->ctx, host, m->grads + m->p_off[index], (size_t)n * 4));
  return check_device_error(m->ctx);
}

orca_status orca_mlp_state_numel(const orca_mlp* m, int slot, int index, int64_t* numel) {
  if (!m || !numel || slot < 0 || slot > 1) return fail(ORCA_INVALID_ARGUMENT, "bad state slot");
  int64_t n;
  ORCA_TRY(orca_mlp_param_numel(m, index, &n));
  const float* base = slot == 0 ? m->state0 : m->state1;
  *numel = base ? n : 0;
  return ORCA_OK;
}

orca_status orca_mlp_get_state(orca_mlp* m, int slot, int index, float* host, int64_t numel) {
  int64_t n;
  ORCA_TRY(orca_mlp_state_numel(m, slot, index, &n));
  if (n == 0 || n != numel || !host) return fail(ORCA_SHAPE_MISMATCH, "get_state: size");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  const float* base = slot == 0 ? m->state0 : m->state1;
  ORCA_TRY(finish_sync(m));
  ORCA_TRY(copy_to_host(m->ctx, host, base + m->p_off[index], (size_t)n * 4));
  return check_device_error(m->ctx);
}

orca_status orca_mlp_set_state(orca_mlp* m, int slot, int index, const float* host,
                               int64_t numel) {
  int64_t n;
  ORCA_TRY(orca_mlp_state_numel(m, slot, index, &n));
  if (n == 0 || n != numel || !host) return fail(ORCA_SHAPE_MISMATCH, "set_state: size");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  float* base = slot == 0 ? m->state0 : m->state1;
  ORCA_TRY(finish_sync(m));
  ORCA_CUDA_TRY(cudaMemcpyAsync(base + m->p_off[index], host, (size_t)n * 4,
                                cudaMemcpyHostToDevice, m->ctx->stream));
  return finish_sync(m);
}

orca_status orca_mlp_get_step(const orca_mlp* m, int64_t* t, int* velocity_started) {
  if (!m || !t || !velocity_started) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  *t = m->t;
  *velocity_started = m->vel_init ? 1 : 0;
  return ORCA_OK;
}

orca_status orca_mlp_set_step(orca_mlp* m, int64_t t, int velocity_started) {
  if (!m || t < 0) return fail(ORCA_INVALID_ARGUMENT, "bad step count");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  m->t = t;
  m->vel_init = velocity_started != 0;
  return ORCA_OK;
}

orca_status orca_mlp_bucket_plan(int n_layers, const int64_t* dims, size_t bucket_bytes,
                                 int capacity, int64_t* offsets, int64_t* counts, int* layers,
                                 int* n_buckets) {
  if (!dims || !n_buckets) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (n_layers < 1 || n_layers > 60) return fail(ORCA_INVALID_ARGUMENT, "n_layers");
  for (int i = 0; i <= n_layers; ++i)
    if (dims[i] < 1) return fail(ORCA_INVALID_ARGUMENT, "dims must be positive");
  std::vector<Bucket> plan;
  bucket_plan(n_layers, dims, bucket_bytes, plan);
  *n_buckets = (int)plan.size();
  if (!offsets && !counts && !layers) return ORCA_OK;
  if (capacity < (int)plan.size())
    return fail(ORCA_INVALID_ARGUMENT, "capacity %d < %d buckets", capacity, (int)plan.size());
  for (size_t i = 0; i < plan.size(); ++i) {
    if (offsets) offsets[i] = plan[i].offset;
    if (counts) counts[i] = plan[i].count;
    if (layers) layers[i] = plan[i].layer;
  }
  return ORCA_OK;
}

// Whether AUTO takes the peer exchange when it can be set up.
constexpr bool kAutoPeer = true;
// ORCA_XCHG=nccl|peer overrides the automatic choice (for measurements).
static int xchg_env() {
  static const int v = [] {
    const char* e = getenv("ORCA_XCHG");
    if (e && strcmp(e, "nccl") == 0) return (int)ORCA_XCHG_NCCL;
    if (e && strcmp(e, "peer") == 0) return (int)ORCA_XCHG_PEER;
    return (int)ORCA_XCHG_AUTO;
  }();
  return v;
}

orca_status orca_mlp_set_exchange(orca_mlp* m, int mode) {
  if (!m) return fail(ORCA_INVALID_ARGUMENT, "null mlp");
  if (mode < ORCA_XCHG_AUTO || mode > ORCA_XCHG_PEER)
    return fail(ORCA_INVALID_ARGUMENT, "exchange mode %d", mode);
  if (m->comm) return fail(ORCA_INVALID_ARGUMENT, "set the exchange before attaching a communicator");
  m->xchg_mode = mode;
  return ORCA_OK;
}

orca_status orca_mlp_exchange_kind(const orca_mlp* m, int* kind) {
  if (!m || !kind) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  *kind = !m->comm ? 0 : (m->pex ? (int)ORCA_XCHG_PEER : (int)ORCA_XCHG_NCCL);
  return ORCA_OK;
}

orca_status orca_mlp_attach_comm(orca_mlp* m, orca_comm* comm, size_t bucket_bytes) {
  if (!m) return fail(ORCA_INVALID_ARGUMENT, "null mlp");
  if (m->pex) {
    // No exchange of the old communicator may still be running.
    ORCA_TRY(sync_stream_for(m->ctx, m->ctx->comm_stream, m->ctx->sync_timeout_s));
    ORCA_TRY(sync_stream_for(m->ctx, m->ctx->stream, m->ctx->sync_timeout_s));
    peer_arena_close(m->pex);
    m->pex = nullptr;
  }
  m->comm = comm;
  m->bucket_bytes = bucket_bytes;
  m->pex_seq = 0;
  if (!comm) return ORCA_OK;
  const int env = xchg_env();
  const int mode = env != ORCA_XCHG_AUTO ? env : m->xchg_mode;
  if (mode == ORCA_XCHG_NCCL || (mode == ORCA_XCHG_AUTO && !kAutoPeer)) return ORCA_OK;
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  ORCA_TRY(sync_stream_for(m->ctx, m->ctx->stream, m->ctx->sync_timeout_s));
  // Every rank opens (collective: the IPC handles travel through the
  // communicator), so every rank must request the same mode.
  const orca_status s = peer_arena_open(comm, m->grads, m->L, &m->pex);
  if (s != ORCA_OK && mode == ORCA_XCHG_PEER) {
    m->comm = nullptr;
    return s;
  }
  return ORCA_OK;   // AUTO: NCCL when the peer mapping is unavailable
}

// One step on device inputs.  inputs_read (nullable) is recorded on the
// compute stream once x_dev and t_dev have been read (the input split and the
// target copy come first), after which their buffers may be overwritten.
static orca_status step_device_locked(orca_mlp* m, const float* x_dev, const float* t_dev,
                                      float* loss_dev, cudaEvent_t inputs_read = nullptr) {
  orca_ctx* ctx = m->ctx;
  const uint64_t l0 = ctx->launches.load();
  const int64_t B = m->B, C = m->dims[m->L];
  const int pr = prof_open(m, "split_input", 0.0, 12.0 * B * m->dims[0]);
  ORCA_TRY(split_input(m, x_dev));
  prof_close(m, pr);
  if (t_dev != m->t_buf)
    ORCA_CUDA_TRY(cudaMemcpyAsync(m->t_buf, t_dev, (size_t)(B * C) * 4, cudaMemcpyDeviceToDevice,
                                  ctx->stream));
  if (inputs_read) ORCA_CUDA_TRY(cudaEventRecord(inputs_read, ctx->stream));
  ORCA_TRY(mlp_forward_impl(m, true));
  ORCA_TRY(mlp_backward_impl(m));
  ORCA_TRY(mlp_update_impl(m));
  if (loss_dev && loss_dev != m->loss)
    ORCA_CUDA_TRY(cudaMemcpyAsync(loss_dev, m->loss, 4, cudaMemcpyDeviceToDevice, ctx->stream));
  m->last_launches = (int)(ctx->launches.load() - l0);
  return ORCA_OK;
}

orca_status orca_mlp_step_device(orca_mlp* m, const float* x_dev, const float* t_dev,
                                 float* loss_dev) {
  if (!m || !x_dev || !t_dev) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  return step_device_locked(m, x_dev, t_dev, loss_dev);
}

orca_status orca_mlp_graph_capture(orca_mlp* m, const float* x_dev, const float* t_dev,
                                   float* loss_dev) {
  if (!m || !x_dev || !t_dev) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (m->opt != ORCA_OPT_SGD)
    return fail(ORCA_NOT_IMPLEMENTED, "graph capture: SGD only (AdamW's per-step constants)");
  if (m->comm) return fail(ORCA_INVALID_ARGUMENT, "graph capture: detach the communicator");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  if (m->profiling) return fail(ORCA_INVALID_ARGUMENT, "graph capture: profiling is on");
  orca_ctx* ctx = m->ctx;
  if (m->graph_exec) {
    cudaGraphExecDestroy(m->graph_exec);
    m->graph_exec = nullptr;
  }
  // The first momentum step differs (v = g); capture a steady-state step.  The
  // ordinary step also performs every one-time set-up (kernel attributes,
  // cluster occupancy) outside the capture.
  if (!m->vel_init) ORCA_TRY(step_device_locked(m, x_dev, t_dev, loss_dev));
  ORCA_TRY(sync_stream(ctx));
  const uint64_t l0 = ctx->launches.load();
  ORCA_CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  const orca_status s = step_device_locked(m, x_dev, t_dev, loss_dev);
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  const int launches = (int)(ctx->launches.load() - l0);
  ctx->launches -= (uint64_t)launches;      // captured, not run
  if (s != ORCA_OK) {
    if (graph) cudaGraphDestroy(graph);
    return s;
  }
  if (e != cudaSuccess || !graph)
    return fail(ORCA_CUDA_ERROR, "graph capture failed: %s", cudaGetErrorString(e));
  const cudaError_t ei = cudaGraphInstantiate(&m->graph_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess) {
    m->graph_exec = nullptr;
    return fail(ORCA_CUDA_ERROR, "graph instantiation failed: %s", cudaGetErrorString(ei));
  }
  m->graph_launches = launches;
  return ORCA_OK;
}

orca_status orca_mlp_graph_replay(orca_mlp* m) {
  if (!m) return fail(ORCA_INVALID_ARGUMENT, "null mlp");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  if (!m->graph_exec) return fail(ORCA_INVALID_ARGUMENT, "no captured step");
  if (m->comm) return fail(ORCA_INVALID_ARGUMENT, "graph replay: a communicator is attached");
  ORCA_CUDA_TRY(cudaGraphLaunch(m->graph_exec, m->ctx->stream));
  count_launch(m->ctx, (uint64_t)m->graph_launches);
  m->last_launches = m->graph_launches;
  return ORCA_OK;
}

orca_status orca_mlp_graph_release(orca_mlp* m) {
  if (!m) return ORCA_OK;
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  if (m->graph_exec) {
    ORCA_TRY(sync_stream(m->ctx));
    cudaGraphExecDestroy(m->graph_exec);
    m->graph_exec = nullptr;
  }
  return ORCA_OK;
}

// Loss and the device error word come back through pinned memory (the copies
// do not block), then one bounded wait covers the whole step.
static orca_status read_loss_locked(orca_mlp* m, float* loss) {
  orca_ctx* ctx = m->ctx;
  ORCA_CUDA_TRY(cudaMemcpyAsync(&m->host_stage[0], m->loss, 4, cudaMemcpyDeviceToHost,
                                ctx->stream));
  ORCA_CUDA_TRY(cudaMemcpyAsync(&m->host_stage[1], ctx->dev_err, 4, cudaMemcpyDeviceToHost,
                                ctx->stream));
  ORCA_TRY(finish_sync(m));
  *loss = m->host_stage[0];
  int h;
  memcpy(&h, &m->host_stage[1], sizeof(int));
  if (h != DEV_OK) return check_device_error(ctx);   // clears the word, maps the code
  return ORCA_OK;
}

orca_status orca_mlp_step(orca_mlp* m, const float* x, const float* t, float* loss) {
  if (!m || !x || !t) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  orca_ctx* ctx = m->ctx;
  const int64_t B = m->B, C = m->dims[m->L];
  ORCA_CUDA_TRY(cudaMemcpyAsync(m->x_stage, x, (size_t)(B * m->dims[0]) * 4,
                                cudaMemcpyHostToDevice, ctx->stream));
  ORCA_CUDA_TRY(cudaMemcpyAsync(m->t_buf, t, (size_t)(B * C) * 4, cudaMemcpyHostToDevice,
                                ctx->stream));
  ORCA_TRY(step_device_locked(m, m->x_stage, m->t_buf, nullptr));
  if (loss) return read_loss_locked(m, loss);
  return ORCA_OK;
}

// Memory type of a host pointer: 1 page-locked, 0 pageable, -1 device or
// managed memory (refused).
static int host_memory_kind(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (a.type == cudaMemoryTypeHost) return 1;
  if (a.type == cudaMemoryTypeUnregistered) return 0;
  return -1;
}

static orca_status ensure_staging(orca_mlp* m) {
  if (m->copy_stream) return ORCA_OK;
  const size_t xb = (size_t)(m->B * m->dims[0]) * 4, tb = (size_t)(m->B * m->dims[m->L]) * 4;
  for (int i = 0; i < ORCA_MLP_STAGE_SLOTS; ++i) {
    if (!m->ev_staged[i])
      ORCA_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_staged[i], cudaEventDisableTiming));
    if (!m->ev_consumed[i])
      ORCA_CUDA_TRY(cudaEventCreateWithFlags(&m->ev_consumed[i], cudaEventDisableTiming));
    if (m->slot_x[i]) continue;
    void* p = nullptr;
    if (cudaMalloc(&p, xb + tb) != cudaSuccess) {
      cudaGetLastError();
      return fail(ORCA_CUDA_ERROR, "staging slot allocation (%zu bytes) failed", xb + tb);
    }
    m->allocs.push_back(p);
    m->slot_x[i] = static_cast<float*>(p);
    m->slot_t[i] = reinterpret_cast<float*>(static_cast<char*>(p) + xb);
  }
  ORCA_CUDA_TRY(cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking));
  return ORCA_OK;
}

orca_status orca_mlp_stage_batch(orca_mlp* m, int slot, const float* x, const float* t) {
  if (!m || !x || !t) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (slot < 0 || slot >= ORCA_MLP_STAGE_SLOTS)
    return fail(ORCA_INVALID_ARGUMENT, "slot must be in [0, %d)", ORCA_MLP_STAGE_SLOTS);
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  orca_ctx* ctx = m->ctx;
  const int kx = host_memory_kind(x), kt = host_memory_kind(t);
  if (kx < 0 || kt < 0)
    return fail(ORCA_INVALID_ARGUMENT, "stage_batch takes host memory (use orca_mlp_step_device)");
  ORCA_TRY(ensure_staging(m));
  if (kx == 1 && kt == 1) {
    // Fully asynchronous: the copy waits on the device until the slot's last
    // step has read it.
    ORCA_CUDA_TRY(cudaStreamWaitEvent(m->copy_stream, m->ev_consumed[slot], 0));
  } else {
    // A pageable copy waits, on the host and without a bound, for the copy
    // stream's earlier work: make both waits bounded first.
    ORCA_TRY(wait_event_for(m->ev_consumed[slot], ctx->sync_timeout_s));
    ORCA_TRY(sync_stream_for(ctx, m->copy_stream, ctx->sync_timeout_s));
  }
  const size_t xb = (size_t)(m->B * m->dims[0]) * 4, tb = (size_t)(m->B * m->dims[m->L]) * 4;
  ORCA_CUDA_TRY(cudaMemcpyAsync(m->slot_x[slot], x, xb, cudaMemcpyHostToDevice, m->copy_stream));
  ORCA_CUDA_TRY(cudaMemcpyAsync(m->slot_t[slot], t, tb, cudaMemcpyHostToDevice, m->copy_stream));
  ORCA_CUDA_TRY(cudaEventRecord(m->ev_staged[slot], m->copy_stream));
  m->slot_ready[slot] = true;
  return ORCA_OK;
}

orca_status orca_mlp_step_staged(orca_mlp* m, int slot, float* loss) {
  if (!m) return fail(ORCA_INVALID_ARGUMENT, "null mlp");
  if (slot < 0 || slot >= ORCA_MLP_STAGE_SLOTS)
    return fail(ORCA_INVALID_ARGUMENT, "slot must be in [0, %d)", ORCA_MLP_STAGE_SLOTS);
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  if (!m->slot_ready[slot])
    return fail(ORCA_INVALID_ARGUMENT, "slot %d holds no staged batch", slot);
  ORCA_CUDA_TRY(cudaStreamWaitEvent(m->ctx->stream, m->ev_staged[slot], 0));
  m->slot_ready[slot] = false;
  ORCA_TRY(step_device_locked(m, m->slot_x[slot], m->slot_t[slot], nullptr,
                              m->ev_consumed[slot]));
  if (loss) return read_loss_locked(m, loss);
  return ORCA_OK;
}

orca_status orca_mlp_forward(orca_mlp* m, const float* x, const float* t, float* logits,
                             float* loss) {
  if (!m || !x) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  orca_ctx* ctx = m->ctx;
  const int64_t B = m->B, C = m->dims[m->L];
  ORCA_CUDA_TRY(cudaMemcpyAsync(m->x_stage, x, (size_t)(B * m->dims[0]) * 4,
                                cudaMemcpyHostToDevice, ctx->stream));
  ORCA_TRY(split_input(m, m->x_stage));
  if (t) {
    ORCA_CUDA_TRY(cudaMemcpyAsync(m->t_buf, t, (size_t)(B * C) * 4, cudaMemcpyHostToDevice,
                                  ctx->stream));
  }
  ORCA_TRY(mlp_forward_impl(m, false));
  if (t) {
    launch_ce_rows(ctx->stream, m->logits, m->t_buf, B, C, 1.0f / (float)B, nullptr,
                   m->row_loss);
    ce_loss_kernel<<<1, CE_LOSS_THREADS, 0, ctx->stream>>>(m->row_loss, B, 1.0f / (float)B, m->loss);
    count_launch(ctx, 2);
  }
  ORCA_TRY(finish_sync(m));
  if (logits) ORCA_TRY(copy_to_host(ctx, logits, m->logits, (size_t)(B * C) * 4));
  if (loss && t) ORCA_TRY(copy_to_host(ctx, loss, m->loss, 4));
  return check_device_error(ctx);
}

orca_status orca_mlp_profile_begin(orca_mlp* m) {
  if (!m) return fail(ORCA_INVALID_ARGUMENT, "null mlp");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  m->profiling = true;
  for (auto& s : m->sites) { s.ms = 0; s.count = 0; }
  return ORCA_OK;
}

orca_status orca_mlp_profile_end(orca_mlp* m, int* n_sites) {
  if (!m || !n_sites) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  ORCA_TRY(check_ctx(m->ctx));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  m->profiling = false;
  ORCA_TRY(finish_sync(m));
  for (auto& r : m->recs) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      m->sites[r.site].ms += ms;
      m->sites[r.site].count += 1;
    }
    m->event_pool.push_back(r.a);
    m->event_pool.push_back(r.b);
  }
  m->recs.clear();
  *n_sites = (int)m->sites.size();
  return ORCA_OK;
}

orca_status orca_mlp_profile_site(const orca_mlp* m, int i, const char** name, double* ms_total,
                                  int* launches, double* flops_per_launch,
                                  double* bytes_per_launch, int* gemm_path) {
  if (!m || i < 0 || i >= (int)m->sites.size()) return fail(ORCA_INVALID_ARGUMENT, "bad site");
  const auto& s = m->sites[i];
  if (name) *name = s.name.c_str();
  if (ms_total) *ms_total = s.ms;
  if (launches) *launches = s.count;
  if (flops_per_launch) *flops_per_launch = s.flops;
  if (bytes_per_launch) *bytes_per_launch = s.bytes;
  if (gemm_path) *gemm_path = s.gemm_path;
  return ORCA_OK;
}

orca_status orca_mlp_launches_per_step(const orca_mlp* m, int* count) {
  if (!m || !count) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  *count = m->last_launches;
  return ORCA_OK;
}

}  // extern "C"

// Forward: activations as planes; logits plain.  with_loss_grad also runs the
// fused CE forward+backward into loss / dlogits.
static orca_status mlp_forward_impl(orca_mlp* m, bool with_loss_grad) {
  orca_ctx* ctx = m->ctx;
  const int L = m->L;
  const int64_t B = m->B, C = m->dims[L];
  for (int l = 0; l < L; ++l) {
    const int64_t K = m->dims[l], N = m->dims[l + 1];
    Operand a, w;
    a.hi = l == 0 ? m->x_planes : m->act_planes[l];
    a.ld = l == 0 ? m->x_ld : K;
    a.lo = a.hi + B * a.ld;
    a.mn_major = false;
    w.hi = m->w_hi[l];
    w.lo = m->w_lo[l];
    w.ld = N;
    w.mn_major = true;
    Epilogue ep;
    ep.bias = m->bias[l];
    if (l + 1 < L) {
      ep.mode = EPI_BIAS_RELU_SPLIT;
      ep.out = m->act_planes[l + 1];
      ep.out_lo = ep.out + B * N;
      ep.ldc = N;
    } else {
      ep.mode = EPI_BIAS;
      ep.out = m->logits;
      ep.ldc = N;
    }
    bool fused_head = false;
    if (m->use_head && l == L - 2) {
      // The classifier layer's product rides on this GEMM's epilogue when it
      // takes the tensor cores.
      Epilogue ed = ep;
      ed.dot_w = m->head_w;
      ed.dot_n = (int)C;
      ed.dot_out = m->head_part;
      ed.dot_ldp = m->head_ldp;
      if (gemm_select(ctx, B, N, K, a, w, ed, m->gemm_path) == GEMM_TC) {
        ep = ed;
        fused_head = true;
        ORCA_TRY(head_pack_weights(ctx, m->w_hi[L - 1], m->w_lo[L - 1], N, (int)C, m->head_w));
      }
    }
    const int path = gemm_select(ctx, B, N, K, a, w, ep, m->gemm_path);
    // The ReLU decisions as bits for the dX product of layer l + 1 (not for
    // the classifier pass, which reads the activation itself).
    if (l + 1 < L) {
      // ORCA_RELU_BITS=0 keeps the dX masks on the activation planes.
      static const bool bits_on = [] {
        const char* e = getenv("ORCA_RELU_BITS");
        return !(e && e[0] == '0');
      }();
      const bool bits = bits_on && path == GEMM_TC && !(m->use_head && l + 1 == L - 1);
      ep.relu_bits_out = bits ? m->relu_bits[l + 1] : nullptr;
      ep.bits_ld = cdiv(N, 32);
      m->relu_bits_ok[l + 1] = bits ? 1 : 0;
    }
    const int pr = prof_open(m, "gemm_fwd_l" + std::to_string(l), 2.0 * B * N * K,
                             4.0 * (2 * B * K + 2 * K * N + (l + 1 < L ? 2 : 1) * B * N), path);
    ORCA_TRY(gemm(ctx, B, N, K, a, w, ep, m->gemm_path, m->workspace, m->workspace_bytes));
    prof_close(m, pr);
    if (fused_head) {
      const int ph = prof_open(m, "head_logits", 2.0 * B * N * C,
                               4.0 * (cdiv(N, DOT_SLICE) * B * m->head_ldp + B * C + C));
      ORCA_TRY(head_logits(ctx, m->head_part, cdiv(N, DOT_SLICE), B, (int)C, m->head_ldp,
                           m->bias[L - 1], m->logits));
      prof_close(m, ph);
      break;   // the classifier layer is done
    }
  }
  if (with_loss_grad) {
    const int pr = prof_open(m, "softmax_ce", 0.0, 4.0 * (3 * B * C + B));
    launch_ce_rows(ctx->stream, m->logits, m->t_buf, B, C, 1.0f / (float)B, m->dlogits,
                   m->row_loss);
    ce_loss_kernel<<<1, CE_LOSS_THREADS, 0, ctx->stream>>>(m->row_loss, B, 1.0f / (float)B, m->loss);
    count_launch(ctx, 2);
    prof_close(m, pr);
    ORCA_CUDA_TRY(cudaGetLastError());
  }
  return ORCA_OK;
}

// SMs left to a gradient all-reduce during the dX GEMM that follows it, and
// the share of that GEMM's tiles run on the remaining SMs (ORCA_COMM_SMS,
// ORCA_COMM_SPLIT).  Off by default: measured at 2 GPUs, giving
// the all-reduce 16 or 24 SMs made the GEMM 0.3-0.55 ms slower while the
// all-reduce, contending for memory with it, still took 1.4-2.1 ms; the step
// was 1.5-3 % slower than with the GEMM on every SM.
//
// With the peer exchange the reservation is on by default (ORCA_PEER_SMS,
// 16): its kernel moves a layer's gradients at close to NVLink speed from a
// handful of SMs, so the layer-1 exchange finishes inside the first part of
// the dX GEMM.  (It cannot share an SM with a GEMM CTA: the GEMM's ten warps
// at 168 registers leave too few registers on the scheduler partitions.)
struct CommOverlap {
  int reserve_sms;
  double first_fraction;
};
static CommOverlap comm_overlap(bool peer) {
  static const CommOverlap v[2] = {
      [] {
        CommOverlap o{0, 0.5};
        if (const char* e = getenv("ORCA_COMM_SMS")) o.reserve_sms = std::max(0, atoi(e));
        if (const char* e = getenv("ORCA_COMM_SPLIT")) {
          const double f = atof(e);
          if (f > 0.0 && f < 1.0) o.first_fraction = f;
        }
        return o;
      }(),
      [] {
        CommOverlap o{16, 0.5};
        if (const char* e = getenv("ORCA_PEER_SMS")) o.reserve_sms = std::max(0, atoi(e));
        if (const char* e = getenv("ORCA_COMM_SPLIT")) {
          const double f = atof(e);
          if (f > 0.0 && f < 1.0) o.first_fraction = f;
        }
        return o;
      }()};
  return v[peer ? 1 : 0];
}

static orca_status launch_layer_allreduce(orca_mlp* m, int l) {
  orca_ctx* ctx = m->ctx;
  ORCA_CUDA_TRY(cudaEventRecord(m->ev_layer[l], ctx->stream));
  ORCA_CUDA_TRY(cudaStreamWaitEvent(ctx->comm_stream, m->ev_layer[l], 0));
  if (m->pex) {
    // The whole layer in one exchange (its kernel runs beside the GEMMs).
    const int64_t n = m->dims[l] * m->dims[l + 1] + m->dims[l + 1];
    const int pr = prof_open(m, "allreduce_l" + std::to_string(l), 0.0, 4.0 * (double)n, -1,
                             ctx->comm_stream);
    // Layers whose exchange overlaps a GEMM run on the SMs the GEMM leaves
    // free; the first layer's runs after the last GEMM, on every SM.
    const int sms = l > 0 ? comm_overlap(true).reserve_sms : 0;
    ORCA_TRY(peer_arena_allreduce_avg(m->pex, l, m->p_off[2 * l], n, m->pex_seq,
                                      ctx->comm_stream, sms));
    prof_close(m, pr);
    ORCA_CUDA_TRY(cudaEventRecord(m->ev_reduced[l], ctx->comm_stream));
    return ORCA_OK;
  }
  std::vector<Bucket> plan;
  bucket_plan(m->L, m->dims.data(), m->bucket_bytes, plan);
  // Timed on the comm stream: from the layer's gradients being ready to
  // their average being complete (includes waiting for SMs).
  const int64_t n = m->dims[l] * m->dims[l + 1] + m->dims[l + 1];
  const int pr = prof_open(m, "allreduce_l" + std::to_string(l), 0.0, 4.0 * (double)n, -1,
                           ctx->comm_stream);
  for (const Bucket& b : plan) {
    if (b.layer != l) continue;
    ORCA_TRY(comm_allreduce_avg_stream(m->comm, m->grads + b.offset, (size_t)b.count,
                                       ctx->comm_stream));
  }
  prof_close(m, pr);
  ORCA_CUDA_TRY(cudaEventRecord(m->ev_reduced[l], ctx->comm_stream));
  return ORCA_OK;
}

static orca_status mlp_backward_impl(orca_mlp* m) {
  orca_ctx* ctx = m->ctx;
  const int L = m->L;
  const int64_t B = m->B;
  if (m->pex) ++m->pex_seq;
  // g: gradient w.r.t. the current layer's pre-activation output.
  const float* g_hi = m->dlogits;
  const float* g_lo = nullptr;
  int64_t g_ld = m->dims[L];
  if (m->dlogit_planes) {
    // hi + lo == dlogits exactly, so every path computes the same products.
    const int64_t n = B * m->dims[L];
    const int pr = prof_open(m, "split_dlogits", 0.0, 12.0 * n);
    ORCA_TRY(split_planes(ctx, m->dlogits, m->dlogit_planes, m->dlogit_planes + n, n));
    prof_close(m, pr);
    g_hi = m->dlogit_planes;
    g_lo = m->dlogit_planes + n;
  }
  int cur = 0;
  for (int l = L - 1; l >= 0; --l) {
    const int64_t K = m->dims[l], N = m->dims[l + 1];
    // db = sum over the batch (ExpandBackward -> sum_to_shape [B,N] -> [1,N]).
    int pr = -1;
    // The classifier pass already summed the dZ of layer L - 2, and layer 0's
    // bias gradient comes out of its dW product (the input's column of ones).
    if (!(m->use_head && l == L - 2) && l != 0) {
      pr = prof_open(m, "colsum_l" + std::to_string(l), (double)B * N,
                     4.0 * ((g_lo ? 2 : 1) * B * N + N));
      ORCA_TRY(colsum(ctx, g_hi, g_lo, B, N, g_ld, m->grads + m->p_off[2 * l + 1],
                      m->colsum_part));
      prof_close(m, pr);
    }
    if (m->use_head && l == L - 1) {
      // dW and dX of the classifier layer in one pass over its input.
      pr = prof_open(m, "head_bwd_l" + std::to_string(l), 4.0 * B * N * K,
                     4.0 * (2 * B * K + B * N + 2 * K * N + 2 * B * K + K * N));
      // ... and the bias gradient of layer l - 1 (the column sums of its dZ).
      ORCA_TRY(head_backward(ctx, B, K, (int)N, g_hi, m->act_planes[l], m->act_planes[l] + B * K,
                             m->w_hi[l], m->w_lo[l], m->dz[cur], m->dz[cur] + B * K,
                             m->head_part, m->grads + m->p_off[2 * l],
                             m->grads + m->p_off[2 * (l - 1) + 1]));
      prof_close(m, pr);
      if (m->comm) ORCA_TRY(launch_layer_allreduce(m, l));
      g_hi = m->dz[cur];
      g_lo = m->dz[cur] + B * K;
      g_ld = K;
      cur ^= 1;
      continue;
    }
    // dW = act^T @ g : M = K (features), N, K_gemm = B.  For layer 0 the
    // input planes carry a column of ones after the K features, so the
    // product has K + 1 rows and its last row, sum_m g[m, :], is db0 -- which
    // the arena stores right after dW0.
    Operand at, g;
    at.hi = l == 0 ? m->x_planes : m->act_planes[l];
    at.ld = l == 0 ? m->x_ld : K;
    at.lo = at.hi + B * at.ld;
    at.mn_major = true;
    const int64_t dw_rows = l == 0 ? K + 1 : K;
    g.hi = g_hi;
    g.lo = g_lo;
    g.ld = g_ld;
    g.mn_major = true;
    Epilogue ew;
    ew.mode = EPI_STORE;
    ew.out = m->grads + m->p_off[2 * l];
    ew.ldc = N;
    pr = prof_open(m, "gemm_dw_l" + std::to_string(l), 2.0 * B * N * K,
                   4.0 * (2 * B * K + (g_lo ? 2 : 1) * B * N + K * N),
                   gemm_select(ctx, dw_rows, N, B, at, g, ew, m->gemm_path));
    ORCA_TRY(gemm(ctx, dw_rows, N, B, at, g, ew, m->gemm_path, m->workspace,
                  m->workspace_bytes));
    prof_close(m, pr);
    if (m->comm) ORCA_TRY(launch_layer_allreduce(m, l));
    if (l == 0) break;
    // dX = g @ W^T, masked by the ReLU of the layer input (> 0), split.
    Operand ga, wt;
    ga.hi = g_hi;
    ga.lo = g_lo;
    ga.ld = g_ld;
    ga.mn_major = false;
    wt.hi = m->w_hi[l];
    wt.lo = m->w_lo[l];
    wt.ld = N;
    wt.mn_major = false;
    Epilogue ex;
    ex.mode = EPI_MASK_SPLIT;
    ex.out = m->dz[cur];
    ex.out_lo = m->dz[cur] + B * K;
    ex.ldc = K;
    ex.mask_hi = m->act_planes[l];
    ex.mask_lo = m->act_planes[l] + B * K;
    const int dx_path = gemm_select(ctx, B, K, N, ga, wt, ex, m->gemm_path);
    if (dx_path == GEMM_TC && m->relu_bits_ok[l]) {
      ex.relu_bits = m->relu_bits[l];
      ex.bits_ld = cdiv(K, 32);
    }
    // Bytes: g, W (both planes), the mask (planes or bits) and dZ (planes).
    const double mask_bytes = ex.relu_bits ? 4.0 * B * cdiv(K, 32) : 8.0 * B * K;
    pr = prof_open(m, "gemm_dx_l" + std::to_string(l), 2.0 * B * N * K,
                   4.0 * ((g_lo ? 2 : 1) * B * N + 2 * K * N + 2 * B * K) + mask_bytes, dx_path);
    const CommOverlap ov = comm_overlap(m->pex != nullptr);
    if (m->comm && dx_path == GEMM_TC && ov.reserve_sms > 0 && ov.reserve_sms < ctx->sm_count) {
      // This layer's gradient all-reduce was just queued on the comm stream.
      // The persistent GEMM would take every SM before the collective's CTAs
      // are dispatched, so its first part runs on fewer CTAs and leaves
      // reserve_sms SMs to the all-reduce; the rest runs on all SMs.
      const int64_t tiles = gemm_tc_tiles(B, K);
      TileRange first, rest;
      first.end = (int64_t)(ov.first_fraction * (double)tiles);
      first.max_ctas = ctx->sm_count - ov.reserve_sms;
      rest.begin = first.end;
      ORCA_TRY(gemm(ctx, B, K, N, ga, wt, ex, m->gemm_path, m->workspace, m->workspace_bytes,
                    &first));
      ORCA_TRY(gemm(ctx, B, K, N, ga, wt, ex, m->gemm_path, m->workspace, m->workspace_bytes,
                    &rest));
    } else {
      ORCA_TRY(gemm(ctx, B, K, N, ga, wt, ex, m->gemm_path, m->workspace, m->workspace_bytes));
    }
    prof_close(m, pr);
    g_hi = ex.out;
    g_lo = ex.out_lo;
    g_ld = K;
    cur ^= 1;
  }
  // With a communicator the optimizer waits per layer (mlp_update_impl), so
  // the update of the layers reduced first overlaps the last all-reduce.
  return ORCA_OK;
}

static orca_status mlp_update_impl(orca_mlp* m) {
  orca_ctx* ctx = m->ctx;
  const int L = m->L;
  if (m->opt == ORCA_OPT_ADAMW) m->t += 1;
  // Algorithmic bytes per parameter: SGD reads p, g and writes p (12 B);
  // momentum adds v read + write (20 B); AdamW reads p, g, m, v, writes p, m, v (28 B).
  const double bpp = m->opt == ORCA_OPT_ADAMW ? 28.0 : (m->mom != 0.0 ? 20.0 : 12.0);
  const int pr = prof_open(m, "optimizer", 0.0, bpp * (double)m->n_params);
  // Last layer first: that is the order the backward pass (and the gradient
  // all-reduce) finishes the layers in.  Each parameter's update is
  // independent, so the order does not change any result.
  for (int l = L - 1; l >= 0; --l) {
    const int64_t K = m->dims[l], N = m->dims[l + 1];
    if (m->comm) ORCA_CUDA_TRY(cudaStreamWaitEvent(ctx->stream, m->ev_reduced[l], 0));
    for (int which = 0; which < 2; ++which) {
      const int idx = 2 * l + which;
      const int64_t n = which == 0 ? K * N : N;
      float* hi = which == 0 ? m->w_hi[l] : m->bias[l];
      float* lo = which == 0 ? m->w_lo[l] : nullptr;
      const float* g = m->grads + m->p_off[idx];
      if (m->opt == ORCA_OPT_SGD) {
        float* v = m->state0 ? m->state0 + m->p_off[idx] : nullptr;
        launch_sgd(ctx, hi, lo, g, v, n,
                   sgd_args(m->lr, m->mom, m->damp, m->wd, m->vel_init ? 0 : 1));
      } else {
        launch_adamw(ctx, hi, lo, g, m->state0 + m->p_off[idx], m->state1 + m->p_off[idx], n,
                     adam_args(m->lr, m->b1, m->b2, m->eps, m->wd, m->t));
      }
    }
  }
  prof_close(m, pr);
  m->vel_init = true;
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

// =============================================================== fused ops on buffers
extern "C" {

orca_status orca_linear_fwd(orca_ctx* ctx, const orca_buf* x, const orca_buf* w, const orca_buf* b,
                            int64_t m, int64_t k, int64_t n, int relu, orca_buf** out) {
  ORCA_TRY(check_ctx(ctx));
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!x || !w || !out) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (x->n < (size_t)(m * k) || w->n < (size_t)(k * n) || (b && b->n < (size_t)n))
    return fail(ORCA_SHAPE_MISMATCH, "linear_fwd: buffer sizes");
  ORCA_TRY(new_buf(ctx, (size_t)(m * n), ORCA_F32, out));
  float* scratch = nullptr;
  const size_t elems = 2 * (size_t)(m * k) + 2 * (size_t)(k * n) + (relu ? 2 * (size_t)(m * n) : 0) +
                       (b ? 0 : (size_t)n);
  ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&scratch), elems * 4, ctx->stream));
  float* xh = scratch;
  float* wh = xh + 2 * m * k;
  float* oh = wh + 2 * k * n;
  float* zb = relu ? oh + 2 * m * n : oh;
  ORCA_TRY(split_planes(ctx, (const float*)x->ptr, xh, xh + m * k, m * k));
  ORCA_TRY(split_planes(ctx, (const float*)w->ptr, wh, wh + k * n, k * n));
  const float* bias = (const float*)(b ? b->ptr : nullptr);
  if (!b) {
    ORCA_CUDA_TRY(cudaMemsetAsync(zb, 0, (size_t)n * 4, ctx->stream));
    bias = zb;
  }
  Operand oa, ob;
  oa.hi = xh; oa.lo = xh + m * k; oa.ld = k;
  ob.hi = wh; ob.lo = wh + k * n; ob.ld = n; ob.mn_major = true;
  Epilogue ep;
  ep.bias = bias;
  ep.ldc = n;
  if (relu) {
    ep.mode = EPI_BIAS_RELU_SPLIT;
    ep.out = oh;
    ep.out_lo = oh + m * n;
  } else {
    ep.mode = EPI_BIAS;
    ep.out = (float*)(*out)->ptr;
  }
  orca_status s = gemm(ctx, m, n, k, oa, ob, ep, GEMM_AUTO);
  if (s == ORCA_OK && relu) {
    merge_planes_kernel<<<ew_grid(ctx, m * n), 256, 0, ctx->stream>>>(oh, oh + m * n,
                                                                      (float*)(*out)->ptr, m * n);
    count_launch(ctx);
  }
  cudaFreeAsync(scratch, ctx->stream);
  return s;
}

orca_status orca_linear_bwd(orca_ctx* ctx, const orca_buf* x, const orca_buf* w, const orca_buf* dy,
                            const orca_buf* mask, int64_t m, int64_t k, int64_t n, orca_buf** dx,
                            orca_buf** dw, orca_buf** db) {
  ORCA_TRY(check_ctx(ctx));
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!x || !w || !dy || !dw || !db) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (m < 1 || k < 1 || n < 1) return fail(ORCA_INVALID_ARGUMENT, "linear_bwd: empty shape");
  if (x->n < (size_t)(m * k) || w->n < (size_t)(k * n) || dy->n < (size_t)(m * n) ||
      (mask && mask->n < (size_t)(m * k)))
    return fail(ORCA_SHAPE_MISMATCH, "linear_bwd: buffer sizes");
  for (const orca_buf* b : {x, w, dy, mask})
    if (b && b->dtype != ORCA_F32) return fail(ORCA_UNSUPPORTED_DTYPE, "linear_bwd: F32 only");
  if (dx) *dx = nullptr;
  *dw = *db = nullptr;
  ORCA_TRY(new_buf(ctx, (size_t)(k * n), ORCA_F32, dw));
  orca_status s = new_buf(ctx, (size_t)n, ORCA_F32, db);
  if (s == ORCA_OK && dx) s = new_buf(ctx, (size_t)(m * k), ORCA_F32, dx);
  float* scratch = nullptr;
  const size_t elems = 2 * (size_t)(m * k) + 2 * (size_t)(k * n) + 2 * (size_t)(m * n) +
                       (size_t)(cdiv(m, COLSUM_ROWS) * n);
  if (s == ORCA_OK &&
      cudaMallocAsync(reinterpret_cast<void**>(&scratch), elems * 4, ctx->stream) != cudaSuccess)
    s = fail(ORCA_CUDA_ERROR, "linear_bwd: scratch allocation failed");
  if (s == ORCA_OK) {
    float* xh = scratch;
    float* wh = xh + 2 * m * k;
    float* gh = wh + 2 * k * n;
    float* part = gh + 2 * m * n;
    s = split_planes(ctx, (const float*)x->ptr, xh, xh + m * k, m * k);
    if (s == ORCA_OK) s = split_planes(ctx, (const float*)w->ptr, wh, wh + k * n, k * n);
    if (s == ORCA_OK) s = split_planes(ctx, (const float*)dy->ptr, gh, gh + m * n, m * n);
    // dW = x^T dy (MatMulBackward, orca-autograd/src/backend.rs:1448-1499).
    Operand at, g;
    at.hi = xh; at.lo = xh + m * k; at.ld = k; at.mn_major = true;
    g.hi = gh; g.lo = gh + m * n; g.ld = n; g.mn_major = true;
    Epilogue ew;
    ew.mode = EPI_STORE;
    ew.out = (float*)(*dw)->ptr;
    ew.ldc = n;
    if (s == ORCA_OK) s = gemm(ctx, k, n, m, at, g, ew, GEMM_AUTO);
    // db = sum over rows of dy (ExpandBackward -> sum_to_shape, backend.rs:1675-1698).
    if (s == ORCA_OK) s = colsum(ctx, (const float*)dy->ptr, nullptr, m, n, n,
                                 (float*)(*db)->ptr, part);
    if (s == ORCA_OK && dx) {
      // dX = dy W^T, then the ReLU mask of the layer below (ReluBackward,
      // backend.rs:1624-1646: the gradient passes where the input was > 0).
      Operand ga, wt;
      ga.hi = gh; ga.lo = gh + m * n; ga.ld = n;
      wt.hi = wh; wt.lo = wh + k * n; wt.ld = n;
      Epilogue ex;
      ex.mode = EPI_STORE;
      ex.out = (float*)(*dx)->ptr;
      ex.ldc = k;
      s = gemm(ctx, m, k, n, ga, wt, ex, GEMM_AUTO);
      if (s == ORCA_OK && mask) {
        mask_kernel<<<ew_grid(ctx, m * k), 256, 0, ctx->stream>>>(
            (float*)(*dx)->ptr, (const float*)mask->ptr, m * k);
        count_launch(ctx);
        if (cudaGetLastError() != cudaSuccess) s = fail(ORCA_CUDA_ERROR, "linear_bwd: mask");
      }
    }
    cudaFreeAsync(scratch, ctx->stream);
  }
  if (s != ORCA_OK) {
    for (orca_buf** o : {dx, dw, db})
      if (o && *o) {
        orca_buf_release(*o);
        *o = nullptr;
      }
  }
  return s;
}

orca_status orca_softmax_ce_fwd_bwd(orca_ctx* ctx, const orca_buf* logits, const orca_buf* target,
                                    int64_t batch, int64_t classes, orca_buf** loss,
                                    orca_buf** dlogits) {
  ORCA_TRY(check_ctx(ctx));
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!logits || !target || !loss) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (batch < 1 || classes < 1) return fail(ORCA_INVALID_ARGUMENT, "empty batch");
  if (logits->n < (size_t)(batch * classes) || target->n < (size_t)(batch * classes))
    return fail(ORCA_SHAPE_MISMATCH, "softmax_ce: buffer sizes");
  ORCA_TRY(new_buf(ctx, 1, ORCA_F32, loss));
  float* dp = nullptr;
  if (dlogits) {
    ORCA_TRY(new_buf(ctx, (size_t)(batch * classes), ORCA_F32, dlogits));
    dp = (float*)(*dlogits)->ptr;
  }
  float* rows = nullptr;
  ORCA_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&rows), (size_t)batch * 4, ctx->stream));
  const float inv_b = 1.0f / (float)batch;
  launch_ce_rows(ctx->stream, (const float*)logits->ptr, (const float*)target->ptr, batch,
                 classes, inv_b, dp, rows);
  ce_loss_kernel<<<1, CE_LOSS_THREADS, 0, ctx->stream>>>(rows, batch, inv_b, (float*)(*loss)->ptr);
  count_launch(ctx, 2);
  cudaFreeAsync(rows, ctx->stream);
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

// ---- softmax-CE without allocation ------------------------------------------
// Row losses of orca_softmax_ce_fwd_bwd_noalloc live in this fixed device
// array instead of a per-call allocation.  Every GPU that loads the library
// holds it until the process exits.  Host code must not hand the symbol
// itself to a kernel (on the host it is only a stand-in for the device
// array); its device address is looked up once per device when a context is
// created on that device (orca_ctx_create, device current), so the entry
// point itself makes no runtime look-up.
}  // extern "C"

namespace orca {
constexpr int64_t kCeScratchRows = int64_t(1) << 20;   // 4 MiB of f32 row losses
static __device__ __align__(256) float g_ce_row_scratch[kCeScratchRows];
constexpr int kMaxDevices = 128;
static std::atomic<float*> g_ce_scratch_addr[kMaxDevices] = {};   // per device, set once
static std::mutex g_ce_scratch_mu;

// Called by orca_ctx_create with `device` current.  Idempotent.
orca_status ce_scratch_setup(int device) {
  if (device < 0 || device >= kMaxDevices)
    return fail(ORCA_INVALID_ARGUMENT, "device index %d", device);
  std::lock_guard<std::mutex> lk(g_ce_scratch_mu);
  if (g_ce_scratch_addr[device].load()) return ORCA_OK;
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_ce_row_scratch);
  if (e != cudaSuccess || !ptr) {
    (void)cudaGetLastError();   // not sticky: keep it from failing a later, unrelated check
    return fail(ORCA_CUDA_ERROR, "cudaGetSymbolAddress(row-loss scratch) failed: %s",
                cudaGetErrorString(e));
  }
  g_ce_scratch_addr[device].store(static_cast<float*>(ptr));
  return ORCA_OK;
}
}  // namespace orca

extern "C" {

orca_status orca_softmax_ce_fwd_bwd_noalloc(orca_ctx* ctx, const float* logits,
                                            const float* target, int64_t batch, int64_t classes,
                                            float* loss, float* dlogits) {
  ORCA_TRY(check_ctx(ctx));   // makes ctx->device current
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!logits || !target || !loss) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (batch < 1 || classes < 1) return fail(ORCA_INVALID_ARGUMENT, "empty batch");
  if (batch > kCeScratchRows)
    return fail(ORCA_INVALID_ARGUMENT,
                "batch %lld exceeds the %lld rows of the fixed no-allocation scratch; "
                "use orca_softmax_ce_fwd_bwd for larger batches",
                (long long)batch, (long long)kCeScratchRows);
  float* rows = ctx->device < kMaxDevices ? g_ce_scratch_addr[ctx->device].load() : nullptr;
  if (!rows)
    return fail(ORCA_INTERNAL, "the no-allocation scratch of device %d was not set up when "
                "its context was created", ctx->device);
  // Every row of the scratch that ce_loss_kernel reads is written first by
  // ce_kernel on the same stream, so nothing needs clearing between calls.
  const float inv_b = 1.0f / (float)batch;
  launch_ce_rows(ctx->stream, logits, target, batch, classes, inv_b, dlogits, rows);
  ce_loss_kernel<<<1, CE_LOSS_THREADS, 0, ctx->stream>>>(rows, batch, inv_b, loss);
  count_launch(ctx, 2);
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

orca_status orca_sgd_step(orca_ctx* ctx, orca_buf* p, const orca_buf* g, orca_buf* v, double lr,
                          double momentum, double dampening, double weight_decay, int first) {
  ORCA_TRY(check_ctx(ctx));
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!p || !g) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (g->n != p->n || (v && v->n != p->n)) return fail(ORCA_SHAPE_MISMATCH, "sgd_step: sizes");
  if (momentum != 0.0 && !v) return fail(ORCA_INVALID_ARGUMENT, "sgd_step: momentum needs v");
  const int64_t n = (int64_t)p->n;
  launch_sgd(ctx, (float*)p->ptr, nullptr, (const float*)g->ptr, v ? (float*)v->ptr : nullptr, n,
             sgd_args(lr, momentum, dampening, weight_decay, first));
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

orca_status orca_adamw_step(orca_ctx* ctx, orca_buf* p, const orca_buf* g, orca_buf* m,
                            orca_buf* v, double lr, double beta1, double beta2, double eps,
                            double weight_decay, int64_t t) {
  ORCA_TRY(check_ctx(ctx));
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (!p || !g || !m || !v) return fail(ORCA_INVALID_ARGUMENT, "null argument");
  if (g->n != p->n || m->n != p->n || v->n != p->n)
    return fail(ORCA_SHAPE_MISMATCH, "adamw_step: sizes");
  if (t < 1) return fail(ORCA_INVALID_ARGUMENT, "adamw_step: t starts at 1");
  const int64_t n = (int64_t)p->n;
  launch_adamw(ctx, (float*)p->ptr, nullptr, (const float*)g->ptr, (float*)m->ptr,
               (float*)v->ptr, n, adam_args(lr, beta1, beta2, eps, weight_decay, t));
  ORCA_CUDA_TRY(cudaGetLastError());
  return ORCA_OK;
}

}  // extern "C"
