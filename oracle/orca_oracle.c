/*
 * orca_oracle.c -- CPU restatement of Orca's FP32 MLP training path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker, never the product); see
 * orca_oracle.h for scope.  Every function names the reference lines it
 * restates.  Build: oracle/Makefile (-O3 -ffp-contract=off -fopenmp).
 */
#include "orca_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;

void oc_set_threads(int n) {
  g_threads = n;
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#endif
}

int oc_get_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

/* Element-wise loops: the reference runs these as rayon par_iter maps
 * (orca-backend-cpu/src/backend.rs:118-125 and siblings); each element is an
 * independent single rounding, so threading does not change any bit. */
#define EW_LOOP(n) _Pragma("omp parallel for schedule(static) if((n) > 65536)") \
  for (int64_t i = 0; i < (n); ++i)

void oc_add(const float* a, const float* b, float* out, int64_t n) { EW_LOOP(n) out[i] = a[i] + b[i]; }
void oc_sub(const float* a, const float* b, float* out, int64_t n) { EW_LOOP(n) out[i] = a[i] - b[i]; }
void oc_mul(const float* a, const float* b, float* out, int64_t n) { EW_LOOP(n) out[i] = a[i] * b[i]; }
void oc_div(const float* a, const float* b, float* out, int64_t n) { EW_LOOP(n) out[i] = a[i] / b[i]; }
void oc_mul_scalar(const float* a, float s, float* out, int64_t n) { EW_LOOP(n) out[i] = a[i] * s; }
/* `if val > 0 { val } else { 0 }` (backend.rs:384-386): NaN maps to 0. */
void oc_relu(const float* a, float* out, int64_t n) { EW_LOOP(n) out[i] = a[i] > 0.0f ? a[i] : 0.0f; }
/* 1/(1+exp(-x)) in f32 (backend.rs:406-408). */
void oc_sigmoid(const float* a, float* out, int64_t n) {
  EW_LOOP(n) out[i] = 1.0f / (1.0f + expf(-a[i]));
}
void oc_exp(const float* a, float* out, int64_t n) { EW_LOOP(n) out[i] = expf(a[i]); }
/* ln(max(x, 1e-7)) (backend.rs:577). */
void oc_log(const float* a, float* out, int64_t n) { EW_LOOP(n) out[i] = logf(fmaxf(a[i], 1e-7f)); }
void oc_sqrt(const float* a, float* out, int64_t n) { EW_LOOP(n) out[i] = sqrtf(a[i]); }
/* grad if x > 0 else 0, with x the ReLU INPUT primal (backend.rs:432-434). */
void oc_relu_backward(const float* g, const float* x, float* out, int64_t n) {
  EW_LOOP(n) out[i] = x[i] > 0.0f ? g[i] : 0.0f;
}
/* g * y * (1 - y) (backend.rs:458-460). */
void oc_sigmoid_backward(const float* g, const float* y, float* out, int64_t n) {
  EW_LOOP(n) out[i] = (g[i] * y[i]) * (1.0f - y[i]);
}
void oc_exp_backward(const float* g, const float* y, float* out, int64_t n) { EW_LOOP(n) out[i] = g[i] * y[i]; }
/* g / x, no clamp (backend.rs:629). */
void oc_log_backward(const float* g, const float* x, float* out, int64_t n) { EW_LOOP(n) out[i] = g[i] / x[i]; }
/* g / (2 y) (backend.rs:755). */
void oc_sqrt_backward(const float* g, const float* y, float* out, int64_t n) {
  EW_LOOP(n) out[i] = g[i] / (2.0f * y[i]);
}
void oc_div_backward_lhs(const float* g, const float* r, float* out, int64_t n) { EW_LOOP(n) out[i] = g[i] / r[i]; }
/* g * (-l / (r*r)) (backend.rs:727). */
void oc_div_backward_rhs(const float* g, const float* l, const float* r, float* out, int64_t n) {
  EW_LOOP(n) out[i] = g[i] * (-l[i] / (r[i] * r[i]));
}
/* Serial lhs + rhs (backend.rs:761-774). */
void oc_accumulate_grad(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* ---- shape helpers: backend.rs:17-49 --------------------------------------- */
#define OC_MAX_RANK 16

static int64_t numel(const int64_t* s, int r) {
  int64_t n = 1;
  for (int i = 0; i < r; ++i) n *= s[i];
  return n;
}

/* pad_shape_left (backend.rs:17-26): left-pad with ones to target rank; a
 * longer shape yields all ones, as in the reference. */
static void pad_left(const int64_t* s, int r, int target, int64_t* out) {
  for (int i = 0; i < target; ++i) out[i] = 1;
  if (r <= target)
    for (int i = 0; i < r; ++i) out[target - r + i] = s[i];
}

static void strides_of(const int64_t* s, int r, int64_t* st) {
  int64_t cur = 1;
  for (int i = r - 1; i >= 0; --i) { st[i] = cur; cur *= s[i]; }
}

/* expand (backend.rs:466-497): out[i] = in[map(i)] with broadcast dims
 * (size 1 after left padding) pinned to index 0. */
int oc_expand(const float* in, const int64_t* in_shape, int in_rank,
              float* out, const int64_t* out_shape, int out_rank) {
  if (in_rank > OC_MAX_RANK || out_rank > OC_MAX_RANK) return -1;
  int64_t padded[OC_MAX_RANK], in_st[OC_MAX_RANK];
  pad_left(in_shape, in_rank, out_rank, padded);
  strides_of(padded, out_rank, in_st);
  int64_t n = numel(out_shape, out_rank);
  for (int64_t i = 0; i < n; ++i) {
    int64_t rem = i, idx = 0;
    for (int d = out_rank - 1; d >= 0; --d) {
      int64_t c = rem % out_shape[d];
      rem /= out_shape[d];
      if (padded[d] != 1) idx += c * in_st[d];
    }
    out[i] = in[idx];
  }
  return 0;
}

/* sum_to_shape (backend.rs:499-530): out starts at 0 and every input element
 * is added to its target in ascending linear input order (serial f32). */
int oc_sum_to_shape(const float* in, const int64_t* in_shape, int in_rank,
                    float* out, const int64_t* out_shape, int out_rank) {
  if (in_rank > OC_MAX_RANK || out_rank > OC_MAX_RANK) return -1;
  int64_t padded[OC_MAX_RANK], out_st[OC_MAX_RANK];
  pad_left(out_shape, out_rank, in_rank, padded);
  strides_of(padded, in_rank, out_st);
  int64_t n_out = numel(out_shape, out_rank), n_in = numel(in_shape, in_rank);
  for (int64_t i = 0; i < n_out; ++i) out[i] = 0.0f;
  for (int64_t i = 0; i < n_in; ++i) {
    int64_t rem = i, idx = 0;
    for (int d = in_rank - 1; d >= 0; --d) {
      int64_t c = rem % in_shape[d];
      rem /= in_shape[d];
      if (padded[d] != 1) idx += c * out_st[d];
    }
    out[idx] = out[idx] + in[i];
  }
  return 0;
}

/* max_to_shape (backend.rs:1336-1381): init f32::MIN, strict `>` update. */
int oc_max_to_shape(const float* in, const int64_t* in_shape, int in_rank,
                    float* out, const int64_t* out_shape, int out_rank) {
  if (in_rank > OC_MAX_RANK || out_rank > OC_MAX_RANK) return -1;
  int64_t padded[OC_MAX_RANK], out_st[OC_MAX_RANK];
  if (out_rank < in_rank) pad_left(out_shape, out_rank, in_rank, padded);
  else for (int i = 0; i < out_rank; ++i) padded[i] = out_shape[i];
  int pr = out_rank < in_rank ? in_rank : out_rank;
  strides_of(padded, pr, out_st);
  int64_t n_out = numel(out_shape, out_rank), n_in = numel(in_shape, in_rank);
  for (int64_t i = 0; i < n_out; ++i) out[i] = -FLT_MAX;
  for (int64_t i = 0; i < n_in; ++i) {
    int64_t rem = i, idx = 0;
    for (int d = in_rank - 1; d >= 0; --d) {
      int64_t c = rem % in_shape[d];
      rem /= in_shape[d];
      if (padded[d] != 1) idx += c * out_st[d];
    }
    if (in[i] > out[idx]) out[idx] = in[i];
  }
  return 0;
}

/* max_to_shape_backward (backend.rs:1383-1435): every input equal to its
 * group's max receives 0 + grad_out (ties all receive it). */
int oc_max_to_shape_backward(const float* g, const float* in_primal,
                             const float* out_primal,
                             const int64_t* in_shape, int in_rank,
                             const int64_t* out_shape, int out_rank,
                             float* grad_in) {
  if (in_rank > OC_MAX_RANK || out_rank > OC_MAX_RANK) return -1;
  int64_t padded[OC_MAX_RANK], out_st[OC_MAX_RANK];
  if (out_rank < in_rank) pad_left(out_shape, out_rank, in_rank, padded);
  else for (int i = 0; i < out_rank; ++i) padded[i] = out_shape[i];
  int pr = out_rank < in_rank ? in_rank : out_rank;
  strides_of(padded, pr, out_st);
  int64_t n_in = numel(in_shape, in_rank);
  for (int64_t i = 0; i < n_in; ++i) {
    int64_t rem = i, idx = 0;
    for (int d = in_rank - 1; d >= 0; --d) {
      int64_t c = rem % in_shape[d];
      rem /= in_shape[d];
      if (padded[d] != 1) idx += c * out_st[d];
    }
    grad_in[i] = 0.0f;
    if (in_primal[i] == out_primal[idx]) grad_in[i] = 0.0f + g[idx];
  }
  return 0;
}

/* transpose (backend.rs:223-289): materialised copy with dims swapped. */
int oc_transpose(const float* in, const int64_t* shape, int rank, int dim0, int dim1, float* out) {
  if (rank > OC_MAX_RANK || dim0 < 0 || dim1 < 0 || dim0 >= rank || dim1 >= rank) return -1;
  int64_t oshape[OC_MAX_RANK], in_st[OC_MAX_RANK], out_st[OC_MAX_RANK];
  for (int i = 0; i < rank; ++i) oshape[i] = shape[i];
  int64_t tmp = oshape[dim0]; oshape[dim0] = oshape[dim1]; oshape[dim1] = tmp;
  strides_of(shape, rank, in_st);
  strides_of(oshape, rank, out_st);
  int64_t n = numel(shape, rank);
  for (int64_t o = 0; o < n; ++o) {
    int64_t cur = o, idx = 0;
    for (int i = 0; i < rank; ++i) {
      int64_t c = cur / out_st[i];
      cur %= out_st[i];
      int od = i == dim0 ? dim1 : (i == dim1 ? dim0 : i);
      idx += c * in_st[od];
    }
    out[o] = in[idx];
  }
  return 0;
}

/* Single-threaded GEMM, as the reference's `matrixmultiply::sgemm` built with
 * default features (orca-backend-cpu/Cargo.toml:11; call backend.rs:197-212).
 * Each C element is ((0 + a0*b0) + a1*b1) + ... with k ascending; the i-k-j
 * blocking only changes memory order, never the per-element summation order. */
__attribute__((target_clones("avx2", "default")))
static void gemm_block(const float* A, const float* B, float* C, int64_t m,
                       int64_t k, int64_t n) {
  const int64_t NB = 512, KB = 128;
  for (int64_t jj = 0; jj < n; jj += NB) {
    int64_t jn = n - jj < NB ? n - jj : NB;
    for (int64_t kk = 0; kk < k; kk += KB) {
      int64_t kn = k - kk < KB ? k - kk : KB;
      for (int64_t i = 0; i < m; ++i) {
        float* c = C + i * n + jj;
        const float* a = A + i * k + kk;
        for (int64_t q = 0; q < kn; ++q) {
          const float av = a[q];
          const float* b = B + (kk + q) * n + jj;
          for (int64_t j = 0; j < jn; ++j) c[j] = c[j] + av * b[j];
        }
      }
    }
  }
}

/* Alternative, equally valid FP32 summation orders -- used only to measure
 * how sensitive a training trajectory is to the (unpinned) summation order of
 * the reference's GEMM.  0: k ascending, separate multiply and add (default);
 * 1: k ascending with fused multiply-add; 2: partial sums over k-blocks of
 * 256, then added in block order; 3: exact product rounded once (f64);
 * 4: the packed FMA kernel of sgemm_packed.c (timing stand-in for the
 * reference's matrixmultiply; falls back to order 0 without AVX2/FMA). */
static int g_gemm_order = 0;
void oc_set_gemm_order(int order) { g_gemm_order = order; }

static void gemm_variant(const float* A, const float* B, float* C, int64_t m, int64_t k, int64_t n) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      if (g_gemm_order == 1) {
        float acc = 0.0f;
        for (int64_t q = 0; q < k; ++q) acc = fmaf(A[i * k + q], B[q * n + j], acc);
        C[i * n + j] = acc;
      } else if (g_gemm_order == 2) {
        float acc = 0.0f;
        for (int64_t q0 = 0; q0 < k; q0 += 256) {
          float part = 0.0f;
          for (int64_t q = q0; q < k && q < q0 + 256; ++q) part = part + A[i * k + q] * B[q * n + j];
          acc = acc + part;
        }
        C[i * n + j] = acc;
      } else {
        double acc = 0.0;
        for (int64_t q = 0; q < k; ++q) acc += (double)A[i * k + q] * (double)B[q * n + j];
        C[i * n + j] = (float)acc;
      }
    }
}

/* Threads of the default-order GEMM (1 = the reference's single thread).
 * Rows are split between threads; every element keeps its k-ascending
 * chain, so the result is the same bit for bit at any thread count.  Tests
 * raise it to check wide layers in seconds; timed baselines keep 1. */
static int g_gemm_threads = 1;
void oc_set_gemm_threads(int n) { g_gemm_threads = n; }

int oc_sgemm_packed_mt(const float* A, const float* B, float* C, int64_t m, int64_t k, int64_t n,
                       int threads);

static void gemm_default(const float* A, const float* B, float* C, int64_t m, int64_t k,
                         int64_t n) {
  memset(C, 0, (size_t)(m * n) * sizeof(float));
#ifdef _OPENMP
  if (g_gemm_threads != 1 && m >= 16) {
    const int nt = g_gemm_threads > 0 ? g_gemm_threads : omp_get_max_threads();
    const int64_t rows = (m + nt - 1) / nt;
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int t = 0; t < nt; ++t) {
      const int64_t r0 = (int64_t)t * rows;
      if (r0 < m) {
        const int64_t rn = m - r0 < rows ? m - r0 : rows;
        gemm_block(A + r0 * k, B, C + r0 * n, rn, k, n);
      }
    }
    return;
  }
#endif
  gemm_block(A, B, C, m, k, n);
}

void oc_matmul(const float* a, const float* b, float* c, int64_t batch,
               int64_t m, int64_t k, int64_t n) {
  for (int64_t bi = 0; bi < batch; ++bi) {
    float* cb = c + bi * m * n;
    const float* ab = a + bi * m * k;
    const float* bb = b + bi * k * n;
    if (g_gemm_order == 4) {
#ifdef _OPENMP
      const int nt = g_gemm_threads > 0 ? g_gemm_threads : omp_get_max_threads();
#else
      const int nt = 1;
#endif
      if (oc_sgemm_packed_mt(ab, bb, cb, m, k, n, nt) == 0) continue;
    }
    if (g_gemm_order != 0 && g_gemm_order != 4) {
      gemm_variant(ab, bb, cb, m, k, n);
      continue;
    }
    gemm_default(ab, bb, cb, m, k, n);
  }
}

/* ---- softmax cross-entropy ---------------------------------------------------
 * Forward: python/orca/nn/loss.py:83-100 on top of max_to_shape, expand,
 * sub, exp, sum_to_shape, log (clamped), add, mul, __neg__ (= mul_scalar -1,
 * orca-python/src/lib.rs:642-658), sum_to_shape and mean (= sum * f32(1/numel),
 * lib.rs:664-669).
 * Backward: the 21 nodes that forward pushes, swept in reverse push order
 * (tape.rs:114) with the per-node rules of orca-autograd/src/backend.rs
 * (MulScalar 1565-1587, SumToShape 1701-1723, Mul 1590-1621, Expand 1675-1698,
 * Sub 1533-1562, Add 1380-1402, Log 1773-1793, Exp 1750-1770, MaxToShape
 * 1405-1433) and grads accumulated existing + new (tape.rs:34-47).  Expand
 * of a same-shape tensor contributes 0 + g (sum_to_shape to the same shape). */
void oc_softmax_ce(const float* P, const float* T, int64_t B, int64_t C, float* loss, float* dP) {
  const float invB = 1.0f / (float)B;
  float total = 0.0f;
  float* Mx = (float*)malloc(sizeof(float) * (size_t)B);
  float* Sx = (float*)malloc(sizeof(float) * (size_t)B);
  for (int64_t b = 0; b < B; ++b) {
    const float* p = P + b * C;
    const float* t = T + b * C;
    float m = -FLT_MAX;
    for (int64_t c = 0; c < C; ++c) if (p[c] > m) m = p[c];
    float s = 0.0f;
    for (int64_t c = 0; c < C; ++c) s = s + expf(p[c] - m);
    const float lse = m + logf(fmaxf(s, 1e-7f));
    float per = 0.0f;
    for (int64_t c = 0; c < C; ++c) {
      const float ls = p[c] - lse;
      const float tl = t[c] * ls;
      per = per + tl * -1.0f;
    }
    total = total + per;
    Mx[b] = m;
    Sx[b] = s;
  }
  *loss = total * invB;
  if (dP) {
    const float g_tl = invB * -1.0f;          /* MulScalar(-1) of g_NL = invB */
    for (int64_t b = 0; b < B; ++b) {
      const float* p = P + b * C;
      const float* t = T + b * C;
      float* d = dP + b * C;
      const float m = Mx[b], s = Sx[b];
      /* g_s0 = sum_c (g_LSE / Sx), g_LSE = 0 + (g_LS * -1), g_LS = 0 + g_tl*t */
      float g_s0 = 0.0f;
      for (int64_t c = 0; c < C; ++c) {
        const float g_ls = 0.0f + g_tl * t[c];
        const float g_lse = 0.0f + g_ls * -1.0f;
        const float g_lg = 0.0f + g_lse;
        g_s0 = g_s0 + g_lg / s;
      }
      /* grads[M] = (0 + g_LSE) + (0 + (g_S * -1)); g_m0 = sum_c grads[M] */
      float g_m0 = 0.0f;
      for (int64_t c = 0; c < C; ++c) {
        const float g_ls = 0.0f + g_tl * t[c];
        const float g_lse = 0.0f + g_ls * -1.0f;
        const float e = expf(p[c] - m);
        const float g_s = g_s0 * e;
        const float gm = (0.0f + g_lse) + (0.0f + g_s * -1.0f);
        g_m0 = g_m0 + gm;
        /* grads[P] = (0 + g_LS) + (0 + g_S), then + max-path term */
        d[c] = (0.0f + g_ls) + (0.0f + g_s);
      }
      for (int64_t c = 0; c < C; ++c) {
        const float gi = (p[c] == m) ? 0.0f + g_m0 : 0.0f;
        d[c] = d[c] + gi;
      }
    }
  }
  free(Mx);
  free(Sx);
}

/* ---- the composed MLP step ----------------------------------------------------
 * Forward: Sequential.forward (python/orca/nn/container.py:13-17) over
 * Linear.forward (linear.py:74-79: x @ W, then + bias.expand) and ReLU
 * (activation.py:21).  Backward per Linear, in reverse tape order: Add ->
 * Expand(bias) -> sum_to_shape([B,N] -> [1,N]) for db (ExpandBackward,
 * orca-autograd/src/backend.rs:1675-1698), then MatMulBackward (1448-1499):
 * dX = g @ transpose(W) (skipped for the input, which has no node id) and
 * dW = transpose(X) @ g; ReluBackward (1624-1646) uses the ReLU input. */
static int mlp_run(int L, const int64_t* dims, int64_t B, const float* const* W,
                   const float* const* bias, const float* x, const float* t,
                   float* loss, float* const* dW, float* const* db, float* logits) {
  if (L < 1 || B < 1) return -1;
  float** act = (float**)calloc((size_t)L + 1, sizeof(float*));  /* act[l] = input of layer l */
  float** pre = (float**)calloc((size_t)L, sizeof(float*));      /* pre[l] = Z + b */
  int rc = 0;
  act[0] = (float*)x;
  for (int l = 0; l < L; ++l) {
    const int64_t K = dims[l], N = dims[l + 1];
    float* z = (float*)malloc(sizeof(float) * (size_t)(B * N));
    oc_matmul(act[l], W[l], z, 1, B, K, N);
    for (int64_t i = 0; i < B; ++i)
      for (int64_t j = 0; j < N; ++j) z[i * N + j] = z[i * N + j] + bias[l][j];
    pre[l] = z;
    if (l + 1 < L) {
      float* a = (float*)malloc(sizeof(float) * (size_t)(B * N));
      oc_relu(z, a, B * N);
      act[l + 1] = a;
    }
  }
  const int64_t C = dims[L];
  if (logits) memcpy(logits, pre[L - 1], sizeof(float) * (size_t)(B * C));
  float* g = dW ? (float*)malloc(sizeof(float) * (size_t)(B * C)) : NULL;
  oc_softmax_ce(pre[L - 1], t, B, C, loss, g);
  if (dW) {
    for (int l = L - 1; l >= 0; --l) {
      const int64_t K = dims[l], N = dims[l + 1];
      /* db: sum_to_shape [B,N] -> [1,N], ascending rows per column */
      for (int64_t j = 0; j < N; ++j) db[l][j] = 0.0f;
      for (int64_t i = 0; i < B; ++i)
        for (int64_t j = 0; j < N; ++j) db[l][j] = db[l][j] + g[i * N + j];
      /* dX first (MatMulBackward handles lhs before rhs; independent values) */
      float* gprev = NULL;
      if (l > 0) {
        float* wt = (float*)malloc(sizeof(float) * (size_t)(K * N));
        int64_t ws[2] = {K, N};
        oc_transpose(W[l], ws, 2, 0, 1, wt);
        gprev = (float*)malloc(sizeof(float) * (size_t)(B * K));
        oc_matmul(g, wt, gprev, 1, B, N, K);
        free(wt);
        oc_relu_backward(gprev, pre[l - 1], gprev, B * K);
      }
      float* xt = (float*)malloc(sizeof(float) * (size_t)(B * K));
      int64_t xs[2] = {B, K};
      oc_transpose(act[l], xs, 2, 0, 1, xt);
      oc_matmul(xt, g, dW[l], 1, K, B, N);
      free(xt);
      free(g);
      g = gprev;
    }
  }
  for (int l = 1; l < L; ++l) free(act[l]);
  for (int l = 0; l < L; ++l) free(pre[l]);
  free(act);
  free(pre);
  return rc;
}

int oc_mlp_forward_backward(int n_layers, const int64_t* dims, int64_t batch,
                            const float* const* W, const float* const* b,
                            const float* x, const float* t, float* loss,
                            float* const* dW, float* const* db, float* logits) {
  if (!dW || !db) return -1;
  return mlp_run(n_layers, dims, batch, W, b, x, t, loss, dW, db, logits);
}

int oc_mlp_forward(int n_layers, const int64_t* dims, int64_t batch,
                   const float* const* W, const float* const* b, const float* x,
                   const float* t, float* loss, float* logits) {
  return mlp_run(n_layers, dims, batch, W, b, x, t, loss, NULL, NULL, logits);
}

/* ---- optimizers ----------------------------------------------------------------
 * Python floats reach Rust as f32 (Operand::Scalar(f32), orca-python/src/
 * lib.rs:13-16); compound constants are evaluated in Python double first. */

/* SGD.step (python/orca/optim/sgd.py:55-79). */
void oc_sgd_step(float* p, const float* g, float* v, int64_t n, double lr,
                 double momentum, double dampening, double weight_decay, int first) {
  const float f_lr = (float)lr, f_wd = (float)weight_decay, f_mom = (float)momentum;
  const float f_1md = (float)(1.0 - dampening);
  EW_LOOP(n) {
    float gi = g[i];
    if (weight_decay != 0.0) gi = gi + p[i] * f_wd;
    if (momentum != 0.0) {
      float vi;
      if (first) vi = gi;
      else if (dampening != 0.0) vi = v[i] * f_mom + gi * f_1md;
      else vi = v[i] * f_mom + gi;
      v[i] = vi;
      gi = vi;
    }
    const float upd = gi * f_lr;
    p[i] = p[i] - upd;
  }
}

/* AdamW.step (python/orca/optim/adamw.py:75-99). */
void oc_adamw_step(float* p, const float* g, float* m, float* v, int64_t n,
                   double lr, double beta1, double beta2, double eps,
                   double weight_decay, int64_t t) {
  const float c_decay = (float)(1.0 - lr * weight_decay);
  const float c_b1 = (float)beta1, c_1mb1 = (float)(1.0 - beta1);
  const float c_b2 = (float)beta2, c_1mb2 = (float)(1.0 - beta2);
  const float c_bc1 = (float)(1.0 / (1.0 - pow(beta1, (double)t)));
  const float c_bc2 = (float)(1.0 / (1.0 - pow(beta2, (double)t)));
  const float c_eps = (float)eps, c_lr = (float)lr;
  EW_LOOP(n) {
    const float gi = g[i];
    const float decayed = p[i] * c_decay;
    const float mi = m[i] * c_b1 + gi * c_1mb1;
    const float vi = v[i] * c_b2 + (gi * gi) * c_1mb2;
    m[i] = mi;
    v[i] = vi;
    const float mh = mi * c_bc1;
    const float vh = vi * c_bc2;
    const float denom = sqrtf(vh) + c_eps;
    const float upd = (mh / denom) * c_lr;
    p[i] = decayed - upd;
  }
}

/* DistributedDataParallel.all_reduce_gradients averaging
 * (python/orca/distributed.py:238-256): Python-float (f64) accumulation of
 * the f32 gradients, times f64 1/world, packed back to f32. */
void oc_ddp_average(const float* const* rank_grads, int world, int64_t n, float* out) {
  const double inv = 1.0 / (double)world;
  EW_LOOP(n) {
    double s = (double)rank_grads[0][i];
    for (int r = 1; r < world; ++r) s += (double)rank_grads[r][i];
    out[i] = (float)(s * inv);
  }
}
