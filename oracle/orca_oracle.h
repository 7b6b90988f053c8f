/*
 * orca_oracle.h -- CPU restatement of Orca's FP32 MLP training path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA
 * backend is compared against; it is never linked into, loaded by or called
 * from the product library (liborca_cuda.so) or its Python host code.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm use it.
 *
 * It restates two layers of the reference (cowoksoftspoken/orcaml):
 *   1. the primitive ops of the CPU backend
 *      (orca-backend-cpu/src/backend.rs), one C function per Backend-trait
 *      method that the MLP path reaches, with the same element order,
 *      accumulation order and special cases (log clamp, max ties, ...);
 *   2. the composition of those ops that the reference's Python frontend and
 *      tape autograd perform for one training step
 *      (python/orca/nn/{linear,activation,loss}.py, optim/{sgd,adamw}.py,
 *      distributed.py, orca-autograd/src/backend.rs backward nodes in the
 *      reverse push order of orca-autograd/src/tape.rs:107-118).
 *
 * All arithmetic is IEEE binary32 with one rounding per reference op; the
 * library is compiled with -ffp-contract=off so no multiply-add is fused.
 * The GEMM sums over k in ascending order per output element.  The
 * reference's GEMM comes from the third-party crate `matrixmultiply` 0.3
 * (not vendored, no Cargo.lock; call site orca-backend-cpu/src/backend.rs:
 * 197-212) whose blocking/FMA choice is not pinned, so GEMM results are
 * pinned only to the reference's small known-answer tests.
 */
#ifndef ORCA_ORACLE_H
#define ORCA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- primitive ops: orca-backend-cpu/src/backend.rs ---------------------- */
void oc_add(const float* a, const float* b, float* out, int64_t n);          /* :104-128 */
void oc_sub(const float* a, const float* b, float* out, int64_t n);          /* :291-315 */
void oc_mul(const float* a, const float* b, float* out, int64_t n);          /* :340-373 */
void oc_div(const float* a, const float* b, float* out, int64_t n);          /* :635-659 */
void oc_mul_scalar(const float* a, float s, float* out, int64_t n);          /* :317-338 */
void oc_relu(const float* a, float* out, int64_t n);                         /* :375-390 */
void oc_sigmoid(const float* a, float* out, int64_t n);                      /* :392-412 */
void oc_exp(const float* a, float* out, int64_t n);                          /* :549-564 */
void oc_log(const float* a, float* out, int64_t n);                          /* :566-581 */
void oc_sqrt(const float* a, float* out, int64_t n);                         /* :661-676 */
void oc_relu_backward(const float* g, const float* x, float* out, int64_t n);   /* :414-438 */
void oc_sigmoid_backward(const float* g, const float* y, float* out, int64_t n);/* :440-464 */
void oc_exp_backward(const float* g, const float* y, float* out, int64_t n);    /* :583-607 */
void oc_log_backward(const float* g, const float* x, float* out, int64_t n);    /* :609-633 */
void oc_sqrt_backward(const float* g, const float* y, float* out, int64_t n);   /* :734-759 */
void oc_div_backward_lhs(const float* g, const float* r, float* out, int64_t n);/* :678-701 */
void oc_div_backward_rhs(const float* g, const float* l, const float* r,
                         float* out, int64_t n);                               /* :703-731 */
void oc_accumulate_grad(const float* a, const float* b, float* out, int64_t n);/* :761-774 */
/* Shape ops return 0 on success, -1 on a rank/shape error. */
int oc_expand(const float* in, const int64_t* in_shape, int in_rank,
              float* out, const int64_t* out_shape, int out_rank);             /* :466-497 */
int oc_sum_to_shape(const float* in, const int64_t* in_shape, int in_rank,
                    float* out, const int64_t* out_shape, int out_rank);       /* :499-530 */
int oc_max_to_shape(const float* in, const int64_t* in_shape, int in_rank,
                    float* out, const int64_t* out_shape, int out_rank);       /* :1336-1381 */
int oc_max_to_shape_backward(const float* g, const float* in_primal,
                             const float* out_primal,
                             const int64_t* in_shape, int in_rank,
                             const int64_t* out_shape, int out_rank,
                             float* grad_in);                                  /* :1383-1435 */
int oc_transpose(const float* in, const int64_t* shape, int rank,
                 int dim0, int dim1, float* out);                              /* :223-289 */
/* Batched row-major C[b] = A[b] (m x k) * B[b] (k x n), k ascending. :130-221 */
void oc_matmul(const float* a, const float* b, float* c,
               int64_t batch, int64_t m, int64_t k, int64_t n);
/* Select an alternative FP32 summation order for oc_matmul (0 = default);
 * for sensitivity studies only.  4 = the packed FMA kernel of
 * sgemm_packed.c, a timing stand-in for matrixmultiply's design. */
void oc_set_gemm_order(int order);
/* Threads of the default-order GEMM (1, the reference's, by default; <= 0 =
 * all).  Rows are split between threads, so results do not change. */
void oc_set_gemm_threads(int n);
/* Timing stand-in for matrixmultiply 0.3's sgemm (BLIS loop nest, packed
 * panels, 8x8 FMA micro-kernel); -1 without AVX2/FMA. */
int oc_sgemm_packed(const float* A, const float* B, float* C, int64_t m, int64_t k, int64_t n);

/* ---- composed training step ------------------------------------------------ */
/* Forward + softmax cross-entropy + backward of Sequential(Linear, ReLU, ...,
 * Linear) on one batch, returning per-parameter gradients in Module.parameters()
 * order (W0,b0,W1,b1,...).  dims has n_layers+1 entries; W[l] is
 * [dims[l], dims[l+1]] ([in,out], python/orca/nn/linear.py:29) and b[l] is
 * [1, dims[l+1]].  t is the one-hot (or any) target [batch, dims[n_layers]].
 * logits (nullable) receives the last Linear's output.  Returns 0 or -1. */
int oc_mlp_forward_backward(int n_layers, const int64_t* dims, int64_t batch,
                            const float* const* W, const float* const* b,
                            const float* x, const float* t,
                            float* loss, float* const* dW, float* const* db,
                            float* logits);
/* Forward + loss only (no tape), same arithmetic as the forward half above. */
int oc_mlp_forward(int n_layers, const int64_t* dims, int64_t batch,
                   const float* const* W, const float* const* b,
                   const float* x, const float* t, float* loss, float* logits);
/* python/orca/nn/loss.py:59-100 + orca-python/src/lib.rs:664-669 forward and
 * the reverse sweep of its 21 tape nodes. dP may be NULL (forward only). */
void oc_softmax_ce(const float* P, const float* T, int64_t batch, int64_t classes,
                   float* loss, float* dP);

/* python/orca/optim/sgd.py:46-79.  v may be NULL when momentum == 0.
 * first != 0 marks the first step (velocity buffer empty). */
void oc_sgd_step(float* p, const float* g, float* v, int64_t n, double lr,
                 double momentum, double dampening, double weight_decay, int first);
/* python/orca/optim/adamw.py:48-99; t is the step count after increment. */
void oc_adamw_step(float* p, const float* g, float* m, float* v, int64_t n,
                   double lr, double beta1, double beta2, double eps,
                   double weight_decay, int64_t t);
/* python/orca/distributed.py:232-256: f64 sum over ranks in rank order,
 * times 1/world in f64, rounded to f32. */
void oc_ddp_average(const float* const* rank_grads, int world, int64_t n, float* out);

/* Threads used by the element-wise loops (the reference uses rayon there;
 * its GEMM is single-threaded).  <= 0 means all available. */
void oc_set_threads(int n);
int oc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
