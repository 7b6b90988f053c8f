/*
 * sgemm_packed.c -- a TIMING stand-in for the reference's GEMM.
 *
 * TEST INFRASTRUCTURE ONLY (bench.py's CPU-baseline and reference legs);
 * never linked into the product library.
 *
 * The reference's CPU backend multiplies with the third-party crate
 * `matrixmultiply` 0.3, default features, single-threaded
 * (orca-backend-cpu/Cargo.toml:11, call site orca-backend-cpu/src/backend.rs:
 * 197-212).  That crate is not vendored in the reference, so its code is not
 * here; this file restates its published design (the BLIS loop nest) so that
 * the timed CPU baseline runs at a comparable speed:
 *   - loops, outer to inner: column blocks of NC = 1024, depth blocks of
 *     KC = 256, row blocks of MC = 64, then NR-wide and MR-tall panels;
 *   - B's KC x NC block is packed into NR-wide row-major panels and A's
 *     MC x KC block into MR-tall column-major panels, both zero-padded;
 *   - an MR x NR = 8 x 8 register-blocked micro-kernel with one 8-wide
 *     vector accumulator per output row, fused multiply-adds (the crate
 *     selects its FMA kernel at run time when the CPU has FMA);
 *   - the first depth block stores, later depth blocks accumulate into C;
 *     edge tiles go through a temporary and are copied in.
 * Its per-element summation order (KC-blocked, FMA) differs from the
 * oracle's k-ascending one, so it is used for timing only; parity always
 * runs on oc_matmul's default order.
 */
#include <immintrin.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MR 8
#define NR 8
#define KC 256
#define MC 64
#define NC 1024

__attribute__((target("avx2,fma")))
static void kernel_8x8(int64_t kc, const float* ap, const float* bp, float* c, int64_t ldc,
                       int accumulate) {
  __m256 c0 = _mm256_setzero_ps(), c1 = _mm256_setzero_ps(), c2 = _mm256_setzero_ps(),
         c3 = _mm256_setzero_ps(), c4 = _mm256_setzero_ps(), c5 = _mm256_setzero_ps(),
         c6 = _mm256_setzero_ps(), c7 = _mm256_setzero_ps();
  for (int64_t p = 0; p < kc; ++p) {
    const __m256 b = _mm256_load_ps(bp + NR * p);
    const float* a = ap + MR * p;
    c0 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 0), b, c0);
    c1 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 1), b, c1);
    c2 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 2), b, c2);
    c3 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 3), b, c3);
    c4 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 4), b, c4);
    c5 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 5), b, c5);
    c6 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 6), b, c6);
    c7 = _mm256_fmadd_ps(_mm256_broadcast_ss(a + 7), b, c7);
  }
  __m256 acc[MR] = {c0, c1, c2, c3, c4, c5, c6, c7};
  for (int i = 0; i < MR; ++i) {
    float* row = c + i * ldc;
    __m256 v = acc[i];
    if (accumulate) v = _mm256_add_ps(_mm256_loadu_ps(row), v);
    _mm256_storeu_ps(row, v);
  }
}

/* A[m0.., k0..] (row-major, lda) -> MR-tall panels, column-major in each. */
static void pack_a(const float* A, int64_t lda, int64_t mc, int64_t kc, float* out) {
  for (int64_t i0 = 0; i0 < mc; i0 += MR) {
    const int64_t mr = mc - i0 < MR ? mc - i0 : MR;
    for (int64_t p = 0; p < kc; ++p) {
      for (int64_t i = 0; i < mr; ++i) out[p * MR + i] = A[(i0 + i) * lda + p];
      for (int64_t i = mr; i < MR; ++i) out[p * MR + i] = 0.0f;
    }
    out += MR * kc;
  }
}

/* B[k0.., n0..] (row-major, ldb) -> NR-wide panels, row-major in each. */
static void pack_b(const float* B, int64_t ldb, int64_t kc, int64_t nc, float* out) {
  for (int64_t j0 = 0; j0 < nc; j0 += NR) {
    const int64_t nr = nc - j0 < NR ? nc - j0 : NR;
    for (int64_t p = 0; p < kc; ++p) {
      const float* src = B + p * ldb + j0;
      for (int64_t j = 0; j < nr; ++j) out[p * NR + j] = src[j];
      for (int64_t j = nr; j < NR; ++j) out[p * NR + j] = 0.0f;
    }
    out += NR * kc;
  }
}

/* Row blocks of MC rows of one (column block, depth block) step.  Every
 * element of C belongs to exactly one row block, so splitting row blocks
 * between threads leaves each element's arithmetic unchanged. */
static void row_blocks(const float* A, float* C, int64_t m, int64_t k, int64_t n, int64_t j0,
                       int64_t nc, int64_t p0, int64_t kc, const float* bpack, int64_t i_first,
                       int64_t i_step, float* apack) {
  float tmp[MR * NR];
  for (int64_t i0 = i_first; i0 < m; i0 += i_step) {
    const int64_t mc = m - i0 < MC ? m - i0 : MC;
    pack_a(A + i0 * k + p0, k, mc, kc, apack);
    for (int64_t jr = 0; jr < nc; jr += NR) {
      const int64_t nr = nc - jr < NR ? nc - jr : NR;
      for (int64_t ir = 0; ir < mc; ir += MR) {
        const int64_t mr = mc - ir < MR ? mc - ir : MR;
        float* c = C + (i0 + ir) * n + j0 + jr;
        const float* ap = apack + ir * kc;
        const float* bp = bpack + jr * kc;
        if (mr == MR && nr == NR) {
          kernel_8x8(kc, ap, bp, c, n, p0 > 0);
        } else {
          kernel_8x8(kc, ap, bp, tmp, NR, 0);
          for (int64_t i = 0; i < mr; ++i)
            for (int64_t j = 0; j < nr; ++j)
              c[i * n + j] = p0 > 0 ? c[i * n + j] + tmp[i * NR + j] : tmp[i * NR + j];
        }
      }
    }
  }
}

/* C (m x n, row-major) = A (m x k) * B (k x n) on `threads` threads (1 = the
 * reference's single thread; the result does not depend on it).  Returns -1
 * when the CPU lacks AVX2/FMA or memory runs out (the caller then uses its
 * own loop). */
int oc_sgemm_packed_mt(const float* A, const float* B, float* C, int64_t m, int64_t k, int64_t n,
                       int threads) {
  if (!__builtin_cpu_supports("avx2") || !__builtin_cpu_supports("fma")) return -1;
  if (threads < 1) threads = 1;
  float* bpack = (float*)aligned_alloc(64, sizeof(float) * KC * (NC + NR));
  float* apack = (float*)aligned_alloc(64, sizeof(float) * KC * (MC + MR) * (size_t)threads);
  if (!bpack || !apack) {
    free(bpack);
    free(apack);
    return -1;
  }
  if (k == 0) memset(C, 0, sizeof(float) * (size_t)(m * n));
  for (int64_t j0 = 0; j0 < n; j0 += NC) {
    const int64_t nc = n - j0 < NC ? n - j0 : NC;
    for (int64_t p0 = 0; p0 < k; p0 += KC) {
      const int64_t kc = k - p0 < KC ? k - p0 : KC;
      pack_b(B + p0 * n + j0, n, kc, nc, bpack);
      if (threads == 1) {
        row_blocks(A, C, m, k, n, j0, nc, p0, kc, bpack, 0, MC, apack);
      } else {
#pragma omp parallel for num_threads(threads) schedule(static, 1)
        for (int t = 0; t < threads; ++t)
          row_blocks(A, C, m, k, n, j0, nc, p0, kc, bpack, (int64_t)t * MC,
                     (int64_t)threads * MC, apack + (size_t)t * KC * (MC + MR));
      }
    }
  }
  free(bpack);
  free(apack);
  return 0;
}

int oc_sgemm_packed(const float* A, const float* B, float* C, int64_t m, int64_t k, int64_t n) {
  return oc_sgemm_packed_mt(A, B, C, m, k, n, 1);
}
