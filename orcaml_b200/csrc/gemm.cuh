// gemm.cuh -- FP32-accurate GEMM with fused epilogues for the MLP step.
//
// C[M,N] = A[M,K] * B[K,N] (+ epilogue).  Operands are stored as a pair of
// fp32 planes: `hi` holds TF32-exact values and `lo` the exact fp32 residual
// (x == hi + lo), so the tcgen05 kernel can form hi*hi + hi*lo + lo*hi on the
// TF32 tensor cores without any conversion pass.  Either operand may be
// K-major (element (mn,k) at mn*ld + k) or MN-major (at k*ld + mn), which
// covers X@W, dY@W^T and X^T@dY without materialised transposes.
#pragma once

#include "common.cuh"

namespace orca {

struct Operand {
  const float* hi = nullptr;   // TF32-exact plane (or plain fp32 when lo == nullptr)
  const float* lo = nullptr;   // residual plane; nullptr = operand is plain fp32
  int64_t ld = 0;              // leading dimension in elements
  bool mn_major = false;
};

enum EpiMode : int {
  EPI_STORE = 0,            // out = acc
  EPI_BIAS = 1,             // out = acc + bias[n]
  EPI_BIAS_RELU_SPLIT = 2,  // a = relu(acc + bias[n]); (out, out_lo) = split(a)
  EPI_MASK_SPLIT = 3,       // g = (mask_hi + mask_lo)[m,n] > 0 ? acc : 0; (out, out_lo) = split(g)
  EPI_SPLIT = 4,            // (out, out_lo) = split(acc)
};

struct Epilogue {
  int mode = EPI_STORE;
  float* out = nullptr;
  float* out_lo = nullptr;
  int64_t ldc = 0;
  const float* bias = nullptr;
  const float* mask_hi = nullptr;   // same [M, ldc] layout as out
  const float* mask_lo = nullptr;
};

// AUTO: tensor cores when eligible and large enough; SIMT: FFMA kernels only;
// TC: tensor cores whenever eligible (skinny/unaligned shapes still use SIMT).
enum GemmPath : int { GEMM_AUTO = 0, GEMM_SIMT = 1, GEMM_TC = 2 };

// Enqueue on ctx->stream.  `workspace`/`workspace_bytes` may be null/0; the
// split-K skinny kernels then allocate stream-ordered scratch.
orca_status gemm(orca_ctx* ctx, int64_t M, int64_t N, int64_t K, const Operand& A,
                 const Operand& B, const Epilogue& ep, int path,
                 float* workspace = nullptr, size_t workspace_bytes = 0);

// Whether the tcgen05 kernel can take these operands at all.
bool gemm_tc_eligible(int64_t M, int64_t N, int64_t K, const Operand& A, const Operand& B);

// Which path `gemm` would take (for reporting and tests).
int gemm_select(orca_ctx* ctx, int64_t M, int64_t N, int64_t K, const Operand& A,
                const Operand& B, const Epilogue& ep, int path);

// Split a plain fp32 array into (hi, lo) planes: n elements.
orca_status split_planes(orca_ctx* ctx, const float* x, float* hi, float* lo, int64_t n);

}  // namespace orca
