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
  // ReLU decisions as bits, word [m * bits_ld + n / 32] bit n % 32 = (value at
  // (m, n) > 0), on the tensor-core path only: EPI_BIAS_RELU_SPLIT writes them
  // to relu_bits_out when it is set; EPI_MASK_SPLIT reads its mask from
  // relu_bits when it is set (4 bytes per 32 columns instead of both mask
  // planes, 8 bytes per element) in full 32-column groups; edge groups and
  // the other paths read the mask planes, which EPI_MASK_SPLIT always needs.
  uint32_t* relu_bits_out = nullptr;
  const uint32_t* relu_bits = nullptr;
  int64_t bits_ld = 0;
  // Next-layer dot (EPI_BIAS_RELU_SPLIT on the tensor-core path only): the
  // activation a[m, n] also feeds the classifier layer's product.  Slice s of
  // 128 output columns writes, for j < dot_n (<= 16),
  //   dot_out[(s * M + m) * dot_ldp + j] = sum_{n in slice} a[m, n] * W[n, j]
  // (sequential FMA over n), W given as fp32 rows of 16 (zero past dot_n):
  // W[n, j] = dot_w[n * 16 + j], 16-byte aligned (see head_pack_weights).
  const float* dot_w = nullptr;
  int dot_n = 0;
  float* dot_out = nullptr;
  int64_t dot_ldp = 0;
  // Tensor-core path: full 128-bit output stores carry an L2 evict-first
  // policy (the output streams past the operands instead of evicting them).
  int store_evict_first = 0;
};

// Columns of the activation covered by one dot_out slice.
constexpr int DOT_SLICE = 128;
constexpr int HEAD_MAX_CLASSES = 16;

// AUTO: tensor cores when eligible and large enough; SIMT: FFMA kernels only;
// TC: tensor cores whenever eligible (skinny/unaligned shapes still use SIMT).
// On the tensor cores, AUTO and TC take the CTA-pair kernel for products with
// an MN-major A operand and M >= 256 (the dW products), the single-CTA kernel
// otherwise (ORCA_GEMM_PAIR=0 / =1: never / always); TC_SINGLE and TC_PAIR
// force one or the other.
enum GemmPath : int { GEMM_AUTO = 0, GEMM_SIMT = 1, GEMM_TC = 2, GEMM_TC_SINGLE = 3,
                      GEMM_TC_PAIR = 4 };
inline bool gemm_path_is_tc(int path) {
  return path == GEMM_TC || path == GEMM_TC_SINGLE || path == GEMM_TC_PAIR;
}

// Enqueue on ctx->stream.  `workspace`/`workspace_bytes` may be null/0; the
// split-K skinny kernels then allocate stream-ordered scratch.
// Part of the single-CTA tensor-core product: the tiles [begin, end) of its
// raster order, on at most max_ctas CTAs (0 = one per SM).  Two launches over
// [0, t) on fewer CTAs and [t, tiles) on all of them leave SMs free for a
// collective during the first (see mlp.cu).
struct TileRange {
  int64_t begin = 0, end = -1;   // end < 0: to the last tile
  int max_ctas = 0;
};

orca_status gemm(orca_ctx* ctx, int64_t M, int64_t N, int64_t K, const Operand& A,
                 const Operand& B, const Epilogue& ep, int path,
                 float* workspace = nullptr, size_t workspace_bytes = 0,
                 const TileRange* range = nullptr);
// Number of tiles of the single-CTA tensor-core kernel for an M x N output.
int64_t gemm_tc_tiles(int64_t M, int64_t N);

// Whether the tcgen05 kernel can take these operands at all.
bool gemm_tc_eligible(int64_t M, int64_t N, int64_t K, const Operand& A, const Operand& B);

// Which path `gemm` would take (for reporting and tests).
int gemm_select(orca_ctx* ctx, int64_t M, int64_t N, int64_t K, const Operand& A,
                const Operand& B, const Epilogue& ep, int path);

// Classifier layer with C <= HEAD_MAX_CLASSES outputs.
// head_logits: logits[m, j] = (sum over s of part[(s*M + m)*ldp + j]) + bias[j],
// the slices summed in order -- the reduction of the next-layer dot above.
orca_status head_logits(orca_ctx* ctx, const float* part, int64_t slices, int64_t M, int C,
                        int64_t ldp, const float* bias, float* logits);
// head_backward: from g = dlogits [B, C] (plain fp32), the layer input
// act = (act_hi + act_lo) [B, H] and W = (w_hi + w_lo) [H, C], in one pass
// over act: dZ[m, n] = act > 0 ? sum_j g[m, j] W[n, j] : 0 written as planes,
// dW[n, j] = sum_m act[m, n] g[m, j] and, when db is given, the bias gradient
// of the layer below db[n] = sum_m dZ[m, n] (row blocks summed in order
// through `part`, which needs head_part_floats(B, H, C) floats).
// W_packed[n * 16 + j] = (w_hi + w_lo)[n * C + j] for j < C, 0 for C <= j < 16:
// the classifier weights in the layout the next-layer dot reads.
orca_status head_pack_weights(orca_ctx* ctx, const float* w_hi, const float* w_lo, int64_t H,
                              int C, float* packed);
int64_t head_row_blocks(int64_t B);
int64_t head_part_floats(int64_t B, int64_t H, int C);
orca_status head_backward(orca_ctx* ctx, int64_t B, int64_t H, int C, const float* g,
                          const float* act_hi, const float* act_lo, const float* w_hi,
                          const float* w_lo, float* dz_hi, float* dz_lo, float* part, float* dw,
                          float* db = nullptr);

// Split a plain fp32 array into (hi, lo) planes: n elements.
orca_status split_planes(orca_ctx* ctx, const float* x, float* hi, float* lo, int64_t n);

}  // namespace orca
