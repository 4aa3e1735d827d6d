// Host interface of the tcgen05 projection GEMM (gemm.cu).
#pragma once
#include "common.cuh"

namespace yuf {

enum GemmEpi {
  GEMM_EPI_F32 = 0,        // C (fp32) = acc, or C += acc when beta != 0 (residual add);
                           //   tanh(acc) for batch 0 when tanh_batch0 (beta 0)
  GEMM_EPI_BF16 = 1,       // C (bf16) = acc, tanh(acc) for batch 0 when tanh_batch0
  GEMM_EPI_SWIGLU = 2,     // C (bf16) [M, n_out] = SiLU(in) * gate; W rows packed per 64:
                           //   [in 64g .. 64g+63 | gate 64g .. 64g+63] for g = 0, 1, ...
  GEMM_EPI_SWIGLU_F32 = 3  // the same with an fp32 output
};

// One projection C[z] = A[z] . W[z]^T for z < batch (bf16 operands, K-major,
// fp32 accumulation).  A: a_rows rows of lda elements (batch z starts at row
// z * a_brows); W: w_rows rows of K elements (batch z at row z * w_brows);
// C: rows of ldc elements, batch z at element z * c_bstride.  M, N, K per
// batch.  A and W rows must be 16-byte aligned (lda, K multiples of 8).
struct GemmArgs {
  const void* A;
  long long lda, a_rows, a_brows;
  const void* W;
  long long w_rows, w_brows;
  void* C;
  long long ldc, c_bstride;
  int M, N, K, batch;
  int epi;
  float beta;
  int tanh_batch0;
  int n_out;  // GEMM_EPI_SWIGLU: output columns (the FFN hidden width)
};

// Kernel parameters (device side).
struct GemmParams {
  void* C;
  long long ldc, c_bstride, a_brows, w_brows;
  int M, N, K, batch, m_tiles, n_tiles;
  float beta;
  int tanh_batch0, n_out, vec;
};

yuf_status_t gemm_bf16(const GemmArgs& g, cudaStream_t s);

// fp32 operands at fp32 accuracy on the tensor cores (3xTF32): A fp32 [rows, lda]
// (split into tf32 high and low parts inside the kernel), W given as its two
// parts, W_hi (the tf32 high part) and W_lo (the remainder), each [w_rows, K]
// fp32 contiguous (g.W = W_hi).  C = A_lo W_hi^T + A_hi W_lo^T + A_hi W_hi^T.
// lda and K multiples of 4; the epilogues as above (fp32 outputs: GEMM_EPI_F32,
// GEMM_EPI_SWIGLU_F32).
yuf_status_t gemm_tf32x3(const GemmArgs& g, const void* W_lo, cudaStream_t s);
// W [rows, K] fp32 -> (hi, lo): hi = W with the low 13 mantissa bits cleared, lo = W - hi
void split_tf32_host(const float* w, size_t n, float* hi, float* lo);
// expired bounded waits of the GEMM kernel since the last call (clears the count)
unsigned int gemm_wait_timeouts();

}  // namespace yuf
