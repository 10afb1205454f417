// Host interface of the fused ghost cross-gram kernel (ghost_gram.cu).
#pragma once

#include "gemm_tc.cuh"

namespace bw {

struct GhostParams {
  int M;   // B1 * S1 rows of side 1
  int N;   // B2 * S2 rows of side 2
  int K;   // activation width
  int D;   // gradient width
  int B1, S1, B2, S2;
  float* out;  // (B1, B2) fp32, accumulated with atomics
  long long ldo;
  int* err;
  // Embedding layers: with token ids set, the activation Gram is the token-equality mask
  // [tok1[r] == tok2[c]] (one-hot activations) and no activation GEMM runs.
  const long long* tok1;
  const long long* tok2;
  // Only the i == j terms (per-sample norms / dots of two factor sets of one batch): CTAs
  // whose row and column sample ranges do not overlap leave at once.
  int diag_only;
};

void ghost_gram_launch(const GemmOperand& a1, const GemmOperand& a2, const GemmOperand& g1,
                       const GemmOperand& g2, GhostParams p, cudaStream_t stream);

}  // namespace bw
