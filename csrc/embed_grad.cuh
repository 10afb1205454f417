// Host interface of the dense per-sample embedding-gradient kernel (embed_grad.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace bw {

// out: (R, E) rows, R = B * vocab, every row written exactly once (zero where no token of
// that sample has that id).  keys: the n token keys b * vocab + id in ascending order,
// order: the token row of g (n, E) behind each sorted key.  E a multiple of 16 / elem size.
// elem_bytes is 2 (bf16 in, bf16 out) or 4 (fp32 in, fp32 out).
void embedding_dense_grad(const int64_t* keys, const int64_t* order, const void* g, void* out, long long R, int n,
                          int E, int elem_bytes, cudaStream_t s);

}  // namespace bw
