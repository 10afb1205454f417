// Host interface of the dense per-sample embedding-gradient kernel (embed_grad.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace bw {

// out: (R, E) rows, R = B * vocab, every row written exactly once (zero where no token of
// that sample has that id).  order: the token rows of g (n, E) sorted by key b * vocab + id;
// starts (R + 1): row r's tokens are order[starts[r] .. starts[r + 1]).  E a multiple of
// 16 / elem size; elem_bytes is 2 (bf16 in, bf16 out) or 4 (fp32 in, fp32 out).
void embedding_dense_grad(const int64_t* starts, const int64_t* order, const void* g, void* out, long long R, int E,
                          int elem_bytes, cudaStream_t s);

}  // namespace bw
