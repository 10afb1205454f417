// Host interface of the expert-parallel dispatch (moe_ep.cu).
#pragma once

#include <cuda_runtime.h>

namespace bw {

// Store row r of src (token r / rows_per_token, row stride token_stride bf16 elements) into
// peer dst_rank[r]'s receive buffer at row dst_row[r] (cols bf16, a multiple of 8), with its
// origin (self, r) into that peer's origin table.
void moe_dispatch(const void* src, long long token_stride, const int* dst_rank, const int* dst_row,
                  void* const* peer_rows, int2* const* peer_meta, int world, int rows, int cols, int self,
                  int rows_per_token, cudaStream_t s);

}  // namespace bw
