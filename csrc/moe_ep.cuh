// Host interface of the expert-parallel dispatch (moe_ep.cu).
#pragma once

#include <cuda_runtime.h>

namespace bw {

// Store row r of src (token r / rows_per_token, row stride token_stride bf16 elements) into
// peer dst_rank[r]'s receive buffer at row dst_row[r] (cols bf16, a multiple of 8), with its
// origin (self, r) into that peer's origin table (no origin is written when peer_meta is null:
// rows returned to their sources by their recorded origin need none).
void moe_dispatch(const void* src, long long token_stride, const int* dst_rank, const int* dst_row,
                  void* const* peer_rows, int2* const* peer_meta, int world, int rows, int cols, int self,
                  int rows_per_token, cudaStream_t s);

// counts[e] += number of rows (entries of topi, int64 expert ids) routed to expert e.
void moe_count(const long long* topi, int rows, int* counts, cudaStream_t s);

// Receive-buffer rows of this rank's routed rows (dest rank, row) from every source's
// histogram, plus this rank's owner-side ragged-GEMM tables and received-row total.
void moe_place(const long long* topi, int rows, const int* all_counts, int world, int rank, int e_l, int* cursor,
               int* dest, int* dst_row, int* tile_prefix, int* base, int* len, int* total, cudaStream_t s);

// y[t] = sum_j w[t * k + j] * slots[t * k + j] for t < tokens (bf16 rows of cols, fp32 w).
void moe_combine(const void* slots, const float* w, void* y, int tokens, int k, int cols, cudaStream_t s);

// Backward of moe_combine fused with the slot-gradient dispatch: dw[r] = <slots[r], dy[r / k]>
// and bf16(w[r] * dy[r / k]) stored into peer dst_rank[r]'s receive buffer at row dst_row[r],
// its origin (self, r) into that peer's origin table.
void moe_combine_bwd_dispatch(const void* dy, const void* slots, const float* w, float* dw, const int* dst_rank,
                              const int* dst_row, void* const* peer_rows, int2* const* peer_meta, int world, int rows,
                              int k, int cols, int self, cudaStream_t s);

}  // namespace bw
