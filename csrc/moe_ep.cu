// Expert-parallel MoE data movement over NVLink peer memory.
//
// Dispatch: every (token, top-k slot) row of this rank is stored straight into the receive
// buffer of the rank that owns the slot's expert, at a row precomputed so that each owner's
// rows come out grouped by local expert (16-byte peer stores; one row = one CTA-strided
// loop).  With it goes the row's origin (source rank, source slot row), which the owner's
// expert down-projection GEMM uses to store its output rows back into the SOURCE rank's
// combine buffer from inside its epilogue (see kStoreBF16Scatter in gemm_tc.cu).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "moe_ep.cuh"

namespace bw {
namespace {

constexpr int kMaxRanks = 8;

struct PeerRows {
  uint4* rows[kMaxRanks];  // each rank's receive buffer (peer-mapped)
  int2* meta[kMaxRanks];   // each rank's origin table
};

// Row r of `src` (r = token * k + slot) goes to rank dst_rank[r], row dst_row[r].
__global__ void dispatch_kernel(const uint4* __restrict__ src, const int* __restrict__ dst_rank,
                                const int* __restrict__ dst_row, PeerRows peers, int rows, int vec_per_row,
                                int self, int rows_per_token, int token_stride_vec) {
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int dr = dst_rank[r], drow = dst_row[r];
    const uint4* s = src + (long long)(r / rows_per_token) * token_stride_vec;
    uint4* d = peers.rows[dr] + (long long)drow * vec_per_row;
    for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) d[v] = s[v];
    if (threadIdx.x == 0) peers.meta[dr][drow] = make_int2(self, r);
  }
}

}  // namespace

void moe_dispatch(const void* src, long long token_stride, const int* dst_rank, const int* dst_row,
                  void* const* peer_rows, int2* const* peer_meta, int world, int rows, int cols, int self,
                  int rows_per_token, cudaStream_t s) {
  PeerRows p{};
  for (int r = 0; r < world && r < kMaxRanks; ++r) {
    p.rows[r] = static_cast<uint4*>(peer_rows[r]);
    p.meta[r] = peer_meta[r];
  }
  if (rows <= 0) return;
  const int grid = rows < 148 * 8 ? rows : 148 * 8;
  dispatch_kernel<<<grid, 128, 0, s>>>(static_cast<const uint4*>(src), dst_rank, dst_row, p, rows, cols / 8, self,
                                       rows_per_token, (int)(token_stride / 8));
}

}  // namespace bw
