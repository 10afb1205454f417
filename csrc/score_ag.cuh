// Host interface of the fused all-gather + score GEMM (score_ag.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace bw {

struct AgScoreParams {
  int M;              // rows of the local test shard
  int K;              // packed gradient width
  int world;          // peers gathered (this rank included)
  int rows_per_peer;  // rows of each peer's block (a multiple of 8)
  int splits;         // K split over grid.y
  float alpha;
  float* out;         // (M, world * rows_per_peer) fp32, accumulated with atomics
  long long ldo;
  int* err;
};

// Tile width used for `gathered` = world * rows_per_peer rows (0: unsupported, > 128).
int ag_score_tile_n(int gathered);
void ag_score_launch(const CUtensorMap& tmT, const CUtensorMap* peers, AgScoreParams p, cudaStream_t s);

}  // namespace bw
