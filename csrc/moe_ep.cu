// Expert-parallel MoE data movement over NVLink peer memory.
//
// Dispatch: every (token, top-k slot) row of this rank is stored straight into the receive
// buffer of the rank that owns the slot's expert, at a row precomputed so that each owner's
// rows come out grouped by local expert (16-byte peer stores; one row = one CTA-strided
// loop).  With it goes the row's origin (source rank, source slot row), which the owner's
// expert down-projection GEMM uses to store its output rows back into the SOURCE rank's
// combine buffer from inside its epilogue (see kStoreBF16Scatter in gemm_tc.cu).
// Indices (destination rank and row) come from moe_place_kernel, which keeps every row
// inside the owner's receive buffer.
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

// Row r of `src` (r = token * k + slot) goes to rank dst_rank[r], row dst_row[r].  One warp
// per row; each lane keeps eight 16-byte loads in flight before its stores (a row-per-CTA
// loop with two loads per thread was latency-bound).
constexpr int kDispatchUnroll = 8;

__global__ void dispatch_kernel(const uint4* __restrict__ src, const int* __restrict__ dst_rank,
                                const int* __restrict__ dst_row, PeerRows peers, int rows, int vec_per_row,
                                int self, int rows_per_token, int token_stride_vec) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int dr = dst_rank[r], drow = dst_row[r];
    const uint4* s = src + (long long)(r / rows_per_token) * token_stride_vec;
    uint4* d = peers.rows[dr] + (long long)drow * vec_per_row;
    for (int v0 = lane; v0 < vec_per_row; v0 += 32 * kDispatchUnroll) {
      uint4 x[kDispatchUnroll];
#pragma unroll
      for (int u = 0; u < kDispatchUnroll; ++u) {
        const int v = v0 + u * 32;
        if (v < vec_per_row) x[u] = s[v];
      }
#pragma unroll
      for (int u = 0; u < kDispatchUnroll; ++u) {
        const int v = v0 + u * 32;
        if (v < vec_per_row) d[v] = x[u];
      }
    }
    if (lane == 0 && peers.meta[dr] != nullptr) peers.meta[dr][drow] = make_int2(self, r);
  }
}

__device__ __forceinline__ void unpack_bf8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __bfloat1622float2(h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ uint4 pack_bf8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// Combine: y[t] = sum_j w[t, j] * slots[t * k + j] (bf16 rows, fp32 weights and sums).
__global__ void combine_kernel(const uint4* __restrict__ slots, const float* __restrict__ w, uint4* __restrict__ y,
                               int tokens, int k, int vec_per_row) {
  for (int t = blockIdx.x; t < tokens; t += gridDim.x) {
    for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < k; ++j) {
        const float wj = w[t * k + j];
        float x[8];
        unpack_bf8(slots[(long long)(t * k + j) * vec_per_row + v], x);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(wj, x[e], acc[e]);
      }
      y[(long long)t * vec_per_row + v] = pack_bf8(acc);
    }
  }
}

// Backward of the combine, fused with the dispatch of the slot gradients: for row
// r = t * k + j, dw[r] = <slots[r], dy[t]> and bf16(w[r] * dy[t]) is stored straight into
// owner dst_rank[r]'s receive buffer at row dst_row[r] (16-byte peer stores), with the row's
// origin (the receive tables are shared by every layer of one shape, so the origin table is
// rewritten for this layer's backward).
__global__ void combine_bwd_dispatch_kernel(const uint4* __restrict__ dy, const uint4* __restrict__ slots,
                                            const float* __restrict__ w, float* __restrict__ dw,
                                            const int* __restrict__ dst_rank, const int* __restrict__ dst_row,
                                            PeerRows peers, int rows, int k, int vec_per_row, int self) {
  __shared__ float part[32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int t = r / k;
    const float wr = w[r];
    uint4* d = peers.rows[dst_rank[r]] + (long long)dst_row[r] * vec_per_row;
    if (threadIdx.x == 0) peers.meta[dst_rank[r]][dst_row[r]] = make_int2(self, r);
    float dot = 0.f;
    for (int v = threadIdx.x; v < vec_per_row; v += blockDim.x) {
      float g[8], x[8], o[8];
      unpack_bf8(dy[(long long)t * vec_per_row + v], g);
      unpack_bf8(slots[(long long)r * vec_per_row + v], x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        dot = fmaf(g[e], x[e], dot);
        o[e] = wr * g[e];
      }
      d[v] = pack_bf8(o);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = dot;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += part[i];
      dw[r] = s;
    }
    __syncthreads();
  }
}

// Routing histogram: counts[e] += rows routed to expert e (counts zeroed by the caller).
__global__ void moe_count_kernel(const long long* __restrict__ topi, int rows, int* __restrict__ counts) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x)
    atomicAdd(&counts[(int)topi[r]], 1);
}

// Receive layout of every owner: its rows grouped by local expert, then by source rank.
// all_counts[src][e] = rows source `src` routes to expert e (e = owner * e_l + local expert).
// Each block derives this source's first row per expert in shared memory, then places its
// rows: dst_row = first row of (owner, expert) + a slot claimed with an atomic (the order of
// rows inside one (source, expert) group does not matter: each row carries its origin).
// Block 0 also writes this rank's owner-side tables for the ragged expert GEMM.
__global__ void moe_place_kernel(const long long* __restrict__ topi, int rows, const int* __restrict__ all_counts,
                                 int world, int rank, int e_l, int* __restrict__ cursor, int* __restrict__ dest,
                                 int* __restrict__ dst_row, int* __restrict__ tile_prefix, int* __restrict__ base,
                                 int* __restrict__ len, int* __restrict__ total) {
  extern __shared__ int first[];  // [world * e_l]
  const int experts = world * e_l;
  for (int e = threadIdx.x; e < experts; e += blockDim.x) {
    const int owner = e / e_l, le = e % e_l;
    int off = 0;
    for (int l = 0; l < le; ++l)
      for (int s = 0; s < world; ++s) off += all_counts[s * experts + owner * e_l + l];
    for (int s = 0; s < rank; ++s) off += all_counts[s * experts + e];
    first[e] = off;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    int b = 0, t = 0;
    for (int l = 0; l < e_l; ++l) {
      int n = 0;
      for (int s = 0; s < world; ++s) n += all_counts[s * experts + rank * e_l + l];
      base[l] = b;
      len[l] = n;
      tile_prefix[l] = t;
      b += n;
      t += (n + 255) / 256;  // 256-row blocks, the ragged GEMM's unit
    }
    tile_prefix[e_l] = t;
    *total = b;
  }
  __syncthreads();
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const int e = (int)topi[r];
    dest[r] = e / e_l;
    dst_row[r] = first[e] + atomicAdd(&cursor[e], 1);
  }
}

}  // namespace

void moe_count(const long long* topi, int rows, int* counts, cudaStream_t s) {
  if (rows <= 0) return;
  const int grid = (rows + 255) / 256 < 148 * 4 ? (rows + 255) / 256 : 148 * 4;
  moe_count_kernel<<<grid, 256, 0, s>>>(topi, rows, counts);
}

void moe_place(const long long* topi, int rows, const int* all_counts, int world, int rank, int e_l, int* cursor,
               int* dest, int* dst_row, int* tile_prefix, int* base, int* len, int* total, cudaStream_t s) {
  const int blocks = (rows + 255) / 256;
  const int grid = blocks < 1 ? 1 : (blocks < 148 * 2 ? blocks : 148 * 2);
  moe_place_kernel<<<grid, 256, (size_t)world * e_l * sizeof(int), s>>>(topi, rows, all_counts, world, rank, e_l,
                                                                         cursor, dest, dst_row, tile_prefix, base,
                                                                         len, total);
}

void moe_combine(const void* slots, const float* w, void* y, int tokens, int k, int cols, cudaStream_t s) {
  if (tokens <= 0) return;
  const int grid = tokens < 148 * 8 ? tokens : 148 * 8;
  combine_kernel<<<grid, 256, 0, s>>>(static_cast<const uint4*>(slots), w, static_cast<uint4*>(y), tokens, k,
                                      cols / 8);
}

void moe_combine_bwd_dispatch(const void* dy, const void* slots, const float* w, float* dw, const int* dst_rank,
                              const int* dst_row, void* const* peer_rows, int2* const* peer_meta, int world, int rows,
                              int k, int cols, int self, cudaStream_t s) {
  PeerRows p{};
  for (int r = 0; r < world && r < kMaxRanks; ++r) {
    p.rows[r] = static_cast<uint4*>(peer_rows[r]);
    p.meta[r] = peer_meta[r];
  }
  if (rows <= 0) return;
  const int grid = rows < 148 * 8 ? rows : 148 * 8;
  combine_bwd_dispatch_kernel<<<grid, 128, 0, s>>>(static_cast<const uint4*>(dy), static_cast<const uint4*>(slots),
                                                   w, dw, dst_rank, dst_row, p, rows, k, cols / 8, self);
}

void moe_dispatch(const void* src, long long token_stride, const int* dst_rank, const int* dst_row,
                  void* const* peer_rows, int2* const* peer_meta, int world, int rows, int cols, int self,
                  int rows_per_token, cudaStream_t s) {
  PeerRows p{};
  for (int r = 0; r < world && r < kMaxRanks; ++r) {
    p.rows[r] = static_cast<uint4*>(peer_rows[r]);
    p.meta[r] = peer_meta != nullptr ? peer_meta[r] : nullptr;
  }
  if (rows <= 0) return;
  const int ctas = (rows + 3) / 4;  // four warps (rows) per CTA
  const int grid = ctas < 148 * 8 ? ctas : 148 * 8;
  dispatch_kernel<<<grid, 128, 0, s>>>(static_cast<const uint4*>(src), dst_rank, dst_row, p, rows, cols / 8, self,
                                       rows_per_token, (int)(token_stride / 8));
}

}  // namespace bw
