// Mask-style projection of factorized per-sample gradients (sm_100a): keep M fixed
// coordinates (rows[m], cols[m]) of every per-sample weight gradient dW_b = R_b^T C_b
// without forming dW:
//
//     out[b][m] = sum_t R[b][t][rows[m]] * C[b][t][cols[m]]
//
// One CTA owns sample b and a chunk of coordinates.  It walks the token axis in tiles of
// TT rows: the TT x KR and TT x KC slices of the two factors are copied into shared memory
// with 16-byte loads (each factor row is read once per coordinate chunk, from L2 after the
// first chunk), then every thread gathers its coordinates' pairs from shared memory and
// accumulates in fp32.  The reference gathers with index_select over (B, T, chunk) copies
// (dattri_llm/gradient/ops/projection.py:687-811).
#include "mask_gather.cuh"

#include <stdexcept>

namespace bw {
namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 4;                     // coordinates per thread
constexpr int kChunk = kThreads * kPerThread;     // coordinates per CTA
constexpr int kSmemBudget = 192 * 1024;

__global__ void __launch_bounds__(kThreads)
    mask_gather_kernel(const __nv_bfloat16* __restrict__ R, const __nv_bfloat16* __restrict__ C,
                       const int* __restrict__ rows, const int* __restrict__ cols, float* __restrict__ out, int T,
                       int KR, int KC, int M, int TT) {
  extern __shared__ __align__(16) unsigned char smem[];
  __nv_bfloat16* sR = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sC = sR + (long long)TT * KR;
  const int b = blockIdx.y;
  const int m0 = blockIdx.x * kChunk;
  int r_idx[kPerThread], c_idx[kPerThread];
  float acc[kPerThread];
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int m = m0 + u * kThreads + threadIdx.x;
    r_idx[u] = m < M ? min(max(rows[m], 0), KR - 1) : 0;  // clamped: never outside the tile
    c_idx[u] = m < M ? min(max(cols[m], 0), KC - 1) : 0;
    acc[u] = 0.f;
  }
  const uint4* gR = reinterpret_cast<const uint4*>(R + (long long)b * T * KR);
  const uint4* gC = reinterpret_cast<const uint4*>(C + (long long)b * T * KC);
  for (int t0 = 0; t0 < T; t0 += TT) {
    const int tt = min(TT, T - t0);
    const int nr = tt * (KR / 8), nc = tt * (KC / 8);
    uint4* dR = reinterpret_cast<uint4*>(sR);
    uint4* dC = reinterpret_cast<uint4*>(sC);
    const uint4* srcR = gR + (long long)t0 * (KR / 8);
    const uint4* srcC = gC + (long long)t0 * (KC / 8);
    for (int v = threadIdx.x; v < nr; v += kThreads) dR[v] = srcR[v];
    for (int v = threadIdx.x; v < nc; v += kThreads) dC[v] = srcC[v];
    __syncthreads();
    for (int k = 0; k < tt; ++k) {
      const __nv_bfloat16* rowR = sR + (long long)k * KR;
      const __nv_bfloat16* rowC = sC + (long long)k * KC;
#pragma unroll
      for (int u = 0; u < kPerThread; ++u)
        acc[u] = fmaf(__bfloat162float(rowR[r_idx[u]]), __bfloat162float(rowC[c_idx[u]]), acc[u]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int m = m0 + u * kThreads + threadIdx.x;
    if (m < M) out[(long long)b * M + m] = acc[u];
  }
}

}  // namespace

void mask_gather(const __nv_bfloat16* R, const __nv_bfloat16* C, const int* rows, const int* cols, float* out,
                 int B, int T, int KR, int KC, int M, cudaStream_t s) {
  if (B <= 0 || M <= 0) return;
  const long long row_bytes = (long long)(KR + KC) * 2;
  if (row_bytes > kSmemBudget) throw std::runtime_error("mask_gather: factor rows wider than the shared-memory tile");
  int TT = (int)(kSmemBudget / row_bytes);
  if (TT > 32) TT = 32;
  if (TT < 1) TT = 1;
  const size_t smem = (size_t)TT * row_bytes;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(mask_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    configured[dev & 63] = 1;
  }
  dim3 grid((M + kChunk - 1) / kChunk, B, 1);
  mask_gather_kernel<<<grid, kThreads, smem, s>>>(R, C, rows, cols, out, T, KR, KC, M, TT);
}

}  // namespace bw
