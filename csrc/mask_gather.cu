// Mask-style projection of factorized per-sample gradients (sm_100a): keep M fixed
// coordinates (rows[m], cols[m]) of every per-sample weight gradient dW_b = R_b^T C_b
// without forming dW:
//
//     out[b][m] = sum_t R[b][t][rows[m]] * C[b][t][cols[m]]
//
// Grid: (coordinate chunk, token range, sample).  A CTA walks its token range in tiles of TT
// rows; the tile's R and C rows are contiguous in memory, so each is ONE bulk async copy
// (cp.async.bulk, no tensor map) into shared memory, double-buffered on two mbarriers so the
// next tile lands while this one is gathered.  Every thread gathers its coordinates' pairs
// from shared memory into fp32 sums; with several token ranges per sample the sums meet in
// `out` through atomics (zeroed first).  The reference gathers with index_select over
// (B, T, chunk) copies (dattri_llm/gradient/ops/projection.py:687-811).
#include "mask_gather.cuh"

#include <stdexcept>

#include "tc_common.cuh"

namespace bw {
namespace {

constexpr int kThreads = 256;
constexpr int kPerThread = 4;                     // coordinates per thread
constexpr int kChunk = kThreads * kPerThread;     // coordinates per CTA
constexpr int kSmemBudget = 200 * 1024;           // both buffers
constexpr int kMaxTT = 64;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__global__ void __launch_bounds__(kThreads)
    mask_gather_kernel(const __nv_bfloat16* __restrict__ R, const __nv_bfloat16* __restrict__ C,
                       const int* __restrict__ rows, const int* __restrict__ cols, float* __restrict__ out, int T,
                       int KR, int KC, int M, int TT, int trange, int atomic, int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  const long long buf_elems = (long long)TT * (KR + KC);
  __nv_bfloat16* buf0 = reinterpret_cast<__nv_bfloat16*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * buf_elems * 2);
  const int b = blockIdx.z;
  const int m0 = blockIdx.x * kChunk;
  const int t_begin = blockIdx.y * trange, t_end = min(T, t_begin + trange);
  const int ntiles = t_begin < t_end ? (t_end - t_begin + TT - 1) / TT : 0;
  int r_idx[kPerThread], c_idx[kPerThread];
  float acc[kPerThread];
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int m = m0 + u * kThreads + threadIdx.x;
    r_idx[u] = m < M ? min(max(rows[m], 0), KR - 1) : 0;  // clamped: never outside the tile
    c_idx[u] = m < M ? min(max(cols[m], 0), KC - 1) : 0;
    acc[u] = 0.f;
  }
  const __nv_bfloat16* gR = R + (long long)b * T * KR;
  const __nv_bfloat16* gC = C + (long long)b * T * KC;
  auto issue = [&](int i) {  // tile i into buffer i & 1 (thread 0)
    const int t0 = t_begin + i * TT, tt = min(TT, t_end - t0);
    __nv_bfloat16* dst = buf0 + (i & 1) * buf_elems;
    const uint32_t br = (uint32_t)tt * KR * 2, bc = (uint32_t)tt * KC * 2;
    mbar_arrive_expect_tx(&full[i & 1], br + bc);
    bulk_load(dst, gR + (long long)t0 * KR, br, &full[i & 1]);
    bulk_load(dst + (long long)TT * KR, gC + (long long)t0 * KC, bc, &full[i & 1]);
  };
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2 && i < ntiles; ++i) issue(i);
  }
  bool ok = true;
  for (int i = 0; i < ntiles; ++i) {
    if (ok && !mbar_wait(&full[i & 1], (i >> 1) & 1, err, kErrWaitFull)) ok = false;
    if (ok) {
      const __nv_bfloat16* sR = buf0 + (i & 1) * buf_elems;
      const __nv_bfloat16* sC = sR + (long long)TT * KR;
      const int tt = min(TT, t_end - (t_begin + i * TT));
      for (int k = 0; k < tt; ++k) {
        const __nv_bfloat16* rowR = sR + (long long)k * KR;
        const __nv_bfloat16* rowC = sC + (long long)k * KC;
#pragma unroll
        for (int u = 0; u < kPerThread; ++u)
          acc[u] = fmaf(__bfloat162float(rowR[r_idx[u]]), __bfloat162float(rowC[c_idx[u]]), acc[u]);
      }
    }
    __syncthreads();  // everyone is done with this buffer
    if (threadIdx.x == 0 && ok && i + 2 < ntiles) {
      fence_proxy_async_smem();  // the generic-proxy reads above before the async-proxy refill
      issue(i + 2);
    }
  }
  // drain: no copy may still be landing when the CTA exits (bounded; only after a failed wait)
  if (threadIdx.x == 0 && !ok)
    for (int i = 0; i < ntiles && i < 2; ++i) mbar_wait(&full[i & 1], 0, err, kErrWaitFull);
#pragma unroll
  for (int u = 0; u < kPerThread; ++u) {
    const int m = m0 + u * kThreads + threadIdx.x;
    if (m < M) {
      if (atomic)
        atomicAdd(out + (long long)b * M + m, acc[u]);
      else
        out[(long long)b * M + m] = acc[u];
    }
  }
}

}  // namespace

void mask_gather(const __nv_bfloat16* R, const __nv_bfloat16* C, const int* rows, const int* cols, float* out,
                 int B, int T, int KR, int KC, int M, int* err, cudaStream_t s) {
  if (B <= 0 || M <= 0) return;
  const long long row_bytes = (long long)(KR + KC) * 2;
  if (2 * row_bytes > kSmemBudget) throw std::runtime_error("mask_gather: factor rows wider than the shared-memory tile");
  int TT = (int)(kSmemBudget / (2 * row_bytes));
  if (TT > kMaxTT) TT = kMaxTT;
  if (TT > T) TT = T > 0 ? T : 1;
  const size_t smem = (size_t)2 * TT * row_bytes + 64;
  static int configured[64] = {0};
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev & 63]) {
    cudaFuncSetAttribute(mask_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 64);
    cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    configured[dev & 63] = 1;
  }
  // token ranges: enough CTAs for two per SM, each range at least two tiles long
  const long long base = (long long)((M + kChunk - 1) / kChunk) * B;
  const int tiles = (T + TT - 1) / TT;
  long long ranges = (2LL * sms[dev & 63] + base - 1) / base;
  if (ranges > tiles / 2) ranges = tiles / 2;
  if (ranges < 1) ranges = 1;
  const int trange = (int)(((tiles + ranges - 1) / ranges) * TT);
  ranges = (T + trange - 1) / trange;
  const int atomic = ranges > 1;
  if (atomic) cudaMemsetAsync(out, 0, (size_t)B * M * sizeof(float), s);
  dim3 grid((M + kChunk - 1) / kChunk, (unsigned)ranges, B);
  mask_gather_kernel<<<grid, kThreads, smem, s>>>(R, C, rows, cols, out, T, KR, KC, M, TT, trange, atomic, err);
}

}  // namespace bw
