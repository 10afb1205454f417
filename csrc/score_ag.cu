// Fused all-gather + score GEMM over NVLink (one launch per step).
//
//     out[m][r * R + b] += alpha * sum_k T[m][k] * X_r[b][k]
//
// T is this rank's shard of the packed test matrix (n_local x K, bf16, local HBM); X_r is
// rank r's packed train block (R x K, bf16) living in r's symmetric buffer and read over
// NVLink through a per-peer tensor map (no cluster multicast; every CTA fetches its own
// tiles).  Each pipeline stage loads one 128 x 64 test tile and, from every peer, an R x 64
// slice of its block into consecutive 8-row swizzle atoms of one B tile, so the peers'
// rows are gathered into shared memory exactly when the MMA consumes them: the transfer
// overlaps the math tile by tile and the gathered block never lands in HBM.  K is split
// over CTAs (grid.y) with fp32 atomics into `out`, which the caller zeroes.
#include <cuda_bf16.h>

#include "score_ag.cuh"
#include "tc_common.cuh"

namespace bw {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 128;

template <int BN>
struct AgCfg {
  static constexpr int kTileA = kBM * kBK * 2;
  static constexpr int kTileB = BN * kBK * 2;
  static constexpr int kStages = BN <= 64 ? 8 : 6;
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * (kTileA + kTileB) + 1024 + 256;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    ag_score_kernel(const __grid_constant__ CUtensorMap tmT, const CUtensorMap* __restrict__ peers,
                    AgScoreParams p) {
  using C = AgCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kTileA;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::kStages * C::kTileB);
  uint64_t* empty = full + C::kStages;
  uint64_t* done = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;
  const int split = blockIdx.y;
  const int kblocks = (p.K + kBK - 1) / kBK;
  const int per = (kblocks + p.splits - 1) / p.splits;
  const int kb0 = split * per;
  const int nk = max(0, min(kblocks, kb0 + per) - kb0);
  const int gathered = p.world * p.rows_per_peer;  // live rows of the B tile (<= BN)

  // Rows of the B tile past the gathered ones are never written by TMA: zero them once.
  if (gathered < BN) {
    for (int s = 0; s < C::kStages; ++s) {
      uint4* rowp = reinterpret_cast<uint4*>(sB + s * C::kTileB + gathered * kBK * 2);
      const int n16 = (BN - gathered) * kBK * 2 / 16;
      for (int i = threadIdx.x; i < n16; i += kThreads) rowp[i] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmT);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---- producer: the test tile from local HBM, each peer's slice over NVLink ----
    const uint32_t bytes = C::kTileA + (uint32_t)gathered * kBK * 2;
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1;
      if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrWaitEmpty)) break;
      mbar_arrive_expect_tx(&full[s], bytes);
      const int kc = (kb0 + i) * kBK;
      tma_load_3d(sA + s * C::kTileA, &tmT, &full[s], kc, m0, 0);
      for (int r = 0; r < p.world; ++r)
        tma_load_3d(sB + s * C::kTileB + r * p.rows_per_peer * kBK * 2, peers + r, &full[s], kc, 0, 0);
      issued = i + 1;
    }
    for (int i = max(0, issued - C::kStages); i < issued; ++i)
      mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1, p.err, kErrWaitFull);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1;
      if (!mbar_wait(&full[s], ph, p.err, kErrWaitFull)) break;
      tc_fence_after();
      const uint64_t da = smem_desc_kmajor_sw128(sA + s * C::kTileA);
      const uint64_t db = smem_desc_kmajor_sw128(sB + s * C::kTileB);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k) tc_mma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
      tc_commit(&empty[s]);
    }
    tc_commit(done);
  }
  __syncwarp();

  // ---- epilogue: fp32 atomics of this split's partial sums ----
  const bool ok = nk > 0 ? mbar_wait(done, 0, p.err, kErrWaitDone) : false;
  __syncwarp();
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    uint32_t r[32];
    if (ok) {
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_ld_wait();
    }
    if (!ok || row >= p.M) continue;
    float* o = p.out + (long long)row * p.ldo;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = c0 + j;
      if (j < BN - c0 && n < gathered) atomicAdd(o + n, p.alpha * __uint_as_float(r[j]));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::kTmemCols);
}

template <int BN>
void launch_ag(const CUtensorMap& tmT, const CUtensorMap* peers, const AgScoreParams& p, cudaStream_t s) {
  using C = AgCfg<BN>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(ag_score_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    configured |= 1ull << dev;
  }
  dim3 grid((p.M + kBM - 1) / kBM, p.splits, 1);
  ag_score_kernel<BN><<<grid, kThreads, C::kSmem, s>>>(tmT, peers, p);
}

}  // namespace

int ag_score_tile_n(int gathered) {
  if (gathered <= 16) return 16;
  if (gathered <= 32) return 32;
  if (gathered <= 64) return 64;
  if (gathered <= 128) return 128;
  return 0;
}

void ag_score_launch(const CUtensorMap& tmT, const CUtensorMap* peers, AgScoreParams p, cudaStream_t s) {
  switch (ag_score_tile_n(p.world * p.rows_per_peer)) {
    case 16: launch_ag<16>(tmT, peers, p, s); break;
    case 32: launch_ag<32>(tmT, peers, p, s); break;
    case 64: launch_ag<64>(tmT, peers, p, s); break;
    case 128: launch_ag<128>(tmT, peers, p, s); break;
    default: break;
  }
}

}  // namespace bw
