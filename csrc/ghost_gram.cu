// Fused "ghost" cross-gram of factorized per-sample gradients (sm_100a):
//
//   out[i][j] += sum_{s in sample i, t in sample j} (a1[s] . a2[t]) * (g1[s] . g2[t])
//
// which equals <dW1_i, dW2_j> for dW = g^T a.  Rows r = i*S1 + s of the flattened
// side-1 factors, columns c = j*S2 + t of side 2.  Two kernels:
//   * ghost_gram_persistent (K + D <= 256, the LoGra-projected case): persistent CTAs with
//     the side-1 row block resident in shared memory and double-buffered TMEM accumulators
//     (see its comment below);
//   * ghost_gram_kernel (wider factors): one CTA per 128 x 128 tile, described next.
// ghost_gram_kernel: one CTA owns a 128 x 128 tile of
// the (B1*S1) x (B2*S2) token-pair grid and keeps BOTH Gram tiles in TMEM:
//   columns [0,128)   Ka = A1_tile . A2_tile^T   (K loop over activation features)
//   columns [128,256) Kg = G1_tile . G2_tile^T   (K loop over gradient features)
// One TMA/mbarrier pipeline streams the activation blocks, then the gradient
// blocks; the MMA thread switches accumulator at the boundary.  The epilogue
// multiplies the two tiles elementwise and reduces them to (i, j) partial sums:
// first along its row within each column segment, then across the lanes of a
// warp when they share a sample, into shared-memory bins, finally one global
// fp32 atomic per (i, j) bin.  The (B1 S1) x (B2 S2) products never reach HBM.
//
// Embedding layers (token ids given): the activations are one-hot token ids, so
// Ka[r][c] = [tok1[r] == tok2[c]]; only the gradient Gram runs on the tensor cores and the
// epilogue masks it by token equality -- no vocab-sized buffer, no (B1 S1) x (B2 S2) mask.
#include "ghost_gram.cuh"
#include "tc_common.cuh"

#include <algorithm>

namespace bw {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int kStages = 4;
constexpr int kTile = 128 * BK * 2;  // both operands have 128-row tiles
constexpr int kBinsMax = 4096;       // fp32 bins in the reused pipeline smem
constexpr int kSmem = kStages * 2 * kTile + 1024 + 256;

__global__ void __launch_bounds__(128, 1)
    ghost_gram_kernel(const __grid_constant__ CUtensorMap tA1, const __grid_constant__ CUtensorMap tA2,
                      const __grid_constant__ CUtensorMap tG1, const __grid_constant__ CUtensorMap tG2,
                      GhostParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t* sX = smem;                       // side-1 tiles
  uint8_t* sY = smem + kStages * kTile;     // side-2 tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kTile);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  float* bins = reinterpret_cast<float*>(smem);  // reused after the main loop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * BM;
  if (p.diag_only) {  // uniform over the CTA, before any setup
    const int ia = m0 / p.S1, ib = (min(m0 + BM, p.M) - 1) / p.S1;
    const int ja = n0 / p.S2, jb = (min(n0 + BN, p.N) - 1) / p.S2;
    if (jb < ia || ja > ib) return;
  }
  const bool tok = p.tok1 != nullptr;
  const int nka = tok ? 0 : (p.K + BK - 1) / BK;
  const int nkg = (p.D + BK - 1) / BK;
  const int nk = nka + nkg;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tA1);
    tma_prefetch_desc(&tA2);
    tma_prefetch_desc(&tG1);
    tma_prefetch_desc(&tG2);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&empty[s], ((i / kStages) & 1) ^ 1, p.err, kErrWaitEmpty)) break;
      mbar_arrive_expect_tx(&full[s], 2 * kTile);
      const bool act = i < nka;
      const int kc = (act ? i : i - nka) * BK;
      tma_load_3d(sX + s * kTile, act ? &tA1 : &tG1, &full[s], kc, m0, 0);
      tma_load_3d(sY + s * kTile, act ? &tA2 : &tG2, &full[s], kc, n0, 0);
      issued = i + 1;
    }
    for (int i = max(0, issued - kStages); i < issued; ++i)
      mbar_wait(&full[i % kStages], (i / kStages) & 1, p.err, kErrWaitFull);
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % kStages;
      if (!mbar_wait(&full[s], (i / kStages) & 1, p.err, kErrWaitFull)) break;
      tc_fence_after();
      const bool act = i < nka;
      const int ii = act ? i : i - nka;
      const uint32_t acc = tmem + (act ? 0u : 128u);
      const uint64_t dx = smem_desc_kmajor_sw128(sX + s * kTile);
      const uint64_t dy = smem_desc_kmajor_sw128(sY + s * kTile);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k) tc_mma_f16(acc, dx + 2 * k, dy + 2 * k, idesc, (ii | k) != 0);
      tc_commit(&empty[s]);
    }
    tc_commit(done);
  }
  __syncwarp();
  const bool ok = mbar_wait(done, 0, p.err, kErrWaitDone);
  __syncwarp();
  tc_fence_after();
  // Every stage has been consumed (done fired after the last commit), so the
  // pipeline buffers can be reused as (i, j) bins.
  const int row = m0 + warp * 32 + lane;
  const int i_first = m0 / p.S1;
  const int i_last = min(p.B1 - 1, (min(m0 + BM, p.M) - 1) / p.S1);
  const int j_first = n0 / p.S2;
  const int j_last = min(p.B2 - 1, (min(n0 + BN, p.N) - 1) / p.S2);
  const int ni = i_last - i_first + 1;
  const int nj = j_last - j_first + 1;
  const bool use_bins = ni * nj <= kBinsMax;
  __syncthreads();  // the producer has drained its copies before bins reuse the buffers
  if (use_bins)
    for (int e = threadIdx.x; e < ni * nj; e += blockDim.x) bins[e] = 0.f;
  __syncthreads();
  const int my_i = row / p.S1;
  const bool row_ok = ok && row < p.M;
  const long long my_tok = (tok && row < p.M) ? p.tok1[row] : -1;
  const bool warp_uniform_i = __all_sync(0xffffffffu, (m0 + warp * 32) / p.S1 == my_i) &&
                              __all_sync(0xffffffffu, row < p.M);
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    uint32_t ra[32], rg[32];
    if (!tok) tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, ra);
    tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + 128u + (uint32_t)c0, rg);
    tmem_ld_wait();
    const int cbase = n0 + c0;
    if (cbase >= p.N) continue;  // warp-uniform
    // token mode: lane l holds column (cbase + l)'s id; column cc's id is shuffled from lane cc
    const long long col_tok = (tok && cbase + lane < p.N) ? p.tok2[cbase + lane] : -2;
    // Walk the 32 columns (static register indexing); a column-sample boundary is
    // warp-uniform, so each segment is flushed by the whole warp together.
    auto flush = [&](float v, int j) {
      if (!row_ok) v = 0.f;
      if (warp_uniform_i) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane != 0) return;
      }
      if (!row_ok || my_i >= p.B1 || j >= p.B2 || (p.diag_only && j != my_i)) return;
      if (use_bins)
        atomicAdd(&bins[(my_i - i_first) * nj + (j - j_first)], v);
      else
        atomicAdd(p.out + (long long)my_i * p.ldo + j, v);
    };
    int cur_j = cbase / p.S2;
    int next_b = (cur_j + 1) * p.S2;
    float v = 0.f;
#pragma unroll
    for (int cc = 0; cc < 32; ++cc) {
      if (cbase + cc >= next_b) {
        flush(v, cur_j);
        v = 0.f;
        ++cur_j;
        next_b += p.S2;
      }
      if (tok) {
        const long long t2 = __shfl_sync(0xffffffffu, col_tok, cc);
        if (t2 == my_tok) v += __uint_as_float(rg[cc]);
      } else {
        v += __uint_as_float(ra[cc]) * __uint_as_float(rg[cc]);
      }
    }
    flush(v, cur_j);
  }
  __syncthreads();
  if (use_bins && ok) {
    for (int e = threadIdx.x; e < ni * nj; e += blockDim.x) {
      const int i = i_first + e / nj, j = j_first + e % nj;
      atomicAdd(p.out + (long long)i * p.ldo + j, bins[e]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------------------
// Persistent form for narrow factors (K + D <= 256, e.g. LoGra-projected layers), 320 threads:
// warp 8 = TMA producer, warp 9 = MMA issuer, warps 0-7 = epilogue (warps w and w + 4 read the
// same TMEM lane quadrant -- the same 32 side-1 rows -- and split the tile's columns).  A CTA walks a contiguous
// run of (row block, column block) tiles in row-major order.  The side-1 row block (A1 and G1,
// at most four 64-wide blocks) is loaded once per row block and stays in shared memory; the
// side-2 blocks stream through an 8-stage pipeline.  Two TMEM accumulator pairs (Ka | Kg, 256
// columns each) alternate, so the Hadamard + segment reduction of one tile runs under the
// MMAs of the next.  Each thread (one side-1 row) carries its running (i, j) partial sum
// across chunks and tiles and flushes it when the column sample j (or the row block) changes:
// one warp-reduced fp32 atomic per (warp, j) instead of one per tile.
constexpr int kRes = 4;   // resident side-1 blocks
constexpr int kS2 = 7;    // side-2 stages
constexpr int kEpiWarps = 8;
constexpr int kScratch = kEpiWarps * 32 * 33 * 4;  // per epilogue warp: 32 rows x 33 floats
constexpr int kPSmem = (kRes + kS2) * kTile + kScratch + 1024 + 512;

struct GhostRun {
  int count;  // tiles of this CTA
  int t0;     // full mode: first tile index
  int rb;     // diag mode: the row block
  int cb_lo;  // diag mode: its first column block
  int cbn;    // column blocks
  bool diag;
  __device__ __forceinline__ void tile(int idx, int& rb_out, int& cb_out) const {
    if (diag) {
      rb_out = rb;
      cb_out = cb_lo + idx;
    } else {
      const int t = t0 + idx;
      rb_out = t / cbn;
      cb_out = t - rb_out * cbn;
    }
  }
};

__global__ void __launch_bounds__(320, 1)
    ghost_gram_persistent(const __grid_constant__ CUtensorMap tA1, const __grid_constant__ CUtensorMap tA2,
                          const __grid_constant__ CUtensorMap tG1, const __grid_constant__ CUtensorMap tG2,
                          GhostParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t* s1 = smem;                   // resident side-1 blocks
  uint8_t* s2 = smem + kRes * kTile;    // side-2 stages
  float* scratch = reinterpret_cast<float*>(smem + (kRes + kS2) * kTile);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (kRes + kS2) * kTile + kScratch);
  uint64_t* empty = full + kS2;
  uint64_t* acc_full = empty + kS2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* s1_full = acc_empty + 2;
  uint64_t* s1_empty = s1_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s1_empty + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tok = p.tok1 != nullptr;
  const int nka = tok ? 0 : (p.K + BK - 1) / BK;
  const int nkg = (p.D + BK - 1) / BK;
  const int nk = nka + nkg;
  const int rbn = (p.M + BM - 1) / BM, cbn = (p.N + BN - 1) / BN;

  GhostRun run;
  run.cbn = cbn;
  run.diag = p.diag_only != 0;
  if (run.diag) {  // one CTA per row block, over the column blocks of its own samples
    run.rb = blockIdx.x;
    const int m0 = run.rb * BM;
    const int i_first = m0 / p.S1, i_last = min(p.B1 - 1, (min(m0 + BM, p.M) - 1) / p.S1);
    run.cb_lo = (int)(((long long)i_first * p.S2) / BN);
    const int cb_hi = min(cbn - 1, (int)(((long long)(i_last + 1) * p.S2 - 1) / BN));
    run.count = i_first < p.B2 ? cb_hi - run.cb_lo + 1 : 0;
    run.t0 = 0;
  } else {
    const long long total = (long long)rbn * cbn;
    run.t0 = (int)(total * blockIdx.x / gridDim.x);
    run.count = (int)(total * (blockIdx.x + 1) / gridDim.x) - run.t0;
    run.rb = run.cb_lo = 0;
  }

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tA1);
    tma_prefetch_desc(&tA2);
    tma_prefetch_desc(&tG1);
    tma_prefetch_desc(&tG2);
    for (int s = 0; s < kS2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(s1_full, 1);
    mbar_init(s1_empty, 1);
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      int g = 0, cur_rb = -1, loads = 0;
      bool alive = true;
      for (int idx = 0; idx < run.count && alive; ++idx) {
        int rb, cb;
        run.tile(idx, rb, cb);
        if (rb != cur_rb) {
          if (loads > 0 && !mbar_wait(s1_empty, (loads - 1) & 1, p.err, kErrWaitEmpty)) break;
          mbar_arrive_expect_tx(s1_full, nk * kTile);
          for (int kb = 0; kb < nk; ++kb) {
            const bool act = kb < nka;
            tma_load_3d(s1 + kb * kTile, act ? &tA1 : &tG1, s1_full, (act ? kb : kb - nka) * BK, rb * BM, 0);
          }
          cur_rb = rb;
          ++loads;
        }
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % kS2;
          if (!mbar_wait(&empty[s], ((g / kS2) & 1) ^ 1, p.err, kErrWaitEmpty)) {
            alive = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], kTile);
          const bool act = kb < nka;
          tma_load_3d(s2 + s * kTile, act ? &tA2 : &tG2, &full[s], (act ? kb : kb - nka) * BK, cb * BN, 0);
        }
      }
      // nothing may still be landing in shared memory when the CTA exits
      for (int i = max(0, g - kS2); i < g; ++i) mbar_wait(&full[i % kS2], (i / kS2) & 1, p.err, kErrWaitFull);
      if (loads > 0) mbar_wait(s1_full, (loads - 1) & 1, p.err, kErrWaitFull);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int g = 0, it = 0, cur_rb = -1, loads = 0;
      bool alive = true;
      for (int idx = 0; idx < run.count && alive; ++idx, ++it) {
        int rb, cb;
        run.tile(idx, rb, cb);
        if (rb != cur_rb) {
          if (loads > 0) tc_commit(s1_empty);  // every MMA on the previous row block issued
          if (!mbar_wait(s1_full, loads & 1, p.err, kErrWaitFull)) break;
          tc_fence_after();
          cur_rb = rb;
          ++loads;
        }
        const int b = it & 1;
        if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1, p.err, kErrWaitDone)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * 256);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % kS2;
          if (!mbar_wait(&full[s], (g / kS2) & 1, p.err, kErrWaitFull)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const bool act = kb < nka;
          const int first = act ? 0 : nka;
          const uint64_t dx = smem_desc_kmajor_sw128(s1 + kb * kTile);
          const uint64_t dy = smem_desc_kmajor_sw128(s2 + s * kTile);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_f16(d + (act ? 0u : 128u), dx + 2 * k, dy + 2 * k, idesc, ((kb - first) | k) != 0);
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[b]);
      }
    }
  } else {
    // ---- epilogue: warps 0-7, one side-1 row per thread, half of each tile's columns ----
    const int quad = warp & 3;          // TMEM lane quadrant = the warp's 32 rows
    const int col_half = (warp >> 2) * (BN / 2);
    int cur_rb = -1, cur_j = -1, my_i = 0, it = 0;
    long long my_tok = -1;
    bool row_ok = false, uniform_i = false;
    float v = 0.f;
    auto flush = [&]() {
      if (cur_j < 0) return;
      float x = row_ok ? v : 0.f;
      if (uniform_i) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane != 0) return;
      }
      if (!row_ok || my_i >= p.B1 || cur_j >= p.B2 || (p.diag_only && cur_j != my_i)) return;
      atomicAdd(p.out + (long long)my_i * p.ldo + cur_j, x);
    };
    for (int idx = 0; idx < run.count; ++idx, ++it) {
      int rb, cb;
      run.tile(idx, rb, cb);
      if (rb != cur_rb) {
        flush();
        v = 0.f;
        cur_j = -1;
        cur_rb = rb;
        const int row = rb * BM + quad * 32 + lane;
        row_ok = row < p.M;
        my_i = row / p.S1;
        my_tok = (tok && row_ok) ? p.tok1[row] : -1;
        uniform_i = __all_sync(0xffffffffu, (rb * BM + quad * 32) / p.S1 == my_i && row_ok);
      }
      const int b = it & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (it >> 1) & 1, p.err, kErrWaitDone));
      if (!ok) break;
      tc_fence_after();
      const int n0 = cb * BN;
#pragma unroll 1
      for (int c0 = col_half; c0 < col_half + BN / 2; c0 += 32) {
        uint32_t ra[32], rg[32];
        const uint32_t lanebase = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * 256 + c0);
        if (!tok) tmem_ld_32x32b_x32(lanebase, ra);
        tmem_ld_32x32b_x32(lanebase + 128u, rg);
        tmem_ld_wait();
        if (c0 + 32 >= col_half + BN / 2) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        const int cbase = n0 + c0;
        if (cbase >= p.N) continue;  // warp-uniform
        const long long col_tok = (tok && cbase + lane < p.N) ? p.tok2[cbase + lane] : -2;
        // column cc's product (zero past N: those side-2 rows were zero-filled, or tok2 is -2)
        auto product = [&](int cc) -> float {
          if (tok) return __shfl_sync(0xffffffffu, col_tok, cc) == my_tok ? __uint_as_float(rg[cc]) : 0.f;
          return __uint_as_float(ra[cc]) * __uint_as_float(rg[cc]);
        };
        const int ncols = min(32, p.N - cbase);
        const int j_lo = cbase / p.S2, j_hi = (cbase + ncols - 1) / p.S2;
        if (j_lo == j_hi) {  // the whole chunk lies in one column sample: one sum
          if (j_lo != cur_j) {
            flush();
            v = 0.f;
            cur_j = j_lo;
          }
          float q[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            if (tok)
              q[cc & 3] += product(cc);
            else
              q[cc & 3] = fmaf(__uint_as_float(ra[cc]), __uint_as_float(rg[cc]), q[cc & 3]);
          }
          v += (q[0] + q[1]) + (q[2] + q[3]);
        } else {  // sample boundaries inside the chunk: walk the columns from shared memory
          float* row_scr = scratch + warp * (32 * 33) + lane * 33;
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) row_scr[cc] = product(cc);
          __syncwarp();
#pragma unroll 1
          for (int cc = 0; cc < ncols; ++cc) {
            const int j = (cbase + cc) / p.S2;  // uniform over the warp
            if (j != cur_j) {
              flush();
              v = 0.f;
              cur_j = j;
            }
            v += row_scr[cc];
          }
          __syncwarp();
        }
      }
    }
    flush();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) tmem_dealloc(tmem, 512);
}

}  // namespace

void ghost_gram_launch(const GemmOperand& a1, const GemmOperand& a2, const GemmOperand& g1,
                       const GemmOperand& g2, GhostParams p, cudaStream_t stream) {
  CUtensorMap t_a1 = make_tmap_kmajor_bf16(a1, BM);
  CUtensorMap t_a2 = make_tmap_kmajor_bf16(a2, BN);
  CUtensorMap t_g1 = make_tmap_kmajor_bf16(g1, BM);
  CUtensorMap t_g2 = make_tmap_kmajor_bf16(g2, BN);
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(ghost_gram_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    cudaFuncSetAttribute(ghost_gram_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    configured |= 1ull << dev;
  }
  const bool tok = p.tok1 != nullptr;
  const int nk = (tok ? 0 : (p.K + BK - 1) / BK) + (p.D + BK - 1) / BK;
  const long long rbn = (p.M + BM - 1) / BM, cbn = (p.N + BN - 1) / BN;
  if (nk <= kRes && rbn * cbn > 0) {
    static int sms[64] = {0};
    if (sms[dev & 63] == 0) cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
    const long long grid = p.diag_only ? rbn : std::min<long long>(rbn * cbn, sms[dev & 63]);
    ghost_gram_persistent<<<(unsigned)grid, 320, kPSmem, stream>>>(t_a1, t_a2, t_g1, t_g2, p);
    return;
  }
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, 1);
  ghost_gram_kernel<<<grid, 128, kSmem, stream>>>(t_a1, t_a2, t_g1, t_g2, p);
}

}  // namespace bw
