// Generic batched "TN" GEMM on the 5th-generation tensor cores (sm_100a):
//
//     C[z][m][n] (op)= alpha * sum_k A[z][m][k] * B[zb][n][k]
//
// A and B are bf16 and K-major (k contiguous), which is how every contraction of
// the library is laid out (projection  x . P^T, per-sample outer products over
// tokens, the test x train score, covariance Gram matrices).  One CTA owns one
// 128 x BN output tile:
//   warp 0 / lane 0   TMA producer: 128 x 64 A-tile and BN x 64 B-tile per stage
//   warp 1 / lane 0   MMA issuer:   4 x tcgen05.mma (K=16 each) per stage, fp32 in TMEM
//   warps 0-3         epilogue:     tcgen05.ld 32 lanes x 32 columns per warp and store
// Split-K spreads the K loop over gridDim.z (the epilogue then accumulates with
// fp32 atomics); rows/columns/K beyond the tensor are zero-filled by TMA.
#include "gemm_tc.cuh"
#include "tc_common.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>

namespace bw {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 128;

template <int BN>
struct Cfg {
  static constexpr int kTileA = BM * BK * 2;  // bytes
  static constexpr int kTileB = BN * BK * 2;
  static constexpr int kStages = BN <= 32 ? 8 : (BN <= 64 ? 6 : (BN <= 128 ? 3 : 4));
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static constexpr int kSmem = kStages * (kTileA + kTileB) + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kRed = BM * BN * 4;  // cluster split-K: the peer's fp32 partial tile
  static constexpr bool kClusterOK = kSmem + kRed <= 227 * 1024;
};

// Wait (bounded) until `*flag` reaches `expect` (acquire), then order those generic-proxy
// writes before this thread's later TMA (async-proxy) reads of the same memory.
__device__ __forceinline__ void stage_wait(const int* flag, int expect, int* err) {
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= expect) break;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      report_error(err, kErrWaitStage);
      break;
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Control block of a staged launch (one per CTA, in registers / local scope).
struct StageCtl {
  const CUtensorMap* own;  // this rank's own shard (read in place); a kernel-parameter address
  const int* flags;  // per owner: pieces copied so far (monotonic across launches)
  int expect;        // flag value meaning "this launch's copy of the owner is complete"
  int mode, self, shard;
  unsigned ready;    // owners already waited for (bit mask)
};

// Store one warp's 32 rows x 32 columns (columns [c0, c0 + 32) of the tile at (m0, n0)) from
// the accumulator registers `r`; rows at or past `limit` are dropped.  `tw` is warp-private
// shared scratch (32 x 33 floats) for the transposed peer stores.
template <int BN>
__device__ __forceinline__ void store_chunk(const GemmParams& p, const uint32_t (&r)[32], void* Cbase, int zc, int m0,
                                            int n0, int c0, int warp, int lane, int limit, float* tw) {
  const int row = m0 + warp * 32 + lane;
  const bool row_ok = row < limit;
  const float alpha = p.alpha;
  if (p.c_mode == kPeerSlotF32 && c0 + 32 <= BN && n0 + c0 + 32 <= p.N && (p.ldc & 3) == 0 &&
      (((long long)zc * p.batch_stride_c) & 3) == 0) {
    // Reduce-scatter chunk through a warp-private transpose in the (now idle) stage memory:
    // each store instruction then writes four whole 128-byte row segments instead of 32
    // scattered 16-byte pieces -- full lines on NVLink.
#pragma unroll
    for (int j = 0; j < 32; ++j) tw[lane * 33 + j] = alpha * __uint_as_float(r[j]);
    __syncwarp();
    const long long slot = 4 * p.per4;
    const int cc = (lane & 7) * 4;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int rr = q * 4 + (lane >> 3);
      const int grow = m0 + warp * 32 + rr;
      if (grow < limit) {
        const long long i = (long long)zc * p.batch_stride_c + (long long)grow * p.ldc + n0 + c0 + cc;
        int owner = (int)((i >> 2) / p.per4);
        owner = owner < p.world ? owner : p.world - 1;
        const float* t = tw + rr * 33 + cc;
        *reinterpret_cast<float4*>(p.peers[owner] + p.self_rank * slot + (i - owner * slot)) =
            make_float4(t[0], t[1], t[2], t[3]);
      }
    }
    __syncwarp();
    return;
  }
  if (p.c_mode == kStoreBF16Scatter && c0 + 32 <= BN && n0 + c0 + 32 <= p.N && (p.ldc & 7) == 0) {
    // Rows sent home through a warp-private transpose: each store instruction writes eight
    // whole 64-byte row segments instead of 32 scattered 16-byte pieces.
#pragma unroll
    for (int j = 0; j < 32; ++j) tw[lane * 33 + j] = alpha * __uint_as_float(r[j]);
    __syncwarp();
    const int cc = (lane & 3) * 8;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int rr = q * 8 + (lane >> 2);
      const int grow = m0 + warp * 32 + rr;
      if (grow < limit) {
        const int2 dstm = p.scatter[grow];
        __nv_bfloat16* Cr = reinterpret_cast<__nv_bfloat16*>(p.peers[dstm.x]) + (long long)dstm.y * p.ldc;
        const float* t = tw + rr * 33 + cc;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(t[2 * e], t[2 * e + 1]);
          w[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(Cr + n0 + c0 + cc) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncwarp();
    return;
  }
  if ((p.c_mode == kStoreBF16 || (p.c_mode == kStoreBF16Tail && n0 < p.n_main)) && c0 + 32 <= BN &&
      n0 + c0 + 32 <= p.N && (p.ldc & 7) == 0 &&
      ((reinterpret_cast<uintptr_t>(static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c) & 15) == 0)) {
    // Row-major bf16 through the warp-private transpose: each store instruction writes eight
    // whole 64-byte row segments (full 32-byte sectors) instead of 32 rows' 16-byte pieces.
#pragma unroll
    for (int j = 0; j < 32; ++j) tw[lane * 33 + j] = alpha * __uint_as_float(r[j]);
    __syncwarp();
    const int cc = (lane & 3) * 8;
    __nv_bfloat16* Cz = static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int rr = q * 8 + (lane >> 2);
      const int grow = m0 + warp * 32 + rr;
      if (grow < limit) {
        const float* t = tw + rr * 33 + cc;
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(t[2 * e], t[2 * e + 1]);
          w[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(Cz + (long long)grow * p.ldc + n0 + c0 + cc) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncwarp();
    return;
  }
  if (!row_ok) return;
  const int nbase = n0 + c0;
  if (p.c_mode == kStoreBF16Tail && n0 >= p.n_main) {
    // The tail tile: token-major into C2; consecutive lanes write consecutive tokens.
    const int n2 = p.N - p.n_main;
    __nv_bfloat16* Cz = static_cast<__nv_bfloat16*>(p.C2) + (long long)(row / p.seg2) * n2 * p.seg2 +
                        row % p.seg2;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nbase - p.n_main + j;
      if (j < BN - c0 && n < n2) Cz[(long long)n * p.seg2] = __float2bfloat16(alpha * __uint_as_float(r[j]));
    }
    return;
  }
  const bool bf16_rows = p.c_mode == kStoreBF16 || p.c_mode == kStoreBF16Tail;  // tail tiles returned above
  if (p.c_mode == kSqAccF32) {  // every batch squares into the same matrix
    float* Cr = static_cast<float*>(Cbase) + (long long)row * p.ldc;
    if (c0 + 32 <= BN && nbase + 32 <= p.N && ((reinterpret_cast<uintptr_t>(Cr + nbase) & 15) == 0)) {
      float4* Cv = reinterpret_cast<float4*>(Cr + nbase);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float x0 = alpha * __uint_as_float(r[4 * q]), x1 = alpha * __uint_as_float(r[4 * q + 1]);
        const float x2 = alpha * __uint_as_float(r[4 * q + 2]), x3 = alpha * __uint_as_float(r[4 * q + 3]);
        atomicAdd(Cv + q, make_float4(x0 * x0, x1 * x1, x2 * x2, x3 * x3));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = nbase + j;
        const float x = alpha * __uint_as_float(r[j]);
        if (j < BN - c0 && n < p.N) atomicAdd(Cr + n, x * x);
      }
    }
    return;
  }
  if (p.c_mode == kStoreBF16Scatter) {
    // Row m goes home: rank scatter[m].x, row scatter[m].y of that rank's C (peer memory).
    const int2 dstm = p.scatter[row];
    __nv_bfloat16* Cr = reinterpret_cast<__nv_bfloat16*>(p.peers[dstm.x]) + (long long)dstm.y * p.ldc;
    if (c0 + 32 <= BN && nbase + 32 <= p.N && ((reinterpret_cast<uintptr_t>(Cr + nbase) & 15) == 0)) {
      uint4* Cv = reinterpret_cast<uint4*>(Cr + nbase);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(alpha * __uint_as_float(r[8 * q + 2 * e]),
                                                         alpha * __uint_as_float(r[8 * q + 2 * e + 1]));
          w[e] = *reinterpret_cast<const uint32_t*>(&h);
        }
        Cv[q] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = nbase + j;
        if (j < BN - c0 && n < p.N) Cr[n] = __float2bfloat16(alpha * __uint_as_float(r[j]));
      }
    }
  } else if (p.c_mode == kPeerSlotF32) {
    // Reduce-scatter: element i is stored (plain 16-byte peer stores, no atomics) into its
    // owner's slot for THIS rank; the owner sums its `world` slots after a barrier.
    const long long slot = 4 * p.per4;
    const long long rowoff = (long long)zc * p.batch_stride_c + (long long)row * p.ldc;
    if (c0 + 32 <= BN && nbase + 32 <= p.N && ((rowoff + nbase) & 3) == 0) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const long long i = rowoff + nbase + 4 * q;
        int owner = (int)((i >> 2) / p.per4);
        owner = owner < p.world ? owner : p.world - 1;
        float4* dst = reinterpret_cast<float4*>(p.peers[owner] + p.self_rank * slot + (i - owner * slot));
        *dst = make_float4(alpha * __uint_as_float(r[4 * q]), alpha * __uint_as_float(r[4 * q + 1]),
                           alpha * __uint_as_float(r[4 * q + 2]), alpha * __uint_as_float(r[4 * q + 3]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = nbase + j;
        if (j < BN - c0 && n < p.N) {
          const long long i = rowoff + n;
          int owner = (int)((i >> 2) / p.per4);
          owner = owner < p.world ? owner : p.world - 1;
          p.peers[owner][p.self_rank * slot + (i - owner * slot)] = alpha * __uint_as_float(r[j]);
        }
      }
    }
  } else if ((p.c_mode == kStoreF32 || p.c_mode == kAtomicF32) && c0 + 32 <= BN && nbase + 32 <= p.N &&
             ((reinterpret_cast<uintptr_t>(static_cast<float*>(Cbase) + (long long)zc * p.batch_stride_c +
                                           (long long)row * p.ldc + nbase) & 15) == 0)) {
    // A whole 32-column chunk in range and 16-byte aligned: 8 vector accesses per thread
    // instead of 32 scalar ones (the scalar form saturated the LSU pipe on large tiles).
    float4* Cv = reinterpret_cast<float4*>(static_cast<float*>(Cbase) + (long long)zc * p.batch_stride_c +
                                           (long long)row * p.ldc + nbase);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 v = make_float4(alpha * __uint_as_float(r[4 * q]), alpha * __uint_as_float(r[4 * q + 1]),
                             alpha * __uint_as_float(r[4 * q + 2]), alpha * __uint_as_float(r[4 * q + 3]));
      if (p.c_mode == kAtomicF32) {
        atomicAdd(Cv + q, v);
      } else {
        if (p.beta_accumulate) {
          const float4 o = Cv[q];
          v.x += o.x;
          v.y += o.y;
          v.z += o.z;
          v.w += o.w;
        }
        Cv[q] = v;
      }
    }
  } else if (bf16_rows && c0 + 32 <= BN && nbase + 32 <= p.N &&
             ((reinterpret_cast<uintptr_t>(static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c +
                                           (long long)row * p.ldc + nbase) & 15) == 0)) {
    uint4* Cv = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c +
                                         (long long)row * p.ldc + nbase);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(alpha * __uint_as_float(r[8 * q + 2 * e]),
                                                       alpha * __uint_as_float(r[8 * q + 2 * e + 1]));
        w[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      Cv[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else if (p.c_mode == kStoreF32 || p.c_mode == kAtomicF32) {
    float* Cz = static_cast<float*>(Cbase) + (long long)zc * p.batch_stride_c +
                (long long)row * p.ldc;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nbase + j;
      if (j < BN - c0 && n < p.N) {
        const float v = alpha * __uint_as_float(r[j]);
        if (p.c_mode == kStoreF32)
          Cz[n] = p.beta_accumulate ? Cz[n] + v : v;
        else
          atomicAdd(Cz + n, v);
      }
    }
  } else if (bf16_rows) {
    __nv_bfloat16* Cz = static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c +
                        (long long)row * p.ldc;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nbase + j;
      if (j < BN - c0 && n < p.N) Cz[n] = __float2bfloat16(alpha * __uint_as_float(r[j]));
    }
  } else if (p.c_mode == kStoreBF16T) {  // C^T[z][n][m]; consecutive lanes hit consecutive m
    __nv_bfloat16* Cz = static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nbase + j;
      if (j < BN - c0 && n < p.N)
        Cz[(long long)n * p.ldc + row] = __float2bfloat16(alpha * __uint_as_float(r[j]));
    }
  } else {  // kStoreBF16TB: rows are (segment, t); element (m, n) -> C[m / T][n][m % T], T = ldc
    __nv_bfloat16* Cz = static_cast<__nv_bfloat16*>(Cbase) + (long long)zc * p.batch_stride_c +
                        (long long)(row / p.ldc) * p.N * p.ldc + row % p.ldc;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = nbase + j;
      if (j < BN - c0 && n < p.N) Cz[(long long)n * p.ldc] = __float2bfloat16(alpha * __uint_as_float(r[j]));
    }
  }
}

// One CTA's 128 x BN output tile of batch (za, zb) -> output batch zc at Cbase.  The tensor
// maps may live in kernel parameters or in global memory (grouped launches).
//   b_row_off: subtracted from n0 in B's TMA coordinate (B rows owned by one peer's shard)
//   kpeers / kshard: B's K range is spread over peers, kshard columns each (per-stage map)
//   stage: B is the local staging copy of peer shards being filled by this very launch
//          (see gemm_staged_kernel); tiles of the own shard come from stage->own instead
template <int BN>
__device__ __forceinline__ void gemm_cta(const CUtensorMap* tmA, const CUtensorMap* tmB, const GemmParams& p,
                                         int za, int zb, int zc, int split, void* Cbase, int b_row_off = 0,
                                         const CUtensorMap* kpeers = nullptr, int kshard = 0,
                                         const StageCtl* stage = nullptr, int m0_override = -1,
                                         int row_limit = -1) {
  using C = Cfg<BN>;
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
  const int n0 = blockIdx.x * BN;
  const int m0 = m0_override >= 0 ? m0_override : blockIdx.y * BM;

  const int kblocks = (p.K + BK - 1) / BK;
  const int per = (kblocks + p.splits - 1) / p.splits;
  const int kb0 = split * per;
  const int kb1 = min(kblocks, kb0 + per);
  const int nk = max(0, kb1 - kb0);

  if (threadIdx.x == 0) {
    tma_prefetch_desc(tmA);
    if (kpeers == nullptr) tma_prefetch_desc(tmB);
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
    // ---- TMA producer ----
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1;
      if (!mbar_wait(&empty[s], ph ^ 1, p.err, kErrWaitEmpty)) break;
      mbar_arrive_expect_tx(&full[s], C::kTileA + C::kTileB);
      const int kc = (kb0 + i) * BK;
      tma_load_3d(sA + s * C::kTileA, tmA, &full[s], kc, m0, za);
      if (stage != nullptr) {
        // mode 0: the CTA's B rows belong to one owner; mode 1: the K block's owner.
        const int owner = stage->mode == 0 ? n0 / stage->shard : kc / stage->shard;
        if (owner == stage->self) {
          if (stage->mode == 0)
            tma_load_3d(sB + s * C::kTileB, stage->own, &full[s], kc, n0 - owner * stage->shard, zb);
          else
            tma_load_3d(sB + s * C::kTileB, stage->own, &full[s], kc - owner * stage->shard, n0, zb);
        } else {
          if (!(stage->ready >> owner & 1u)) {
            stage_wait(stage->flags + owner, stage->expect, p.err);
            const_cast<StageCtl*>(stage)->ready |= 1u << owner;
          }
          tma_load_3d(sB + s * C::kTileB, tmB, &full[s], kc, n0, zb);
        }
      } else if (kpeers != nullptr) {
        const int owner = kc / kshard;
        tma_load_3d(sB + s * C::kTileB, kpeers + owner, &full[s], kc - owner * kshard, n0, zb);
      } else {
        tma_load_3d(sB + s * C::kTileB, tmB, &full[s], kc, n0 - b_row_off, zb);
      }
      issued = i + 1;
    }
    // Never leave with a bulk copy still landing in this CTA's shared memory.
    for (int i = max(0, issued - C::kStages); i < issued; ++i)
      mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1, p.err, kErrWaitFull);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kStages;
      const uint32_t ph = (i / C::kStages) & 1;
      if (!mbar_wait(&full[s], ph, p.err, kErrWaitFull)) break;
      tc_fence_after();
      const uint64_t da = smem_desc_kmajor_sw128(sA + s * C::kTileA);
      const uint64_t db = smem_desc_kmajor_sw128(sB + s * C::kTileB);
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        tc_mma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i | k) != 0);
      tc_commit(&empty[s]);
    }
    tc_commit(done);
  }
  __syncwarp();

  // ---- epilogue: warp w owns accumulator rows [32w, 32w+32) ----
  const bool ok = nk > 0 ? mbar_wait(done, 0, p.err, kErrWaitDone) : true;
  __syncwarp();
  tc_fence_after();
  // Cluster split-K: the peer CTA (rank 1) writes its fp32 partial tile into rank 0's shared
  // memory (column-major, so a warp's 32 rows are 32 consecutive words), then both meet at a
  // cluster barrier and rank 0 stores the sum.
  const bool clustered = p.cluster_k > 1;
  const uint32_t crank = clustered ? cluster_ctarank() : 0u;
  float* red = reinterpret_cast<float*>(smem + C::kStages * (C::kTileA + C::kTileB) + 256);
  const int red_row = warp * 32 + lane;
  if (clustered && crank != 0) {
    const uint32_t dst = map_shared_rank(smem_u32(red), 0);
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      if (nk > 0) {
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
        tmem_ld_wait();
      }
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < BN - c0) st_cluster_f32(dst + (uint32_t)(((c0 + j) * BM + red_row) * 4),
                                        (nk > 0 && ok) ? __uint_as_float(r[j]) : 0.f);
    }
  }
  if (clustered) {
    __syncwarp();
    cluster_sync_all();
  }
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    if (clustered && crank != 0) break;
    uint32_t r[32];
    if (nk > 0) {
      tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
      tmem_ld_wait();
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = 0u;
    }
    if (clustered) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < BN - c0) r[j] = __float_as_uint(__uint_as_float(r[j]) + red[(c0 + j) * BM + red_row]);
    }
    if (!ok) continue;
    store_chunk<BN>(p, r, Cbase, zc, m0, n0, c0, warp, lane, row_limit >= 0 ? row_limit : p.M,
                    reinterpret_cast<float*>(smem) + warp * (32 * 33));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, C::kTmemCols);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, BN <= 128 ? 2 : 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   GemmParams p) {
  const int z = blockIdx.z / p.splits;
  const int split = blockIdx.z % p.splits;
  gemm_cta<BN>(&tmA, &tmB, p, z, p.b_shared ? 0 : z, z, split, p.C);
}

// One launch that all-gathers sharded B into a local staging buffer AND multiplies: the
// first `copiers` CTAs first pull their share of the remote shards over NVLink (16-byte
// peer loads, every remote byte once) into `StageArgs::dst`, bumping the owner's flag after
// each piece; then every CTA runs its GEMM tile, waiting for a remote owner's flag only
// when it first needs that owner's rows (mode 0) or K range (mode 1).  Tiles of the own
// shard never wait.  Copiers are the lowest CTA indices, which are dispatched first, so no
// resident CTA waits on a CTA that has not started; the waits are bounded regardless.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_staged_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmStage,
                       const __grid_constant__ CUtensorMap tmOwn, GemmParams p, StageArgs sa) {
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (cta < sa.copiers) {
    const int pieces = sa.pieces_per_owner;
    const int total = pieces * sa.world;
    for (int t = cta; t < total; t += sa.copiers) {
      const int owner = t / pieces, piece = t - owner * pieces;
      if (owner == sa.self) continue;
      const int r0 = piece * sa.piece_rows;
      const int r1 = min(sa.src_rows, r0 + sa.piece_rows);
      const long long vec_per_row = sa.row_elems / 8;
      const long long nvec = (long long)(r1 - r0) * vec_per_row;
      const uint4* src = reinterpret_cast<const uint4*>(sa.src[owner]);
      uint4* dst = reinterpret_cast<uint4*>(sa.dst);
      // Four 16-byte peer loads in flight per thread before their stores.
      for (long long v0 = threadIdx.x; v0 < nvec; v0 += 4 * kThreads) {
        uint4 x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long v = v0 + u * kThreads;
          if (v < nvec) {
            const long long r = r0 + v / vec_per_row, c = v % vec_per_row;
            x[u] = src[(r * sa.src_stride) / 8 + c];
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long v = v0 + u * kThreads;
          if (v < nvec) {
            const long long r = r0 + v / vec_per_row, c = v % vec_per_row;
            dst[((sa.dst_row0[owner] + r) * sa.dst_stride + sa.dst_col0[owner]) / 8 + c] = x[u];
          }
        }
      }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) atomicAdd(sa.flags + owner, 1);
    }
  }
  StageCtl sc;
  sc.own = &tmOwn;
  sc.flags = sa.flags;
  sc.expect = sa.expect;
  sc.mode = sa.mode;
  sc.self = sa.self;
  sc.shard = sa.shard;
  sc.ready = 0u;
  gemm_cta<BN>(&tmA, &tmStage, p, 0, 0, 0, 0, p.C, 0, nullptr, 0, &sc);
}

// ---------------------------------------------------------------------------------------
// Persistent GEMM: one CTA per SM walks a list of 128 x BN output tiles.  Warp roles:
//   warps 0-3  epilogue (TMEM lanes 0-127), warp 4 TMA producer, warp 5 MMA issuer.
// Two TMEM accumulators alternate between tiles, so the epilogue of tile i (TMEM -> registers
// -> global / peer memory) runs while the MMAs of tile i + 1 fill the other accumulator, and
// the stage ring of shared memory runs on across tile boundaries.  Barriers:
//   full[s] / empty[s]   TMA -> MMA / MMA -> TMA per stage;
//   acc_full[b]          MMA -> epilogue (tcgen05.commit after the tile's last K block);
//   acc_empty[b]         epilogue -> MMA (one arrival per epilogue warp).
// Every wait is bounded; a role whose wait gives up leaves its loop (the others then give up
// on their next wait), so an error costs a few seconds at most and never hangs the GPU.
// ---------------------------------------------------------------------------------------
constexpr int kPThreads = 192;

template <int BN>
struct PCfg {
  static constexpr int kTileA = BM * BK * 2;
  static constexpr int kTileB = BN * BK * 2;
  static constexpr int kTw = 4 * 32 * 33 * 4;  // epilogue transpose scratch (4 warps)
  static constexpr int kStages = (220 * 1024 - kTw) / (kTileA + kTileB);
  static constexpr int kSmem = kStages * (kTileA + kTileB) + kTw + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kTmemCols = 2 * BN;
};

// Tile list: dense (tiles_n x tiles_m x batch, n fastest) or, with tile_prefix, the ragged
// row segments of `jobs` expert groups: 256-row block t belongs to the job j with
// tile_prefix[j] <= t < tile_prefix[j + 1] (device tables; tile_prefix counts 256-row
// blocks, the unit of the CTA-pair kernel).
struct TileSched {
  int tiles_n, tiles_m, batch;
  const int* tile_prefix;
  const int* base;
  const int* len;
  int jobs;
  int n_rot;    // dense tiles: column-tile index rotation (a sharded B's own columns first)
  int n_major;  // dense tiles: column tile is the slow index (all row blocks of one B tile in turn)
  int tail_w;   // CTA-pair kernel: width of the last column tile when N is not a multiple of the
                // tile width (a multiple of 32, >= 64; 0 = every tile is full width)
  int tile_w;   // CTA-pair kernel: column tile width, 256 (0 means 256) or 128
  // Stream-K tail (CTA-pair kernel, dense tiles): the last sk_tiles tiles run as two K halves
  // on two pairs in the same wave.  The first half stores its fp32 partial in sk_ws (one
  // 256 x 256 block per split tile) and sets its warps' flags to sk_epoch; the second half
  // waits for them (bounded), adds the partial and runs the epilogue.
  int sk_tiles;
  float* sk_ws;
  int* sk_flags;  // split tile x 8 (CTA rank x epilogue warp), monotonic epochs
  int sk_epoch;
  // Split-K with atomic epilogues (kAtomicF32): every tile runs as ksplit units over disjoint
  // K ranges, each adding its partial into C.  0 or 1 = off.
  int ksplit;
  // Symmetric product (C = A A^T, kAtomicF32, dense, one batch): only the tiles on and above
  // the diagonal run; an off-diagonal tile adds its transpose below the diagonal as well.
  int sym;
};

// A pair kernel work unit: a whole tile (role 0) or a K half of a stream-K tile (role 1: the
// first half, which hands its partial over; role 2: the second half, which finishes the tile).
struct PairUnit {
  int tile, k_lo, k_hi, role, sk;
};

__device__ __forceinline__ PairUnit pair_unit(const TileSched& ts, int total_tiles, int kblocks, int u) {
  PairUnit w;
  if (ts.ksplit > 1) {
    const int part = u % ts.ksplit;
    w.tile = u / ts.ksplit;
    w.k_lo = (int)((long long)kblocks * part / ts.ksplit);
    w.k_hi = (int)((long long)kblocks * (part + 1) / ts.ksplit);
    w.role = 0;
    w.sk = -1;
    return w;
  }
  const int dp = total_tiles - ts.sk_tiles;
  if (u < dp) {
    w.tile = u;
    w.k_lo = 0;
    w.k_hi = kblocks;
    w.role = 0;
    w.sk = -1;
  } else {
    const int v = u - dp, half = v & 1, kh = kblocks >> 1;
    w.sk = v >> 1;
    w.tile = dp + w.sk;
    w.k_lo = half ? kh : 0;
    w.k_hi = half ? kblocks : kh;
    w.role = 1 + half;
  }
  return w;
}

struct TileCoord {
  int m0, n0, za, zb, zc, limit;
  int w;  // CTA-pair kernel: columns of this tile (256, or tail_w for the last column tile)
};

template <int BN>
__device__ __forceinline__ TileCoord decode_tile(const TileSched& ts, const GemmParams& p, int tile) {
  TileCoord c;
  const int rest = tile / ts.tiles_n;
  c.n0 = (tile - rest * ts.tiles_n) * BN;
  if (ts.tile_prefix != nullptr) {
    // the tables count 256-row blocks; this kernel's 128-row tiles are their halves
    const int blk = rest >> 1;
    int lo = 0, hi = ts.jobs - 1;  // largest j with tile_prefix[j] <= blk
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (ts.tile_prefix[mid] <= blk) lo = mid;
      else hi = mid - 1;
    }
    c.m0 = ts.base[lo] + (blk - ts.tile_prefix[lo]) * 2 * BM + (rest & 1) * BM;
    c.za = 0;
    c.zb = lo;
    c.zc = 0;
    c.limit = ts.base[lo] + ts.len[lo];
  } else {
    const int z = rest / ts.tiles_m;
    c.m0 = (rest - z * ts.tiles_m) * BM;
    c.za = z;
    c.zb = p.b_shared ? 0 : z;
    c.zc = z;
    c.limit = p.M;
  }
  return c;
}

template <int BN>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           GemmParams p, TileSched ts) {
  using C = PCfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (sbase & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kTileA;
  float* tw = reinterpret_cast<float*>(sB + S * C::kTileB);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(tw) + C::kTw);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblocks = (p.K + BK - 1) / BK;
  const int total = ts.tile_prefix != nullptr ? ts.tile_prefix[ts.jobs] * 2 * ts.tiles_n
                                              : ts.tiles_n * ts.tiles_m * ts.batch;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ---- TMA producer ----
      int g = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < total && alive; tile += gridDim.x) {
        const TileCoord c = decode_tile<BN>(ts, p, tile);
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % S;
          if (!mbar_wait(&empty[s], ((g / S) & 1) ^ 1, p.err, kErrWaitEmpty)) {
            alive = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::kTileA + C::kTileB);
          tma_load_3d(sA + s * C::kTileA, &tmA, &full[s], kb * BK, c.m0, c.za);
          tma_load_3d(sB + s * C::kTileB, &tmB, &full[s], kb * BK, c.n0, c.zb);
          ++g;
        }
      }
      // Never leave with a bulk copy still landing in this CTA's shared memory.
      for (int i = max(0, g - S); i < g; ++i) mbar_wait(&full[i % S], (i / S) & 1, p.err, kErrWaitFull);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      int g = 0, it = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < total && alive; tile += gridDim.x, ++it) {
        const int b = it & 1;
        if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1, p.err, kErrWaitDone)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int kb = 0; kb < kblocks; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(&full[s], (g / S) & 1, p.err, kErrWaitFull)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_kmajor_sw128(sA + s * C::kTileA);
          const uint64_t db = smem_desc_kmajor_sw128(sB + s * C::kTileB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) tc_mma_f16(d, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          tc_commit(&empty[s]);
        }
        tc_commit(&acc_full[b]);
      }
    }
  } else {
    // ---- epilogue (warps 0-3: TMEM lanes 32w .. 32w + 31) ----
    float* twp = tw + warp * (32 * 33);
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const TileCoord c = decode_tile<BN>(ts, p, tile);
      const int b = it & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (it >> 1) & 1, p.err, kErrWaitDone));
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * BN + c0), r);
        tmem_ld_wait();
        if (c0 + 32 >= BN) {
          // the accumulator is in registers: hand it back to the MMA warp before the last stores
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        store_chunk<BN>(p, r, p.C, c.zc, c.m0, c.n0, c0, warp, lane, c.limit, twp);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, C::kTmemCols);
}

// ---------------------------------------------------------------------------------------
// CTA-pair persistent GEMM (cta_group::2): each cluster of two CTAs on two SMs owns 256 x 256
// output tiles.  Each CTA loads 128 rows of A and 128 rows of B per stage (32 KB instead of
// the 48 KB a 128 x 256 single-SM tile needs for the same MMA work per SM), CTA 0 issues one
// M=256, N=256 MMA per K step over both CTAs' shared memory, and each CTA's epilogue drains
// its own 128 accumulator rows from its own TMEM.  Barriers as in gemm_persistent_kernel, with
// the stage "full" barriers and the accumulator "empty" barriers living in CTA 0: both CTAs'
// TMA loads complete on CTA 0's full barrier (CTA 0 expects the bytes of both), and both
// CTAs' epilogue warps arrive on CTA 0's accumulator-empty barrier; CTA 0's commits arrive on
// the stage-empty and accumulator-full barriers of both CTAs.
// ---------------------------------------------------------------------------------------
struct PairCfg {
  static constexpr int kTileA = 128 * BK * 2;
  static constexpr int kTileB = 128 * BK * 2;
  static constexpr int kTw = 4 * 32 * 33 * 4;
  static constexpr int kStages = (220 * 1024 - kTw) / (kTileA + kTileB);
  static constexpr int kSmem = kStages * (kTileA + kTileB) + kTw + 1024 + 256;
  static constexpr int kTmemCols = 512;  // two 256-column accumulators
};

__device__ __forceinline__ TileCoord decode_pair_tile(const TileSched& ts, const GemmParams& p, int tile) {
  TileCoord c;
  int rest, tn;
  if (ts.sym) {  // upper triangle, row by row: (0,0) (0,1) .. (0,T-1) (1,1) ..
    int tm = 0, left = tile;
    while (left >= ts.tiles_n - tm) {
      left -= ts.tiles_n - tm;
      ++tm;
    }
    c.m0 = tm * 256;
    c.n0 = (tm + left) * 256;
    c.w = (ts.tail_w != 0 && tm + left == ts.tiles_n - 1) ? ts.tail_w : 256;
    c.za = c.zb = c.zc = 0;
    c.limit = p.M;
    return c;
  }
  if (ts.n_major) {  // dense only: tile = tn * (tiles_m * batch) + rest
    const int rows = ts.tiles_m * ts.batch;
    tn = tile / rows;
    rest = tile - tn * rows;
  } else {
    rest = tile / ts.tiles_n;
    tn = tile - rest * ts.tiles_n;
  }
  tn += ts.n_rot;
  if (tn >= ts.tiles_n) tn -= ts.tiles_n;
  const int tile_w = ts.tile_w != 0 ? ts.tile_w : 256;
  c.n0 = tn * tile_w;
  c.w = (ts.tail_w != 0 && tn == ts.tiles_n - 1) ? ts.tail_w : tile_w;
  if (ts.tile_prefix != nullptr) {
    int lo = 0, hi = ts.jobs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (ts.tile_prefix[mid] <= rest) lo = mid;
      else hi = mid - 1;
    }
    c.m0 = ts.base[lo] + (rest - ts.tile_prefix[lo]) * 256;
    c.za = 0;
    c.zb = lo;
    c.zc = 0;
    c.limit = ts.base[lo] + ts.len[lo];
  } else {
    const int z = rest / ts.tiles_m;
    c.m0 = (rest - z * ts.tiles_m) * 256;
    c.za = z;
    c.zb = p.b_shared ? 0 : z;
    c.zc = z;
    c.limit = p.M;
  }
  return c;
}

// kStaged: B is a sharded weight being all-gathered by this very launch (the FSDP forward /
// input-gradient GEMM): before their epilogues, the epilogue warps of every CTA copy pieces of
// the remote shards over NVLink (16-byte peer loads) into the local staging matrix that tmB
// maps, bumping the owner's flag after each piece; the producer reads its own shard in place
// (tmOwn) and waits (bounded) for a remote owner's flag the first time it needs that owner's
// rows (mode 0) or K range (mode 1).  Own-shard work is ordered first (column tiles rotated in
// mode 0, the K loop rotated in mode 1), so the copies overlap the first tiles' MMAs.
template <bool kStaged>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     GemmParams p, TileSched ts, const __grid_constant__ CUtensorMap tmOwn, StageArgs sa) {
  using C = PairCfg;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (sbase & 1023)) & 1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kTileA;
  float* tw = reinterpret_cast<float*>(sB + S * C::kTileB);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(tw) + C::kTw);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1;
  const int pairs = gridDim.x >> 1;
  const int kblocks = (p.K + BK - 1) / BK;
  const int total_tiles = ts.sym ? ts.tiles_n * (ts.tiles_n + 1) / 2
                          : ts.tile_prefix != nullptr ? ts.tile_prefix[ts.jobs] * ts.tiles_n
                                                      : ts.tiles_n * ts.tiles_m * ts.batch;
  // work units: a stream-K tile counts twice, a split-K tile ksplit times
  const int total = ts.ksplit > 1 ? total_tiles * ts.ksplit : total_tiles + ts.sk_tiles;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (kStaged) tma_prefetch_desc(&tmOwn);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // four epilogue warps in each CTA of the pair
    }
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc_pair(tmem_slot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before either CTA signals the other
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs) ----
      int g = 0;
      bool alive = true;
      unsigned ready = 0u;  // staged: remote owners already waited for
      const int kb_rot = (kStaged && sa.mode == 1) ? (sa.self * sa.shard) / BK : 0;
      // B rows staged per CTA and k-step: half the tile width (the tensor map's box height)
      const uint32_t tx_bytes = 2u * (uint32_t)(C::kTileA + ((ts.tile_w != 0 ? ts.tile_w : 256) / 2) * BK * 2);
      const int own_lo = kStaged ? sa.self * sa.shard : 0;
      for (int u = pair; u < total && alive; u += pairs) {
        const PairUnit un = pair_unit(ts, total_tiles, kblocks, u);
        const TileCoord c = decode_pair_tile(ts, p, un.tile);
        // cta_group::2 splits the tile's N columns over the pair: each CTA stages w / 2 rows of B
        const int brow = c.n0 + (c.w >> 1) * (int)rank;
        // mode 0: this CTA's B rows belong to one owner for the whole tile
        const CUtensorMap* bmap = &tmB;
        int brow_map = brow;
        int bz = c.zb;
        if constexpr (!kStaged) {
          if (p.c_mode == kStoreBF16Tail && c.n0 >= p.n_main) {  // the tail tile reads the second B
            bmap = &tmOwn;
            brow_map = brow - p.n_main;
            bz = 0;
          }
        }
        if constexpr (kStaged) {
          if (sa.mode == 0) {
            if (brow >= own_lo && brow < own_lo + sa.shard) {
              bmap = &tmOwn;
              brow_map = brow - own_lo;
            } else {
              const int owner = brow / sa.shard;
              if (owner < sa.world && !(ready >> owner & 1u)) {
                stage_wait(sa.flags + owner, sa.expect, p.err);
                ready |= 1u << owner;
              }
            }
          }
        }
        for (int i = un.k_lo; i < un.k_hi; ++i) {
          const int s = g % S;
          if (!mbar_wait(&empty[s], ((g / S) & 1) ^ 1, p.err, kErrWaitEmpty)) {
            alive = false;
            break;
          }
          int kb = i + kb_rot;
          if (kb >= kblocks) kb -= kblocks;
          const int kc = kb * BK;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], tx_bytes);
          const uint32_t bar = map_shared_rank(smem_u32(&full[s]), 0);
          tma_load_3d_pair(sA + s * C::kTileA, &tmA, bar, kc, c.m0 + 128 * (int)rank, c.za);
          if constexpr (kStaged) {
            if (sa.mode == 0) {
              tma_load_3d_pair(sB + s * C::kTileB, bmap, bar, kc, brow_map, 0);  // rows past N: zero fill
            } else if (kc >= own_lo && kc < own_lo + sa.shard) {
              tma_load_3d_pair(sB + s * C::kTileB, &tmOwn, bar, kc - own_lo, brow, 0);
            } else {
              const int owner = kc / sa.shard;
              if (!(ready >> owner & 1u)) {
                stage_wait(sa.flags + owner, sa.expect, p.err);
                ready |= 1u << owner;
              }
              tma_load_3d_pair(sB + s * C::kTileB, &tmB, bar, kc, brow, 0);
            }
          } else {
            tma_load_3d_pair(sB + s * C::kTileB, bmap, bar, kc, brow_map, bz);  // rows past the end: zero fill
          }
          ++g;
        }
      }
      // CTA 0's full barriers count both CTAs' bytes: once they complete, nothing is landing
      // in either CTA's shared memory (CTA 1 waits for this at the closing cluster barrier).
      if (rank == 0)
        for (int i = max(0, g - S); i < g; ++i) mbar_wait(&full[i % S], (i / S) & 1, p.err, kErrWaitFull);
    }
  } else if (warp == 5) {
    if (lane == 0 && rank == 0) {
      // ---- MMA issuer (CTA 0) ----
      int g = 0, it = 0;
      bool alive = true;
      for (int u = pair; u < total && alive; u += pairs, ++it) {
        const int b = it & 1;
        const PairUnit un = pair_unit(ts, total_tiles, kblocks, u);
        const uint32_t idesc = idesc_bf16_f32(256, decode_pair_tile(ts, p, un.tile).w);
        if (!mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1, p.err, kErrWaitDone)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * 256);
        for (int kb = un.k_lo; kb < un.k_hi; ++kb, ++g) {
          const int s = g % S;
          if (!mbar_wait(&full[s], (g / S) & 1, p.err, kErrWaitFull)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_kmajor_sw128(sA + s * C::kTileA);
          const uint64_t db = smem_desc_kmajor_sw128(sB + s * C::kTileB);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_f16_pair(d, da + 2 * k, db + 2 * k, idesc, ((kb - un.k_lo) | k) != 0);
          tc_commit_pair(&empty[s]);
        }
        tc_commit_pair(&acc_full[b]);
      }
    }
  } else {
    // ---- epilogue (both CTAs; warps 0-3 drain this CTA's 128 accumulator rows) ----
    if constexpr (kStaged) {
      // First the staging copy: pieces of the remote shards, spread over every CTA.
      const int pieces = sa.pieces_per_owner;
      const int all = pieces * sa.world;
      const int et = threadIdx.x;  // 0..127
      for (int t = blockIdx.x; t < all; t += gridDim.x) {
        const int owner = t / pieces, piece = t - owner * pieces;
        if (owner == sa.self) continue;
        const int r0 = piece * sa.piece_rows;
        const int r1 = min(sa.src_rows, r0 + sa.piece_rows);
        const unsigned vec_per_row = (unsigned)(sa.row_elems / 8);
        const unsigned nvec = (unsigned)(r1 - r0) * vec_per_row;  // one piece: far below 2^32
        const uint4* src = reinterpret_cast<const uint4*>(sa.src[owner]) + (long long)r0 * (sa.src_stride / 8);
        uint4* dst = reinterpret_cast<uint4*>(sa.dst) +
                     ((sa.dst_row0[owner] + r0) * sa.dst_stride + sa.dst_col0[owner]) / 8;
        const long long sstride = sa.src_stride / 8, dstride = sa.dst_stride / 8;
        for (unsigned v0 = et; v0 < nvec; v0 += 4 * 128) {
          uint4 x[4];
          unsigned rr[4], cc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const unsigned v = v0 + u * 128;
            rr[u] = v / vec_per_row;
            cc[u] = v - rr[u] * vec_per_row;
            if (v < nvec) x[u] = src[rr[u] * sstride + cc[u]];
          }
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (v0 + u * 128 < nvec) dst[rr[u] * dstride + cc[u]] = x[u];
        }
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps only
        if (et == 0) atomicAdd(sa.flags + owner, 1);
      }
    }
    float* twp = tw + warp * (32 * 33);
    int it = 0;
    for (int u = pair; u < total; u += pairs, ++it) {
      const PairUnit un = pair_unit(ts, total_tiles, kblocks, u);
      const TileCoord c = decode_pair_tile(ts, p, un.tile);
      const int b = it & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (it >> 1) & 1, p.err, kErrWaitDone));
      if (!ok) break;
      tc_fence_after();
      // stream-K: this thread's row of the split tile's fp32 partial, and its warp's flag
      float* part = un.sk >= 0 ? ts.sk_ws + (long long)un.sk * 65536 + (long long)(rank * 128 + warp * 32 + lane) * 256
                               : nullptr;
      int* flag = un.sk >= 0 ? ts.sk_flags + un.sk * 8 + rank * 4 + warp : nullptr;
      if (un.role == 2) {
        if (lane == 0) stage_wait(flag, ts.sk_epoch, p.err);
        __syncwarp();
      }
#pragma unroll 1
      for (int c0 = 0; c0 < c.w; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(b * 256 + c0), r);
        tmem_ld_wait();
        if (c0 + 32 >= c.w) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(map_shared_rank(smem_u32(&acc_empty[b]), 0));
        }
        if (un.role == 1) {  // hand the first K half over: fp32, one 128-byte row segment per thread
          float4* dst = reinterpret_cast<float4*>(part + c0);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
          continue;
        }
        if (un.role == 2) {
          const float4* src = reinterpret_cast<const float4*>(part + c0);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 v = src[q];
            r[4 * q] = __float_as_uint(__uint_as_float(r[4 * q]) + v.x);
            r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + v.y);
            r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + v.z);
            r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + v.w);
          }
        }
        store_chunk<256>(p, r, p.C, c.zc, c.m0 + 128 * (int)rank, c.n0, c0, warp, lane, c.limit, twp);
        if (ts.sym && c.m0 != c.n0) {  // the mirrored block below the diagonal (atomic fp32)
          const int row = c.m0 + 128 * (int)rank + warp * 32 + lane;
          float* Cf = static_cast<float*>(p.C);
          if (row < p.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int n = c.n0 + c0 + j;  // consecutive lanes add consecutive rows' entries
              if (n < p.N) atomicAdd(Cf + (long long)n * p.ldc + row, p.alpha * __uint_as_float(r[j]));
            }
          }
        }
      }
      if (un.role == 1) {  // publish: the partial's stores before the flag (release, GPU scope)
        __threadfence();
        __syncwarp();
        if (lane == 0) asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(flag), "r"(ts.sk_epoch) : "memory");
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while its partner may still signal its barriers
  tc_fence_after();
  if (warp == 5) tmem_dealloc_pair(tmem, C::kTmemCols);
}

// B held by the peers (sharded weights, read over NVLink through per-peer tensor maps in the
// kernel's parameters; no multicast).  mode 0: peer r owns B rows [r*shard, (r+1)*shard)
// (the forward GEMM of a row-sharded weight); mode 1: peer r owns B's K columns
// [r*shard, (r+1)*shard) (the input-gradient GEMM against the transposed shards).
template <int BN>
__global__ void __launch_bounds__(kThreads, BN <= 128 ? 2 : 1)
    gemm_peers_kernel(const __grid_constant__ CUtensorMap tmA, const CUtensorMap* __restrict__ pm,
                      GemmParams p, int mode, int shard) {
  const int z = blockIdx.z / p.splits;
  const int split = blockIdx.z % p.splits;
  if (mode == 0) {
    const int owner = (int)(blockIdx.x * BN) / shard;
    gemm_cta<BN>(&tmA, pm + owner, p, z, 0, z, split, p.C, owner * shard);
  } else {
    gemm_cta<BN>(&tmA, pm, p, z, 0, z, split, p.C, 0, pm, shard);
  }
}

// Grouped launch: CTA z serves job z / batch, batch z % batch of that job; every job has
// the same M, N, K, batch and store mode, its own operands (tensor maps in global memory,
// 64-byte aligned, written before the launch) and output.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_grouped_kernel(const GroupJob* __restrict__ jobs, GemmParams p) {
  const int job = blockIdx.z / p.batch;
  const int b = blockIdx.z % p.batch;
  const GroupJob j = jobs[job];
  gemm_cta<BN>(j.ta, j.tb, p, b, p.b_shared ? 0 : b, b, 0, j.C);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (fn == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
  return fn;
}

template <int BN>
void launch_bn(const GemmOperand& A, const GemmOperand& B, const GemmParams& p,
               cudaStream_t stream) {
  using C = Cfg<BN>;
  CUtensorMap ta = make_tmap_kmajor_bf16(A, BM);
  CUtensorMap tb = make_tmap_kmajor_bf16(B, BN);
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(gemm_tn_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         C::kClusterOK ? C::kSmem + C::kRed : C::kSmem);
    configured |= 1ull << dev;
  }
  GemmParams q = p;
  // A skinny problem (few output tiles, long K) leaves most SMs idle: split K over a
  // 2-CTA cluster that sums through distributed shared memory (no atomics, no extra pass).
  const long long tiles = (long long)((p.N + BN - 1) / BN) * ((p.M + BM - 1) / BM) * p.batch;
  const int kblocks = (p.K + BK - 1) / BK;
  q.cluster_k = 1;
  if (C::kClusterOK && p.splits == 1 && p.c_mode != kAtomicF32 &&
      p.c_mode != kStoreBF16Scatter &&
      tiles * 2 <= 160 && kblocks >= 8) {
    q.cluster_k = 2;
    q.splits = 2;
  }
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, p.batch * q.splits);
  if (q.cluster_k == 1) {
    gemm_tn_kernel<BN><<<grid, kThreads, C::kSmem, stream>>>(ta, tb, q);
    return;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmem + C::kRed;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 2;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gemm_tn_kernel<BN>, ta, tb, q);
}

template <int BN>
void launch_peers_bn(const GemmOperand& A, const CUtensorMap* pm, const GemmParams& p, int mode, int shard,
                     cudaStream_t stream) {
  using C = Cfg<BN>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(gemm_peers_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    configured |= 1ull << dev;
  }
  CUtensorMap ta = make_tmap_kmajor_bf16(A, BM);
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, p.batch * p.splits);
  gemm_peers_kernel<BN><<<grid, kThreads, C::kSmem, stream>>>(ta, pm, p, mode, shard);
}

template <int BN>
void launch_staged_bn(const GemmOperand& A, const GemmOperand& stage_op, const GemmOperand& own,
                      const GemmParams& p, const StageArgs& sa, cudaStream_t stream) {
  using C = Cfg<BN>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(gemm_staged_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    configured |= 1ull << dev;
  }
  CUtensorMap ta = make_tmap_kmajor_bf16(A, BM);
  CUtensorMap ts = make_tmap_kmajor_bf16(stage_op, BN);
  CUtensorMap to = make_tmap_kmajor_bf16(own, BN);
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, 1);
  gemm_staged_kernel<BN><<<grid, kThreads, C::kSmem, stream>>>(ta, ts, to, p, sa);
}

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (count[dev & 63] == 0) cudaDeviceGetAttribute(&count[dev & 63], cudaDevAttrMultiProcessorCount, dev);
  return count[dev & 63];
}

template <int BN>
void launch_persistent_bn(const GemmOperand& A, const GemmOperand& B, const GemmParams& p, const TileSched& ts,
                          long long max_tiles, cudaStream_t stream) {
  using C = PCfg<BN>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(gemm_persistent_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    configured |= 1ull << dev;
  }
  if (max_tiles <= 0) return;
  CUtensorMap ta = make_tmap_kmajor_bf16(A, BM);
  CUtensorMap tb = make_tmap_kmajor_bf16(B, BN);
  const int grid = (int)std::min<long long>(max_tiles, sm_count());
  gemm_persistent_kernel<BN><<<grid, kPThreads, C::kSmem, stream>>>(ta, tb, p, ts);
}

// Clusters of two resident at once for the pair kernel (its shared memory keeps one CTA per
// SM; pairs must fit inside a GPC, so this can be below half the SM count).
int pair_clusters() {
  static int count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (count[dev & 63] == 0) {
    cudaFuncSetAttribute(gemm_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::kSmem);
    cudaFuncSetAttribute(gemm_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::kSmem);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(kPThreads, 1, 1);
    cfg.dynamicSmemBytes = PairCfg::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<false>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = -1;  // clusters unavailable: callers fall back to the single-SM kernel
    }
    count[dev & 63] = n;
  }
  return count[dev & 63];
}

// Width of the last column tile of an N-wide pair GEMM: the remainder rounded up to a multiple
// of 32 (at least 64), so that a narrow remainder does not cost a whole 256-wide tile of MMAs
// (0 when N is a multiple of 256).
int pair_tail_width(int N, int tile_w = 256) {
  const int rem = N % tile_w;
  if (rem == 0) return 0;
  const int w = (rem + 31) / 32 * 32;
  return w < 64 ? 64 : w;
}

// Column tile width of a dense pair GEMM.  Measured on the bench step's shapes, 128-wide
// tiles (M = 256, N = 128 MMAs) ran 1.5-1.9x slower than 256-wide ones even where they
// quantize into fewer waves (8192 x 2048 x 2048: 96 vs 57 us), so every dense launch keeps
// 256; the width stays a kernel parameter (TileSched::tile_w).
int pair_tile_width(long long /*row_tiles*/, int /*N*/, int /*clusters*/) { return 256; }

// Stream-K tail buffers of one (device, stream): launches on one stream run in order, so they
// can share one workspace; epochs tell this launch's flags from earlier ones'.
struct SkBuffers {
  float* ws = nullptr;
  int* flags = nullptr;
  int epoch = 0;
};
constexpr int kSkMaxTiles = 64;  // 16 MiB of fp32 partials per (device, stream)
std::mutex g_sk_mutex;
std::map<std::pair<int, cudaStream_t>, SkBuffers> g_sk_buffers;

// Split the last, partly filled wave of a dense pair GEMM into K halves when that wave holds
// at most half as many tiles as there are resident pairs: its 2 * rem half-tiles then run in
// one wave of half the length (e.g. 256 tiles on 74 pairs: 3.5 waves of time instead of 4).
// Only for plain stores, K of at least eight blocks, and outside stream capture (the epoch is
// a launch argument).
void plan_stream_k(TileSched& ts, const GemmParams& p, long long tiles, int clusters, cudaStream_t stream) {
  ts.sk_tiles = 0;
  if (clusters <= 0 || tiles <= clusters) return;
  const long long rem = tiles % clusters;
  if (rem == 0 || 2 * rem > clusters || rem > kSkMaxTiles || (p.K + BK - 1) / BK < 8) return;
  if (!(p.c_mode == kStoreBF16 || p.c_mode == kStoreBF16Tail || (p.c_mode == kStoreF32 && !p.beta_accumulate)))
    return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_sk_mutex);
  SkBuffers& b = g_sk_buffers[{dev, stream}];
  if (b.ws == nullptr) {
    float* ws = nullptr;
    int* flags = nullptr;
    if (cudaMalloc(&ws, (size_t)kSkMaxTiles * 65536 * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&flags, (size_t)kSkMaxTiles * 8 * sizeof(int)) != cudaSuccess ||
        cudaMemset(flags, 0, (size_t)kSkMaxTiles * 8 * sizeof(int)) != cudaSuccess) {
      cudaGetLastError();
      if (ws != nullptr) cudaFree(ws);
      if (flags != nullptr) cudaFree(flags);
      return;  // no workspace: plain waves
    }
    b.ws = ws;
    b.flags = flags;
  }
  ts.sk_tiles = (int)rem;
  ts.sk_ws = b.ws;
  ts.sk_flags = b.flags;
  ts.sk_epoch = ++b.epoch;
}

// Launch the pair kernel on up to `max_tiles` 256 x 256 tiles; false if it cannot run here.
// `tail`: the second B operand of the kStoreBF16Tail store (nullptr otherwise).
bool launch_pair(const GemmOperand& A, const GemmOperand& B, const GemmParams& p, const TileSched& ts,
                 long long max_tiles, cudaStream_t stream, const GemmOperand* tail = nullptr) {
  const int clusters = pair_clusters();
  if (clusters <= 0) return false;
  if (max_tiles <= 0) return true;
  // The B box is half a column tile: the rows one CTA of the pair stages per k-step.
  const int bbox = (ts.tile_w != 0 ? ts.tile_w : 256) / 2;
  CUtensorMap ta = make_tmap_kmajor_bf16(A, 128);
  CUtensorMap tb = make_tmap_kmajor_bf16(B, bbox);
  CUtensorMap tt = tail != nullptr ? make_tmap_kmajor_bf16(*tail, bbox) : tb;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * (unsigned)std::min<long long>(max_tiles, clusters), 1, 1);
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = PairCfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  StageArgs none{};
  cudaLaunchKernelEx(&cfg, gemm_pair_kernel<false>, ta, tb, p, ts, tt, none);
  return true;
}

// The staged (all-gather fused) GEMM on CTA pairs; false if it cannot run here.
bool launch_pair_staged(const GemmOperand& A, const GemmOperand& stage_op, const GemmOperand& own, GemmParams p,
                        StageArgs sa, cudaStream_t stream) {
  const int clusters = pair_clusters();
  if (clusters <= 0) return false;
  TileSched ts{};
  ts.tiles_n = (p.N + 255) / 256;
  ts.tiles_m = (p.M + 255) / 256;
  ts.batch = 1;
  // mode 0: own columns first and column-major tile order, so the first wave of tiles needs
  // no remote rows at all and the copies run under it
  ts.n_rot = sa.mode == 0 ? (sa.self * sa.shard / 256) % ts.tiles_n : 0;
  ts.n_major = sa.mode == 0 ? 1 : 0;
  const long long tiles = (long long)ts.tiles_n * ts.tiles_m;
  const int n_clusters = (int)std::min<long long>(tiles, clusters);
  sa.copiers = 2 * n_clusters;
  CUtensorMap ta = make_tmap_kmajor_bf16(A, 128);
  CUtensorMap tb = make_tmap_kmajor_bf16(stage_op, 128);
  CUtensorMap to = make_tmap_kmajor_bf16(own, 128);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * (unsigned)n_clusters, 1, 1);
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = PairCfg::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, gemm_pair_kernel<true>, ta, tb, p, ts, to, sa);
  return true;
}

// max_blocks bounds the number of 256-row blocks of all jobs together.
template <int BN>
void launch_ragged_bn(const GemmOperand& A, const GemmOperand& B, const GemmParams& p, const int* tile_prefix,
                      const int* base, const int* len, int jobs, int max_blocks, cudaStream_t stream) {
  TileSched ts{};
  ts.tiles_m = 0;
  ts.batch = 1;
  ts.tile_prefix = tile_prefix;
  ts.base = base;
  ts.len = len;
  ts.jobs = jobs;
  if (BN == 256) {
    ts.tiles_n = (p.N + 255) / 256;
    ts.tail_w = pair_tail_width(p.N);
    if (launch_pair(A, B, p, ts, (long long)max_blocks * ts.tiles_n, stream)) return;
  }
  ts.tiles_n = (p.N + BN - 1) / BN;
  launch_persistent_bn<BN>(A, B, p, ts, (long long)max_blocks * 2 * ts.tiles_n, stream);
}

template <int BN>
void launch_grouped_bn(const GroupJob* jobs, int n_jobs, const GemmParams& p, cudaStream_t stream) {
  using C = Cfg<BN>;
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(gemm_grouped_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    configured |= 1ull << dev;
  }
  dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, n_jobs * p.batch);
  gemm_grouped_kernel<BN><<<grid, kThreads, C::kSmem, stream>>>(jobs, p);
}

}  // namespace

void gemm_peers_launch(const GemmOperand& A, const CUtensorMap* pm, GemmParams p, int mode, int shard, int bn,
                       cudaStream_t stream) {
  if (p.splits < 1) p.splits = 1;
  switch (bn) {
    case 16: launch_peers_bn<16>(A, pm, p, mode, shard, stream); break;
    case 32: launch_peers_bn<32>(A, pm, p, mode, shard, stream); break;
    case 64: launch_peers_bn<64>(A, pm, p, mode, shard, stream); break;
    case 128: launch_peers_bn<128>(A, pm, p, mode, shard, stream); break;
    case 256: launch_peers_bn<256>(A, pm, p, mode, shard, stream); break;
    default: throw std::runtime_error("gemm_peers: unsupported tile width");
  }
}

void gemm_staged_launch(const GemmOperand& A, const GemmOperand& stage_op, const GemmOperand& own, GemmParams p,
                        StageArgs sa, int bn, cudaStream_t stream) {
  p.splits = 1;
  p.batch = 1;
  // CTA pairs when the 128-row B halves never straddle two owners' shards.
  if (p.N > 128 && (sa.mode == 0 ? sa.shard % 128 == 0 : sa.shard % BK == 0) &&
      launch_pair_staged(A, stage_op, own, p, sa, stream))
    return;
  const int ctas = ((p.N + bn - 1) / bn) * ((p.M + BM - 1) / BM);
  sa.copiers = ctas < 148 ? ctas : 148;
  switch (bn) {
    case 64: launch_staged_bn<64>(A, stage_op, own, p, sa, stream); break;
    case 128: launch_staged_bn<128>(A, stage_op, own, p, sa, stream); break;
    case 256: launch_staged_bn<256>(A, stage_op, own, p, sa, stream); break;
    default: throw std::runtime_error("gemm_staged: unsupported tile width");
  }
}

void gemm_ragged_launch(const GemmOperand& A, const GemmOperand& B3, GemmParams p, const int* tile_prefix,
                        const int* base, const int* len, int jobs, int max_tiles, int bn, cudaStream_t stream) {
  p.splits = 1;
  p.batch = 1;
  p.b_shared = 0;
  switch (bn) {
    case 64: launch_ragged_bn<64>(A, B3, p, tile_prefix, base, len, jobs, max_tiles, stream); break;
    case 128: launch_ragged_bn<128>(A, B3, p, tile_prefix, base, len, jobs, max_tiles, stream); break;
    case 256: launch_ragged_bn<256>(A, B3, p, tile_prefix, base, len, jobs, max_tiles, stream); break;
    default: throw std::runtime_error("gemm_ragged: unsupported tile width");
  }
}

void gemm_grouped_launch(const GroupJob* jobs, int n_jobs, GemmParams p, int bn, cudaStream_t stream) {
  p.splits = 1;
  switch (bn) {
    case 16: launch_grouped_bn<16>(jobs, n_jobs, p, stream); break;
    case 32: launch_grouped_bn<32>(jobs, n_jobs, p, stream); break;
    case 64: launch_grouped_bn<64>(jobs, n_jobs, p, stream); break;
    case 128: launch_grouped_bn<128>(jobs, n_jobs, p, stream); break;
    case 256: launch_grouped_bn<256>(jobs, n_jobs, p, stream); break;
    default: throw std::runtime_error("gemm_grouped: unsupported tile width");
  }
}

CUtensorMap make_tmap_kmajor_bf16(const GemmOperand& op, int box_rows) {
  // The encoder is a driver call: make the current device's primary context current on
  // this thread first (a fresh thread -- e.g. autograd's backward worker -- whose device
  // was never switched has none yet, and the runtime only binds one lazily).
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)op.cols, (cuuint64_t)op.rows, (cuuint64_t)op.batch};
  cuuint64_t strides[2] = {(cuuint64_t)op.row_stride * 2, (cuuint64_t)op.batch_stride * 2};
  if (op.batch <= 1) strides[1] = (cuuint64_t)op.row_stride * 2 * (cuuint64_t)op.rows;
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(op.ptr),
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed (" + std::to_string((int)r) +
                             "): operand must be 16-byte aligned with 16-byte row strides");
  return map;
}

int pick_bn(int N) {
  if (N <= 16) return 16;
  if (N <= 32) return 32;
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  return 256;
}

void gram_acc_launch(const GemmOperand& At, GemmParams p, cudaStream_t stream) {
  // C (fp32, M x M) += alpha * At At^T over the upper-triangle tiles, split along K so that
  // the units fill the resident CTA pairs.
  if (At.batch != 1 || p.M != p.N) throw std::runtime_error("gram_acc: one square product");
  p.c_mode = kAtomicF32;
  p.splits = 1;
  p.batch = 1;
  p.b_shared = 1;
  TileSched ts{};
  ts.tiles_n = ts.tiles_m = (p.M + 255) / 256;
  ts.batch = 1;
  ts.sym = 1;
  ts.tail_w = pair_tail_width(p.N);
  const long long tiles = (long long)ts.tiles_n * (ts.tiles_n + 1) / 2;
  const int clusters = pair_clusters();
  const int kblocks = (p.K + BK - 1) / BK;
  long long split = clusters > 0 ? clusters / tiles : 1;
  split = std::max<long long>(1, std::min<long long>(split, kblocks / 4));
  ts.ksplit = (int)split;
  if (!launch_pair(At, At, p, ts, tiles * split, stream))
    throw std::runtime_error("gram_acc: CTA pairs cannot run on this device");
}

bool gemm_tn_tail_launch(const GemmOperand& A, const GemmOperand& B, const GemmOperand& Btail, GemmParams p,
                         cudaStream_t stream) {
  if (p.n_main % 256 != 0 || p.N - p.n_main <= 0 || p.N - p.n_main > 256 || B.rows != p.n_main ||
      Btail.rows != p.N - p.n_main || A.batch != 1 || B.batch != 1 || Btail.batch != 1 || p.seg2 <= 0 ||
      p.M % p.seg2 != 0)
    throw std::runtime_error("gemm_tn_tail: main width must be a multiple of 256, the tail 1..256 rows, one batch");
  p.c_mode = kStoreBF16Tail;
  p.splits = 1;
  p.batch = 1;
  p.b_shared = 1;
  TileSched ts{};
  ts.tiles_m = (p.M + 255) / 256;
  ts.batch = 1;
  ts.tile_w = pair_tile_width(ts.tiles_m, p.n_main, pair_clusters());
  if (p.n_main % ts.tile_w != 0 || p.N - p.n_main > ts.tile_w) ts.tile_w = 256;
  ts.tiles_n = p.n_main / ts.tile_w + 1;
  ts.tail_w = pair_tail_width(p.N - p.n_main, ts.tile_w) == 0 ? ts.tile_w
                                                                 : pair_tail_width(p.N - p.n_main, ts.tile_w);
  const long long ptiles = (long long)ts.tiles_n * ts.tiles_m;
  plan_stream_k(ts, p, ptiles, pair_clusters(), stream);
  return launch_pair(A, B, p, ts, ptiles, stream, &Btail);
}

void gemm_tn_launch(const GemmOperand& A, const GemmOperand& B, GemmParams p, int bn,
                    cudaStream_t stream) {
  if (p.splits < 1) p.splits = 1;
  // More than one wave of tiles without split-K: the persistent kernel (epilogue of one tile
  // overlapped with the MMAs of the next).
  const long long tiles = (long long)((p.N + bn - 1) / bn) * ((p.M + BM - 1) / BM) * p.batch;
  // Few tiles over a long K go to the 2-CTA cluster split-K form of the per-tile kernel (see
  // launch_bn); every other wide (N > 128) problem runs on CTA pairs.
  const bool skinny = tiles * 2 <= 160 && (p.K + BK - 1) / BK >= 8;
  if (p.splits == 1 && bn == 256 && p.K > 0 && !skinny) {
    TileSched ts{};
    ts.tiles_m = (p.M + 255) / 256;
    ts.batch = p.batch;
    ts.jobs = 0;
    ts.tile_w = pair_tile_width((long long)ts.tiles_m * p.batch, p.N, pair_clusters());
    ts.tiles_n = (p.N + ts.tile_w - 1) / ts.tile_w;
    ts.tail_w = pair_tail_width(p.N, ts.tile_w);
    // Row-block-fastest order when B is far larger than the L2 and A is not (an LM head's
    // forward): in column-fastest order every row block streams all of B from HBM again,
    // while walking all row blocks of one column tile in turn reads B once and keeps A,
    // the operand that repeats, resident in the L2.
    const double a_bytes = 2.0 * p.M * p.K, b_bytes = 2.0 * p.N * p.K;
    ts.n_major = p.batch == 1 && ts.tiles_n > ts.tiles_m && b_bytes > 64e6 && a_bytes <= 64e6 ? 1 : 0;
    const long long ptiles = (long long)ts.tiles_n * ts.tiles_m * ts.batch;
    plan_stream_k(ts, p, ptiles, pair_clusters(), stream);
    if (launch_pair(A, B, p, ts, ptiles, stream)) return;
  }
  if (p.splits == 1 && bn >= 64 && p.K > 0 && tiles > sm_count()) {
    TileSched ts{};
    ts.tiles_n = (p.N + bn - 1) / bn;
    ts.tiles_m = (p.M + BM - 1) / BM;
    ts.batch = p.batch;
    ts.jobs = 0;
    switch (bn) {
      case 64: launch_persistent_bn<64>(A, B, p, ts, tiles, stream); return;
      case 128: launch_persistent_bn<128>(A, B, p, ts, tiles, stream); return;
      case 256: launch_persistent_bn<256>(A, B, p, ts, tiles, stream); return;
      default: break;
    }
  }
  switch (bn) {
    case 16: launch_bn<16>(A, B, p, stream); break;
    case 32: launch_bn<32>(A, B, p, stream); break;
    case 64: launch_bn<64>(A, B, p, stream); break;
    case 128: launch_bn<128>(A, B, p, stream); break;
    case 256: launch_bn<256>(A, B, p, stream); break;
    default: throw std::runtime_error("gemm_tn: unsupported tile width");
  }
}

}  // namespace bw
