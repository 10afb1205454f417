// Intra-chunk part of the Mamba2 SSD scan (state-space duality), fused:
//
//     y[s] = sum_{t <= s} (C_s . B_t) exp(cum_s - cum_t) x[t]          (per chunk, per head)
//
// The PyTorch formulation materializes the decayed (chunk x chunk) matrix of every head in
// fp32 -- for Mamba2-2.7B 80 heads x 8 chunks x 256 x 256, 168 MB per layer -- and its
// backward walks it about fifteen times more.  Here the decay exp(cum_s - cum_t) is formed in
// shared memory tile by tile from the chunk's cumulative log-decay, multiplied into the
// group's C.B^T tile (shared by all heads of a group), and consumed at once:
//
//   ssd_fwd_kernel     y tile (64 rows x 64 head channels) per (chunk, head, row block)
//   ssd_bwd_dx_kernel  dx[t] = sum_{s >= t} M[s, t] dy[s]         per (chunk, head, t block)
//   ssd_bwd_dm_kernel  dM = dy x^T per (s block, t block) of the lower triangle, looping over
//                      a slice of the heads of a group: d(C.B^T) summed over those heads in
//                      registers (one atomic add per slice), and d cum from the row and column
//                      sums of dM * M
//
// with M[s, t] = (C_s . B_t) exp(cum_s - cum_t) for t <= s, 0 otherwise.  fp32 throughout
// (CUDA-core FMAs on 4 x 4 register tiles); the chunk's log-decay is non-increasing, so every
// exponent is <= 0.
#include <cuda_runtime.h>

#include "ssd.cuh"

namespace bw {
namespace {

constexpr int kP = 64;   // head channels
constexpr int kT = 64;   // rows of a tile (positions in the chunk)
constexpr int kK = 32;   // positions per inner step
constexpr int kThreads = 256;
constexpr int kHeadSplits = 8;  // d(C.B^T) CTAs per (tile pair, chunk, group): each sums a slice of the heads

__global__ void __launch_bounds__(kThreads)
    ssd_fwd_kernel(const float* __restrict__ cb, const float* __restrict__ cum, const float* __restrict__ x,
                   float* __restrict__ y, int C, int S, int H, int G) {
  __shared__ float ms[kT][kK + 1];
  __shared__ __align__(16) float xs[kK][kP];
  __shared__ float cs[kT], ct[kK];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int s0 = blockIdx.x * kT, c = blockIdx.y;
  const int b = blockIdx.z / H, h = blockIdx.z - b * H, g = h / (H / G);
  const long long hp = (long long)H * kP;
  const float* cbp = cb + (((long long)b * G + g) * C + c) * S * S;
  const float* cump = cum + (((long long)b * H + h) * C + c) * S;
  const float* xp = x + ((long long)b * C + c) * S * hp + (long long)h * kP;
  if (tid < kT) cs[tid] = cump[s0 + tid];
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int t0 = 0; t0 < s0 + kT; t0 += kK) {
    __syncthreads();  // the previous step's tiles are consumed
    if (tid < kK) ct[tid] = cump[t0 + tid];
    for (int i = tid; i < kK * kP / 4; i += kThreads) {
      const int r = i / (kP / 4), q = i - r * (kP / 4);
      reinterpret_cast<float4*>(&xs[r][0])[q] = reinterpret_cast<const float4*>(xp + (long long)(t0 + r) * hp)[q];
    }
    __syncthreads();
    for (int i = tid; i < kT * kK; i += kThreads) {
      const int r = i / kK, k = i - r * kK;
      const int s = s0 + r, t = t0 + k;
      ms[r][k] = t <= s ? cbp[(long long)s * S + t] * __expf(cs[r] - ct[k]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kK; ++k) {
      const float4 v = reinterpret_cast<const float4*>(&xs[k][0])[tx];
      const float bv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = ms[ty * 4 + i][k];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a, bv[j], acc[i][j]);
      }
    }
  }
  float* yp = y + ((long long)b * C + c) * S * hp + (long long)h * kP;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    reinterpret_cast<float4*>(yp + (long long)(s0 + ty * 4 + i) * hp)[tx] =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
}

__global__ void __launch_bounds__(kThreads)
    ssd_bwd_dx_kernel(const float* __restrict__ cb, const float* __restrict__ cum, const float* __restrict__ dy,
                      float* __restrict__ dx, int C, int S, int H, int G) {
  __shared__ float mt[kT][kK + 1];  // [t][s]
  __shared__ __align__(16) float dys[kK][kP];
  __shared__ float ctt[kT], css[kK];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int t0 = blockIdx.x * kT, c = blockIdx.y;
  const int b = blockIdx.z / H, h = blockIdx.z - b * H, g = h / (H / G);
  const long long hp = (long long)H * kP;
  const float* cbp = cb + (((long long)b * G + g) * C + c) * S * S;
  const float* cump = cum + (((long long)b * H + h) * C + c) * S;
  const float* dyp = dy + ((long long)b * C + c) * S * hp + (long long)h * kP;
  if (tid < kT) ctt[tid] = cump[t0 + tid];
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int s0 = t0; s0 < S; s0 += kK) {
    __syncthreads();
    if (tid < kK) css[tid] = cump[s0 + tid];
    for (int i = tid; i < kK * kP / 4; i += kThreads) {
      const int r = i / (kP / 4), q = i - r * (kP / 4);
      reinterpret_cast<float4*>(&dys[r][0])[q] = reinterpret_cast<const float4*>(dyp + (long long)(s0 + r) * hp)[q];
    }
    __syncthreads();
    for (int i = tid; i < kT * kK; i += kThreads) {
      const int k = i / kT, r = i - k * kT;  // consecutive threads: consecutive t (coalesced C.B^T reads)
      const int s = s0 + k, t = t0 + r;
      mt[r][k] = t <= s ? cbp[(long long)s * S + t] * __expf(css[k] - ctt[r]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < kK; ++k) {
      const float4 v = reinterpret_cast<const float4*>(&dys[k][0])[tx];
      const float bv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float a = mt[ty * 4 + i][k];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a, bv[j], acc[i][j]);
      }
    }
  }
  float* dxp = dx + ((long long)b * C + c) * S * hp + (long long)h * kP;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    reinterpret_cast<float4*>(dxp + (long long)(t0 + ty * 4 + i) * hp)[tx] =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
}

// One CTA per (lower-triangle tile pair, chunk, batch x group x head slice).  Thread (ty, tx) owns rows
// s0 + ty + 16 i and columns t0 + tx + 16 j (i, j < 4), so the x tile rows it reads differ
// by one between neighbouring lanes (conflict-free with the 65-word row pitch).
__global__ void __launch_bounds__(kThreads)
    ssd_bwd_dm_kernel(const float* __restrict__ cb, const float* __restrict__ cum, const float* __restrict__ x,
                      const float* __restrict__ dy, float* __restrict__ dcb, float* __restrict__ dcum, int C, int S,
                      int H, int G) {
  __shared__ float dys[kT][kP + 1];
  __shared__ float xs[kT][kP + 1];
  __shared__ float cs[kT], ct[kT];
  __shared__ float colsum[kThreads / 32][kT];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15, warp = tid >> 5, lane = tid & 31;
  int sb = 0;
  const int pair = blockIdx.x;
  while ((sb + 1) * (sb + 2) / 2 <= pair) ++sb;
  const int tb = pair - sb * (sb + 1) / 2;
  const int s0 = sb * kT, t0 = tb * kT, c = blockIdx.y;
  // blockIdx.z = (b * G + g) * kHeadSplits + part: each CTA takes a slice of the group's heads
  const int rep = H / G;
  const int per = (rep + kHeadSplits - 1) / kHeadSplits;
  const int part = blockIdx.z % kHeadSplits, bg = blockIdx.z / kHeadSplits;
  const int b = bg / G, g = bg - b * G;
  const int r_begin = part * per, r_end = min(rep, r_begin + per);
  const long long hp = (long long)H * kP;
  const long long cb_off = (((long long)b * G + g) * C + c) * S * S;
  float cbv[4][4], dcb_acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = s0 + ty + 16 * i, t = t0 + tx + 16 * j;
      cbv[i][j] = t <= s ? cb[cb_off + (long long)s * S + t] : 0.f;
      dcb_acc[i][j] = 0.f;
    }
  const float* xrow = x + ((long long)b * C + c) * S * hp;
  const float* dyrow = dy + ((long long)b * C + c) * S * hp;
  for (int r = r_begin; r < r_end; ++r) {
    const int h = g * rep + r;
    const float* cump = cum + (((long long)b * H + h) * C + c) * S;
    __syncthreads();  // the previous head's tiles and column sums are consumed
    for (int i = tid; i < kT * kP; i += kThreads) {
      const int row = i / kP, col = i - row * kP;
      dys[row][col] = dyrow[(long long)(s0 + row) * hp + (long long)h * kP + col];
      xs[row][col] = xrow[(long long)(t0 + row) * hp + (long long)h * kP + col];
    }
    if (tid < kT) cs[tid] = cump[s0 + tid];
    else if (tid < 2 * kT) ct[tid - kT] = cump[t0 + tid - kT];
    __syncthreads();
    float dm[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) dm[i][j] = 0.f;
#pragma unroll 4
    for (int k = 0; k < kP; ++k) {
      float a[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = dys[ty + 16 * i][k];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = xs[tx + 16 * j][k];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) dm[i][j] = fmaf(a[i], bv[j], dm[i][j]);
    }
    float rowp[4] = {0.f, 0.f, 0.f, 0.f}, colp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int s = s0 + ty + 16 * i, t = t0 + tx + 16 * j;
        if (t <= s) {
          const float decay = __expf(cs[ty + 16 * i] - ct[tx + 16 * j]);
          dcb_acc[i][j] = fmaf(dm[i][j], decay, dcb_acc[i][j]);
          const float p = dm[i][j] * cbv[i][j] * decay;
          rowp[i] += p;
          colp[j] += p;
        }
      }
    // d cum_s += sum_t P[s, t]: the 16 lanes of one ty hold one row's partials
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v = rowp[i];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tx == 0) atomicAdd(dcum + (((long long)b * H + h) * C + c) * S + s0 + ty + 16 * i, v);
    }
    // d cum_t -= sum_s P[s, t]: two ty per warp, then the eight warps through shared memory
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float v = colp[j] + __shfl_xor_sync(0xffffffffu, colp[j], 16);
      if (lane < 16) colsum[warp][tx + 16 * j] = v;
    }
    __syncthreads();
    if (tid < kT) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) v += colsum[w][tid];
      atomicAdd(dcum + (((long long)b * H + h) * C + c) * S + t0 + tid, -v);
    }
  }
  if (r_begin >= r_end) return;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = s0 + ty + 16 * i, t = t0 + tx + 16 * j;
      if (t <= s) atomicAdd(dcb + cb_off + (long long)s * S + t, dcb_acc[i][j]);  // one add per head slice
    }
}

}  // namespace

void ssd_intra_fwd(const float* cb, const float* cum, const float* x, float* y, int B, int C, int S, int H, int G,
                   cudaStream_t s) {
  if (B <= 0 || C <= 0) return;
  ssd_fwd_kernel<<<dim3(S / kT, C, B * H), kThreads, 0, s>>>(cb, cum, x, y, C, S, H, G);
}

void ssd_intra_bwd(const float* cb, const float* cum, const float* x, const float* dy, float* dx, float* dcb,
                   float* dcum, int B, int C, int S, int H, int G, cudaStream_t s) {
  if (B <= 0 || C <= 0) return;
  ssd_bwd_dx_kernel<<<dim3(S / kT, C, B * H), kThreads, 0, s>>>(cb, cum, dy, dx, C, S, H, G);
  const int nb = S / kT;
  ssd_bwd_dm_kernel<<<dim3(nb * (nb + 1) / 2, C, B * G * kHeadSplits), kThreads, 0, s>>>(cb, cum, x, dy, dcb, dcum,
                                                                                         C, S, H, G);
}

}  // namespace bw
