// Per-sample gradients of LayerNorm / RMSNorm affine parameters in one pass:
//
//     dgamma[b] = sum_t  x_hat[b,t] * g[b,t],      dbeta[b] = sum_t g[b,t]
//
// with x_hat recomputed from the raw layer input inside the kernel (row mean / rstd in
// fp32), so neither x_hat nor the (x_hat, 1) factor block ever lands in HBM.  A CTA owns
// a run of tokens of one sample: each warp normalises one token row at a time (16-byte
// loads, warp-shuffle statistics) and adds its products into the CTA's fp32 accumulators
// in shared memory; the CTA then adds those into the sample's output row.
#include <cuda_bf16.h>

#include "norm_grad.cuh"

namespace bw {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <bool kLayerNorm>
__global__ void __launch_bounds__(kWarps * 32)
    norm_psg_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ g, float* __restrict__ dw,
                    float* __restrict__ db, int T, int d, float eps, int tokens_per_cta) {
  extern __shared__ float acc[];  // [d] dgamma, then [d] dbeta
  const int b = blockIdx.y;
  const int t0 = blockIdx.x * tokens_per_cta;
  const int t1 = min(T, t0 + tokens_per_cta);
  for (int i = threadIdx.x; i < 2 * d; i += blockDim.x) acc[i] = 0.f;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = d / 8;
  for (int t = t0 + warp; t < t1; t += kWarps) {
    const long long row = ((long long)b * T + t) * d;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row);
    const uint4* gr = reinterpret_cast<const uint4*>(g + row);
    float s = 0.f, ss = 0.f;
    for (int v = lane; v < nv; v += 32) {
      const uint4 q = xr[v];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        s += f.x + f.y;
        ss += f.x * f.x + f.y * f.y;
      }
    }
    s = warp_sum(s);
    ss = warp_sum(ss);
    const float mean = kLayerNorm ? s / d : 0.f;
    const float var = kLayerNorm ? fmaxf(ss / d - mean * mean, 0.f) : ss / d;
    const float rstd = rsqrtf(var + eps);
    for (int v = lane; v < nv; v += 32) {
      const uint4 qx = xr[v], qg = gr[v];
      const __nv_bfloat162* hx = reinterpret_cast<const __nv_bfloat162*>(&qx);
      const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&qg);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fx = __bfloat1622float2(hx[e]), fg = __bfloat1622float2(hg[e]);
        const int c = v * 8 + 2 * e;
        atomicAdd(&acc[c], (fx.x - mean) * rstd * fg.x);
        atomicAdd(&acc[c + 1], (fx.y - mean) * rstd * fg.y);
        if (db != nullptr) {
          atomicAdd(&acc[d + c], fg.x);
          atomicAdd(&acc[d + c + 1], fg.y);
        }
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    atomicAdd(dw + (long long)b * d + i, acc[i]);
    if (db != nullptr) atomicAdd(db + (long long)b * d + i, acc[d + i]);
  }
}

}  // namespace

void norm_per_sample_grad(const __nv_bfloat16* x, const __nv_bfloat16* g, float* dw, float* db, int B, int T, int d,
                          float eps, bool layer_norm, cudaStream_t s) {
  if (B <= 0 || T <= 0) return;
  // Enough CTAs to fill the GPU, each with several tokens per warp.
  int per = (int)(((long long)B * T + 148 * 2 - 1) / (148 * 2));
  per = per < kWarps ? kWarps : ((per + kWarps - 1) / kWarps) * kWarps;
  dim3 grid((T + per - 1) / per, B);
  const size_t smem = (size_t)2 * d * sizeof(float);
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured >> dev & 1ull)) {
    cudaFuncSetAttribute(norm_psg_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 16384 * 4);
    cudaFuncSetAttribute(norm_psg_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 16384 * 4);
    configured |= 1ull << dev;
  }
  if (layer_norm)
    norm_psg_kernel<true><<<grid, kWarps * 32, smem, s>>>(x, g, dw, db, T, d, eps, per);
  else
    norm_psg_kernel<false><<<grid, kWarps * 32, smem, s>>>(x, g, dw, db, T, d, eps, per);
}

}  // namespace bw
