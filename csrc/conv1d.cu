// Causal depthwise convolution (4 taps) followed by SiLU, the Mamba2 mixer's conv1d + act:
//
//     out[t, c] = silu(bias[c] + sum_{k<4} w[c, k] x[t - 3 + k, c])
//
// The library call runs cuDNN's generic depthwise kernel on the transposed (channels x tokens)
// view, a separate SiLU, and the transposes around them.  Here each thread owns two adjacent
// channels (one 4-byte bf16 pair, so a warp reads 128 contiguous bytes of a token row) over a
// run of 16 tokens and slides a 4-token window along it: every input is read once, straight
// from the token-major projection it is a slice of.  The backward recomputes the
// pre-activation, keeps the last four pre-activation gradients in registers to form dx, and
// sums the tap and bias gradients per run into partial rows that a second launch adds up.
#include <cuda_bf16.h>

#include "conv1d.cuh"

namespace bw {
namespace {

constexpr int kRun = 16;       // tokens per thread (short runs: more threads, more loads in flight)
constexpr int kCThreads = 128;  // channel pairs per CTA
constexpr int K = kConvTaps;

__device__ __forceinline__ float sigm(float v) { return 1.f / (1.f + __expf(-v)); }

__device__ __forceinline__ float2 load2(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}

__global__ void __launch_bounds__(kCThreads)
    conv_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, long long sbx,
                    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                    __nv_bfloat16* __restrict__ out, int L, int C) {
  const int c = 2 * (blockIdx.x * kCThreads + threadIdx.x);
  if (c >= C) return;
  const int b = blockIdx.z, t0 = blockIdx.y * kRun, t1 = min(L, t0 + kRun);
  float w0[K], w1[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    w0[k] = __bfloat162float(w[c * K + k]);
    w1[k] = __bfloat162float(w[(c + 1) * K + k]);
  }
  const float b0 = bias != nullptr ? __bfloat162float(bias[c]) : 0.f;
  const float b1 = bias != nullptr ? __bfloat162float(bias[c + 1]) : 0.f;
  const __nv_bfloat16* xb = x + b * sbx + c;
  float win0[K], win1[K];  // x[t - 3 .. t] of the two channels, newest last
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 - (K - 1) + k;
    const float2 v = t >= 0 ? load2(xb + (long long)t * ldx) : make_float2(0.f, 0.f);
    win0[k] = v.x;
    win1[k] = v.y;
  }
  __nv_bfloat16* ob = out + ((long long)b * L) * C + c;
#pragma unroll 4
  for (int t = t0; t < t1; ++t) {
    const float2 v = load2(xb + (long long)t * ldx);
    win0[K - 1] = v.x;
    win1[K - 1] = v.y;
    float p0 = b0, p1 = b1;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      p0 = fmaf(w0[k], win0[k], p0);
      p1 = fmaf(w1[k], win1[k], p1);
    }
    *reinterpret_cast<__nv_bfloat162*>(ob + (long long)t * C) = __floats2bfloat162_rn(p0 * sigm(p0), p1 * sigm(p1));
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
      win0[k] = win0[k + 1];
      win1[k] = win1[k + 1];
    }
  }
}

__global__ void __launch_bounds__(kCThreads)
    conv_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ x, long long ldx,
                    long long sbx, const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ bias,
                    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, float* __restrict__ db_part, int L,
                    int C) {
  const int c = 2 * (blockIdx.x * kCThreads + threadIdx.x);
  if (c >= C) return;
  const int b = blockIdx.z, t0 = blockIdx.y * kRun, t1 = min(L, t0 + kRun);
  float w0[K], w1[K];
#pragma unroll
  for (int k = 0; k < K; ++k) {
    w0[k] = __bfloat162float(w[c * K + k]);
    w1[k] = __bfloat162float(w[(c + 1) * K + k]);
  }
  const float b0 = bias != nullptr ? __bfloat162float(bias[c]) : 0.f;
  const float b1 = bias != nullptr ? __bfloat162float(bias[c + 1]) : 0.f;
  const __nv_bfloat16* xb = x + b * sbx + c;
  const __nv_bfloat16* gb = dout + ((long long)b * L) * C + c;
  __nv_bfloat16* dxb = dx + ((long long)b * L) * C + c;
  float win0[K], win1[K];  // x[t - 3 .. t]
  float dp0[K], dp1[K];    // pre-activation gradients of t - 3 .. t
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 - (K - 1) + k;
    const float2 v = t >= 0 ? load2(xb + (long long)t * ldx) : make_float2(0.f, 0.f);
    win0[k] = v.x;
    win1[k] = v.y;
    dp0[k] = dp1[k] = 0.f;
  }
  float gw0[K], gw1[K], gb0 = 0.f, gb1 = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) gw0[k] = gw1[k] = 0.f;
  // t runs K - 1 tokens past the run: dx[t'] needs the pre-activation gradients of t' .. t' + 3
#pragma unroll 4
  for (int t = t0; t < t1 + K - 1; ++t) {
    float d0 = 0.f, d1 = 0.f;
    if (t < L) {
      const float2 v = load2(xb + (long long)t * ldx);
      win0[K - 1] = v.x;
      win1[K - 1] = v.y;
      float p0 = b0, p1 = b1;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        p0 = fmaf(w0[k], win0[k], p0);
        p1 = fmaf(w1[k], win1[k], p1);
      }
      const float2 g = load2(gb + (long long)t * C);
      const float s0 = sigm(p0), s1 = sigm(p1);
      d0 = g.x * s0 * (1.f + p0 * (1.f - s0));
      d1 = g.y * s1 * (1.f + p1 * (1.f - s1));
      if (t < t1) {  // this run's tokens: tap and bias gradients
#pragma unroll
        for (int k = 0; k < K; ++k) {
          gw0[k] = fmaf(d0, win0[k], gw0[k]);
          gw1[k] = fmaf(d1, win1[k], gw1[k]);
        }
        gb0 += d0;
        gb1 += d1;
      }
    } else {
      win0[K - 1] = win1[K - 1] = 0.f;
    }
    dp0[K - 1] = d0;
    dp1[K - 1] = d1;
    const int tp = t - (K - 1);  // dx[tp] = sum_j w[3 - j] dpre[tp + j]
    if (tp >= t0) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) {
        a0 = fmaf(w0[K - 1 - j], dp0[j], a0);
        a1 = fmaf(w1[K - 1 - j], dp1[j], a1);
      }
      *reinterpret_cast<__nv_bfloat162*>(dxb + (long long)tp * C) = __floats2bfloat162_rn(a0, a1);
    }
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
      win0[k] = win0[k + 1];
      win1[k] = win1[k + 1];
      dp0[k] = dp0[k + 1];
      dp1[k] = dp1[k + 1];
    }
  }
  const long long part = (long long)b * gridDim.y + blockIdx.y;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    dw_part[(part * C + c) * K + k] = gw0[k];
    dw_part[(part * C + c + 1) * K + k] = gw1[k];
  }
  db_part[part * C + c] = gb0;
  db_part[part * C + c + 1] = gb1;
}

// out[i] = sum over the parts of part[p * n + i] (consecutive threads, consecutive i).
__global__ void __launch_bounds__(256) parts_sum_kernel(const float* __restrict__ part, float* __restrict__ out,
                                                        int parts, long long n) {
  const long long i = (long long)blockIdx.x * 256 + threadIdx.x;
  if (i >= n) return;
  float t = 0.f;
  for (int p = 0; p < parts; ++p) t += part[(long long)p * n + i];
  out[i] = t;
}

}  // namespace

void causal_conv_silu_fwd(const __nv_bfloat16* x, long long ldx, long long sbx, const __nv_bfloat16* w,
                          const __nv_bfloat16* bias, __nv_bfloat16* out, int B, int L, int C, cudaStream_t s) {
  if (B <= 0 || L <= 0) return;
  const dim3 grid((C / 2 + kCThreads - 1) / kCThreads, (L + kRun - 1) / kRun, B);
  conv_fwd_kernel<<<grid, kCThreads, 0, s>>>(x, ldx, sbx, w, bias, out, L, C);
}

int causal_conv_bwd_parts(int B, int L) { return B * ((L + kRun - 1) / kRun); }

void causal_conv_silu_bwd(const __nv_bfloat16* dout, const __nv_bfloat16* x, long long ldx, long long sbx,
                          const __nv_bfloat16* w, const __nv_bfloat16* bias, __nv_bfloat16* dx, float* dw_part,
                          float* db_part, float* dw, float* db, int B, int L, int C, cudaStream_t s) {
  if (B <= 0 || L <= 0) return;
  const dim3 grid((C / 2 + kCThreads - 1) / kCThreads, (L + kRun - 1) / kRun, B);
  conv_bwd_kernel<<<grid, kCThreads, 0, s>>>(dout, x, ldx, sbx, w, bias, dx, dw_part, db_part, L, C);
  const int parts = causal_conv_bwd_parts(B, L);
  const long long nw = (long long)C * K;
  parts_sum_kernel<<<(unsigned)((nw + 255) / 256), 256, 0, s>>>(dw_part, dw, parts, nw);
  parts_sum_kernel<<<(unsigned)((C + 255) / 256), 256, 0, s>>>(db_part, db, parts, C);
}

}  // namespace bw
