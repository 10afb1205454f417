// Gated RMSNorm of the Mamba2 mixer, forward and backward in one pass each:
//
//     h = y * silu(g),   r = 1 / sqrt(mean(h^2) + eps),   out = w * h * r
//
// The unfused module runs about eight elementwise passes forward and fifteen backward over
// fp32 (tokens x 5,120) tensors per layer; here the forward reads y and g once and writes
// the bf16 output (the cast the mixer applies before its out_proj is folded in), and the
// backward reads dout, y and g (a second time from L1 / L2) and writes dy and dg.  One CTA per
// row in the forward; the backward gives each CTA a run of rows so the weight gradient is
// summed per CTA in shared memory, written as one partial row per CTA and summed over the
// CTAs by a second launch (no atomics on the D-wide result).
#include <cuda_bf16.h>

#include "gated_norm.cuh"

namespace bw {
namespace {

constexpr int kThreads = 256;
constexpr int kRowsPerCta = 2;  // 1,024 CTAs for 2,048 rows: enough loads in flight

__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // scratch reuse across calls
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) t += scratch[i];
  return t;
}

__device__ __forceinline__ float sigmoid(float x) { return 1.f / (1.f + __expf(-x)); }

__global__ void __launch_bounds__(kThreads)
    gated_rms_fwd_kernel(const float* __restrict__ y, const __nv_bfloat16* __restrict__ g, long long ldg,
                         const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                         float* __restrict__ rstd, int cols, float eps) {
  __shared__ float scratch[kThreads / 32];
  const long long row = blockIdx.x;
  const float* yr = y + row * cols;
  const __nv_bfloat16* gr = g + row * ldg;
  float ss = 0.f;
#pragma unroll 4
  for (int c = threadIdx.x; c < cols; c += kThreads) {
    const float gv = __bfloat162float(gr[c]);
    const float h = yr[c] * gv * sigmoid(gv);
    ss += h * h;
  }
  const float r = rsqrtf(block_sum(ss, scratch) / cols + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  __nv_bfloat16* o = out + row * cols;
#pragma unroll 4
  for (int c = threadIdx.x; c < cols; c += kThreads) {  // the row again, now from L1 / L2
    const float gv = __bfloat162float(gr[c]);
    o[c] = __float2bfloat16(__bfloat162float(w[c]) * yr[c] * gv * sigmoid(gv) * r);
  }
}

// Each row is read twice (the second time from L1 / L2) instead of being held in registers,
// and the weight-gradient sums of the CTA's rows live in shared memory (each thread owns its
// columns there, so no two threads touch one entry): few registers, many warps per SM, which
// is what this latency-bound pass needs.  The row loops are unrolled so several columns'
// loads are in flight at once.
__global__ void __launch_bounds__(kThreads)
    gated_rms_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const float* __restrict__ y,
                         const __nv_bfloat16* __restrict__ g, long long ldg, const __nv_bfloat16* __restrict__ w,
                         const float* __restrict__ rstd, float* __restrict__ dy, __nv_bfloat16* __restrict__ dg,
                         float* __restrict__ dw_part, int rows, int cols) {
  __shared__ float scratch[kThreads / 32];
  extern __shared__ float dw_acc[];  // [cols]
  for (int c = threadIdx.x; c < cols; c += kThreads) dw_acc[c] = 0.f;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int r1 = min(rows, r0 + kRowsPerCta);
  const float inv_cols = 1.f / cols;
  for (int row = r0; row < r1; ++row) {
    const float* yr = y + (long long)row * cols;
    const __nv_bfloat16* gr = g + (long long)row * ldg;
    const __nv_bfloat16* dr = dout + (long long)row * cols;
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll 4
    for (int c = threadIdx.x; c < cols; c += kThreads) {
      const float gv = __bfloat162float(gr[c]);
      const float d = __bfloat162float(dr[c]);
      const float n = yr[c] * gv * sigmoid(gv) * r;
      dw_acc[c] += d * n;
      dot += d * __bfloat162float(w[c]) * n;
    }
    const float mean = block_sum(dot, scratch) * inv_cols;
#pragma unroll 4
    for (int c = threadIdx.x; c < cols; c += kThreads) {
      const float gv = __bfloat162float(gr[c]);
      const float yv = yr[c];
      const float s = sigmoid(gv);
      const float n = yv * gv * s * r;
      const float dh = r * (__bfloat162float(dr[c]) * __bfloat162float(w[c]) - n * mean);
      dy[(long long)row * cols + c] = dh * gv * s;
      dg[(long long)row * cols + c] = __float2bfloat16(dh * yv * s * (1.f + gv * (1.f - s)));
    }
  }
  float* part = dw_part + (long long)blockIdx.x * cols;  // this CTA's row of partial sums
  for (int c = threadIdx.x; c < cols; c += kThreads) part[c] = dw_acc[c];
}

// dw[c] = sum over the CTAs' partial rows (column sums; consecutive threads, consecutive columns).
__global__ void __launch_bounds__(kThreads) column_sum_kernel(const float* __restrict__ part, float* __restrict__ dw,
                                                              int parts, int cols) {
  const int c = blockIdx.x * kThreads + threadIdx.x;
  if (c >= cols) return;
  float t = 0.f;
  for (int r = 0; r < parts; ++r) t += part[(long long)r * cols + c];
  dw[c] = t;
}

}  // namespace

void gated_rms_fwd(const float* y, const __nv_bfloat16* g, long long ldg, const __nv_bfloat16* w,
                   __nv_bfloat16* out, float* rstd, int rows, int cols, float eps, cudaStream_t s) {
  if (rows <= 0) return;
  gated_rms_fwd_kernel<<<rows, kThreads, 0, s>>>(y, g, ldg, w, out, rstd, cols, eps);
}

int gated_rms_bwd_parts(int rows) { return (rows + kRowsPerCta - 1) / kRowsPerCta; }

void gated_rms_bwd(const __nv_bfloat16* dout, const float* y, const __nv_bfloat16* g, long long ldg,
                   const __nv_bfloat16* w, const float* rstd, float* dy, __nv_bfloat16* dg, float* dw_part, float* dw,
                   int rows, int cols, cudaStream_t s) {
  if (rows <= 0) return;
  const int grid = gated_rms_bwd_parts(rows);
  gated_rms_bwd_kernel<<<grid, kThreads, (size_t)cols * sizeof(float), s>>>(dout, y, g, ldg, w, rstd, dy, dg, dw_part,
                                                                            rows, cols);
  column_sum_kernel<<<(cols + kThreads - 1) / kThreads, kThreads, 0, s>>>(dw_part, dw, grid, cols);
}

}  // namespace bw
