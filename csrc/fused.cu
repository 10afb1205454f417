// Fused memory-bound kernels of the model path: RMSNorm forward/backward, SwiGLU
// forward/backward, and the cross-entropy over bf16 logits (per-row log-sum-exp +
// loss; backward rewrites the logits buffer into dlogits in place).  Every kernel
// reads and writes each element once with 16-byte vector accesses and reduces in
// fp32.  Transcendentals are CUDA's own __expf / __logf (approximate, fp32).
#include "fused.cuh"

#include <cuda_bf16.h>

namespace bw {
namespace {

constexpr int kVec = 8;  // bf16 per 16-byte access

struct __align__(16) Bf8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack(const Bf8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __bfloat1622float2(v.h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ Bf8 pack(const float (&f)[8]) {
  Bf8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < kThreads / 32) t = red[threadIdx.x];
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// ---------------------------------------------------------------- RMSNorm
// One CTA per row; cols must be a multiple of 8 (checked by the host).
template <int kThreads>
__global__ void __launch_bounds__(kThreads) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ y,
                                                               float* __restrict__ rstd, int cols, float eps) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const Bf8* xr = reinterpret_cast<const Bf8*>(x + row * cols);
  const Bf8* wr = reinterpret_cast<const Bf8*>(w);
  Bf8* yr = reinterpret_cast<Bf8*>(y + row * cols);
  const int nv = cols / kVec;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float f[8];
    unpack(xr[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
  ss = block_sum<kThreads>(ss, red);
  const float r = rsqrtf(ss / cols + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float f[8], g[8];
    unpack(xr[i], f);
    unpack(wr[i], g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
    yr[i] = pack(f);
  }
}

// dx = r * (dy*w - xhat * mean(dy*w*xhat)),  xhat = x * r
template <int kThreads>
__global__ void __launch_bounds__(kThreads) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                               const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               const float* __restrict__ rstd,
                                                               __nv_bfloat16* __restrict__ dx, int cols) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const Bf8* dyr = reinterpret_cast<const Bf8*>(dy + row * cols);
  const Bf8* xr = reinterpret_cast<const Bf8*>(x + row * cols);
  const Bf8* wr = reinterpret_cast<const Bf8*>(w);
  Bf8* dxr = reinterpret_cast<Bf8*>(dx + row * cols);
  const int nv = cols / kVec;
  const float r = rstd[row];
  float dot = 0.f;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float a[8], b[8], c[8];
    unpack(dyr[i], a);
    unpack(xr[i], b);
    unpack(wr[i], c);
#pragma unroll
    for (int j = 0; j < 8; ++j) dot += a[j] * c[j] * b[j] * r;
  }
  const float mean = block_sum<kThreads>(dot, red) / cols;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float a[8], b[8], c[8], o[8];
    unpack(dyr[i], a);
    unpack(xr[i], b);
    unpack(wr[i], c);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = r * (a[j] * c[j] - b[j] * r * mean);
    dxr[i] = pack(o);
  }
}

// ---------------------------------------------------------------- SwiGLU
__device__ __forceinline__ float sigmoidf_(float v) { return 1.f / (1.f + __expf(-v)); }

__global__ void swiglu_fwd_kernel(const Bf8* __restrict__ g, const Bf8* __restrict__ u, Bf8* __restrict__ h,
                                  long long nv) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv;
       i += (long long)gridDim.x * blockDim.x) {
    float a[8], b[8];
    unpack(g[i], a);
    unpack(u[i], b);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = a[j] * sigmoidf_(a[j]) * b[j];
    h[i] = pack(a);
  }
}

__global__ void swiglu_bwd_kernel(const Bf8* __restrict__ dh, const Bf8* __restrict__ g,
                                  const Bf8* __restrict__ u, Bf8* __restrict__ dg, Bf8* __restrict__ du,
                                  long long nv) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv;
       i += (long long)gridDim.x * blockDim.x) {
    float d[8], a[8], b[8], og[8], ou[8];
    unpack(dh[i], d);
    unpack(g[i], a);
    unpack(u[i], b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float s = sigmoidf_(a[j]);
      const float silu = a[j] * s;
      ou[j] = d[j] * silu;
      og[j] = d[j] * b[j] * (s + silu * (1.f - s));
    }
    dg[i] = pack(og);
    du[i] = pack(ou);
  }
}

// ---------------------------------------------------------------- cross-entropy
// Row-wise online log-sum-exp over bf16 logits (cols % 8 == 0, 16-byte aligned rows).
template <int kThreads>
__global__ void __launch_bounds__(kThreads) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                          const int64_t* __restrict__ target,
                                                          float* __restrict__ loss, float* __restrict__ lse,
                                                          int cols, long long ld) {
  __shared__ float red_m[32], red_s[32];
  const long long row = blockIdx.x;
  const Bf8* lr = reinterpret_cast<const Bf8*>(logits + row * ld);
  const int nv = cols / kVec;
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nv; i += kThreads) {
    float f[8];
    unpack(lr[i], f);
    float mx = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mx = fmaxf(mx, f[j]);
    const float nm = fmaxf(m, mx);
    float acc = s * __expf(m - nm);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += __expf(f[j] - nm);
    m = nm;
    s = acc;
  }
  // combine (m, s) pairs: warp then block
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    red_m[warp] = m;
    red_s[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY, S = 0.f;
    for (int k = 0; k < kThreads / 32; ++k) {
      const float nm = fmaxf(M, red_m[k]);
      S = (M == -INFINITY ? 0.f : S * __expf(M - nm)) +
          (red_m[k] == -INFINITY ? 0.f : red_s[k] * __expf(red_m[k] - nm));
      M = nm;
    }
    const float l = M + __logf(S);
    lse[row] = l;
    const long long t = target[row];
    loss[row] = (t < 0 || t >= cols) ? 0.f : l - __bfloat162float(logits[row * ld + t]);
  }
}

// logits[row] <- (softmax(row) - onehot(target)) * gscale ; rows with target -100 -> 0
__global__ void ce_bwd_kernel(__nv_bfloat16* __restrict__ logits, const float* __restrict__ lse,
                              const int64_t* __restrict__ target, const float* __restrict__ gscale, int cols,
                              long long ld) {
  const long long row = blockIdx.x;
  Bf8* lr = reinterpret_cast<Bf8*>(logits + row * ld);
  const long long t = target[row];
  const bool ignore = t < 0 || t >= cols;
  const float l = lse[row];
  const float gs = *gscale;
  const int nv = cols / kVec;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float f[8];
    unpack(lr[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const long long c = (long long)i * kVec + j;
      const float p = __expf(f[j] - l) - (c == t ? 1.f : 0.f);
      f[j] = ignore ? 0.f : p * gs;
    }
    lr[i] = pack(f);
  }
}

}  // namespace

void rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, float* rstd, int rows,
                 int cols, float eps, cudaStream_t s) {
  if (rows > 0) rmsnorm_fwd_kernel<256><<<rows, 256, 0, s>>>(x, w, y, rstd, cols, eps);
}

void rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w, const float* rstd,
                 __nv_bfloat16* dx, int rows, int cols, cudaStream_t s) {
  if (rows > 0) rmsnorm_bwd_kernel<256><<<rows, 256, 0, s>>>(dy, x, w, rstd, dx, cols);
}

static int grid_for(long long nv) {
  const long long b = (nv + 255) / 256;
  return (int)(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

void swiglu_fwd(const __nv_bfloat16* g, const __nv_bfloat16* u, __nv_bfloat16* h, long long n, cudaStream_t s) {
  const long long nv = n / kVec;
  if (nv > 0)
    swiglu_fwd_kernel<<<grid_for(nv), 256, 0, s>>>(reinterpret_cast<const Bf8*>(g),
                                                   reinterpret_cast<const Bf8*>(u), reinterpret_cast<Bf8*>(h),
                                                   nv);
}

void swiglu_bwd(const __nv_bfloat16* dh, const __nv_bfloat16* g, const __nv_bfloat16* u, __nv_bfloat16* dg,
                __nv_bfloat16* du, long long n, cudaStream_t s) {
  const long long nv = n / kVec;
  if (nv > 0)
    swiglu_bwd_kernel<<<grid_for(nv), 256, 0, s>>>(
        reinterpret_cast<const Bf8*>(dh), reinterpret_cast<const Bf8*>(g), reinterpret_cast<const Bf8*>(u),
        reinterpret_cast<Bf8*>(dg), reinterpret_cast<Bf8*>(du), nv);
}

void ce_fwd(const __nv_bfloat16* logits, const int64_t* target, float* loss, float* lse, int rows, int cols,
            long long ld, cudaStream_t s) {
  if (rows > 0) ce_fwd_kernel<512><<<rows, 512, 0, s>>>(logits, target, loss, lse, cols, ld);
}

void ce_bwd_inplace(__nv_bfloat16* logits, const float* lse, const int64_t* target, const float* gscale,
                    int rows, int cols, long long ld, cudaStream_t s) {
  if (rows > 0) ce_bwd_kernel<<<rows, 512, 0, s>>>(logits, lse, target, gscale, cols, ld);
}

}  // namespace bw
