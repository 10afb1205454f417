#include <algorithm>
// Row-parallel fused kernels of the decoder path, one warp per row with the row held in
// registers (one HBM read and one write per element):
//   * RMSNorm forward with an optional fused residual add  (h = x + delta; y = rms(h) * w),
//   * RMSNorm backward with an optional fused residual-gradient add
//     (dh = rms_bwd(dy) + dres -- the gradient both residual inputs receive),
//   * rotary position embedding of q and k in one launch (forward rotates by +theta,
//     backward by -theta; any (b, t, h) strides, head dim contiguous),
//   * the per-sample Adam direction  m_hat / (sqrt(v_hat) + eps)  of a gradient block
//     against the optimizer's moments (LESS preconditioning).
// Arithmetic is fp32; bf16 only at loads and stores.
#include <cuda_bf16.h>

#include "rows.cuh"

namespace bw {
namespace {

struct __align__(16) Bf8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const Bf8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 p = __bfloat1622float2(v.h[i]);
    f[2 * i] = p.x;
    f[2 * i + 1] = p.y;
  }
}

__device__ __forceinline__ Bf8 pack8(const float (&f)[8]) {
  Bf8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kWarps = 4;  // rows per CTA

// ------------------------------------------------------------------ RMSNorm fwd
// Lane l owns 8-element vectors l, l+32, ..., l+32(kPer-1) of its row.
template <int kPer>
__global__ void __launch_bounds__(kWarps * 32) rms_fwd_kernel(
    const Bf8* __restrict__ x, const Bf8* __restrict__ delta, Bf8* __restrict__ h, const Bf8* __restrict__ w,
    Bf8* __restrict__ y, float* __restrict__ rstd, int rows, int nv, float inv_cols, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const long long base = row * nv;
  Bf8 keep[kPer];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      Bf8 xv = x[base + v];
      if (delta != nullptr) {
        float a[8], b[8];
        unpack8(xv, a);
        unpack8(delta[base + v], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += b[j];
        xv = pack8(a);  // the residual stream is bf16: normalise the rounded sum
        h[base + v] = xv;
      }
      keep[i] = xv;
      float f[8];
      unpack8(xv, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss * inv_cols + eps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      float f[8], g[8];
      unpack8(keep[i], f);
      unpack8(w[v], g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
      y[base + v] = pack8(f);
    }
  }
}

// ------------------------------------------------------------------ RMSNorm bwd
// dx = r * (dy*w - xhat * mean(dy*w*xhat)) + dres,  xhat = x * r.  dy and x stay packed in
// registers; dres is prefetched into L2 before the reduction and read after it, which keeps
// the register count low enough for 4 CTAs (16 warps) per SM.
template <int kPer>
__global__ void __launch_bounds__(kWarps * 32, kPer <= 8 ? 4 : 2) rms_bwd_kernel(
    const Bf8* __restrict__ dy, const Bf8* __restrict__ x, const Bf8* __restrict__ w,
    const float* __restrict__ rstd, const Bf8* __restrict__ dres, Bf8* __restrict__ dx, int rows, int nv,
    float inv_cols) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const long long base = row * nv;
  const float r = rstd[row];
  Bf8 kdy[kPer], kx[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      kdy[i] = dy[base + v];
      kx[i] = x[base + v];
      if (dres != nullptr) asm volatile("prefetch.global.L2 [%0];" ::"l"(dres + base + v));
    }
  }
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      float a[8], b[8], c[8];
      unpack8(kdy[i], a);
      unpack8(kx[i], b);
      unpack8(w[v], c);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += a[j] * c[j] * b[j];
    }
  }
  const float mean = warp_sum(dot) * r * inv_cols;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int v = lane + 32 * i;
    if (v < nv) {
      float a[8], b[8], c[8], o[8];
      unpack8(kdy[i], a);
      unpack8(kx[i], b);
      unpack8(w[v], c);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r * (a[j] * c[j] - b[j] * r * mean);
      if (dres != nullptr) {
        float d[8];
        unpack8(dres[base + v], d);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] += d[j];
      }
      dx[base + v] = pack8(o);
    }
  }
}

template <int kPer>
void rms_fwd_launch(const RowsNorm& a, cudaStream_t s) {
  const int nv = a.cols / 8;
  const int grid = (a.rows + kWarps - 1) / kWarps;
  rms_fwd_kernel<kPer><<<grid, kWarps * 32, 0, s>>>(
      reinterpret_cast<const Bf8*>(a.x), reinterpret_cast<const Bf8*>(a.delta), reinterpret_cast<Bf8*>(a.h),
      reinterpret_cast<const Bf8*>(a.w), reinterpret_cast<Bf8*>(a.y), a.rstd, a.rows, nv, 1.f / a.cols, a.eps);
}

template <int kPer>
void rms_bwd_launch(const RowsNormBwd& a, cudaStream_t s) {
  const int nv = a.cols / 8;
  const int grid = (a.rows + kWarps - 1) / kWarps;
  rms_bwd_kernel<kPer><<<grid, kWarps * 32, 0, s>>>(
      reinterpret_cast<const Bf8*>(a.dy), reinterpret_cast<const Bf8*>(a.x), reinterpret_cast<const Bf8*>(a.w),
      a.rstd, reinterpret_cast<const Bf8*>(a.dres), reinterpret_cast<Bf8*>(a.dx), a.rows, nv, 1.f / a.cols);
}

// ------------------------------------------------------------------ RoPE
// A CTA covers kTok consecutive tokens of one sequence; thread (head, chunk) rotates 8 pairs
// (x[c*8 .. c*8+8), x[half + c*8 ..)) of its head in each of those tokens.  Consecutive
// threads read consecutive 16-byte vectors (coalesced), and each thread issues all kTok
// tokens' loads before any arithmetic.
constexpr int kTok = 4;

__global__ void __launch_bounds__(1024) rope_kernel(RopeArgs a, float sign) {
  const int chunks = a.head_dim >> 4;
  const int half = a.head_dim >> 1;
  const int per_token = (a.hq + a.hk) * chunks;
  const int i = threadIdx.x;
  if (i >= per_token) return;
  int head = i / chunks;
  const int c = i - head * chunks;
  const bool is_q = head < a.hq;
  if (!is_q) head -= a.hq;
  const RopeTensor T = is_q ? a.q : a.k;
  const long long b = blockIdx.y;
  const int t0 = blockIdx.x * kTok;
  const __nv_bfloat16* src = T.in + b * T.in_sb + (long long)head * T.in_sh + c * 8;
  __nv_bfloat16* dst = T.out + b * T.out_sb + (long long)head * T.out_sh + c * 8;
  Bf8 v1[kTok], v2[kTok];
#pragma unroll
  for (int u = 0; u < kTok; ++u) {
    if (t0 + u < a.seq) {
      const __nv_bfloat16* p = src + (long long)(t0 + u) * T.in_st;
      v1[u] = *reinterpret_cast<const Bf8*>(p);
      v2[u] = *reinterpret_cast<const Bf8*>(p + half);
    }
  }
#pragma unroll
  for (int u = 0; u < kTok; ++u) {
    const int t = t0 + u;
    if (t >= a.seq) break;
    const float4* ct = reinterpret_cast<const float4*>(a.cos + (long long)t * half + c * 8);
    const float4* st = reinterpret_cast<const float4*>(a.sin + (long long)t * half + c * 8);
    const float4 c0 = ct[0], c1 = ct[1], s0 = st[0], s1 = st[1];
    const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float x1[8], x2[8], y1[8], y2[8];
    unpack8(v1[u], x1);
    unpack8(v2[u], x2);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sj = sign * sn[j];
      y1[j] = x1[j] * cs[j] - x2[j] * sj;
      y2[j] = x2[j] * cs[j] + x1[j] * sj;
    }
    __nv_bfloat16* q = dst + (long long)t * T.out_st;
    *reinterpret_cast<Bf8*>(q) = pack8(y1);
    *reinterpret_cast<Bf8*>(q + half) = pack8(y2);
  }
}

// ------------------------------------------------------------------ Adam direction
// out[b, i] = (m / bc1) / (sqrt(v / bc2) + eps),  m = b1 m0 + (1-b1) g,  v = b2 v0 + (1-b2) g^2
__global__ void adam_dir_kernel(const float4* __restrict__ g, const float4* __restrict__ m0,
                                const float4* __restrict__ v0, float4* __restrict__ out, long long rows,
                                long long p4, float b1, float b2, float inv_bc1, float inv_sqrt_bc2, float eps) {
  const long long total = rows * p4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long c = i % p4;
    const float4 gv = g[i], mv = m0[c], vv = v0[c];
    const float ga[4] = {gv.x, gv.y, gv.z, gv.w};
    const float ma[4] = {mv.x, mv.y, mv.z, mv.w};
    const float va[4] = {vv.x, vv.y, vv.z, vv.w};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float m = b1 * ma[j] + (1.f - b1) * ga[j];
      const float v = b2 * va[j] + (1.f - b2) * ga[j] * ga[j];
      o[j] = (m * inv_bc1) / (sqrtf(v) * inv_sqrt_bc2 + eps);
    }
    out[i] = make_float4(o[0], o[1], o[2], o[3]);
  }
}

// ------------------------------------------------------------------ SwiGLU on [gate | up] rows
// h (rows, 2I) holds the gate half then the up half of each row; out (rows, I) = silu(gate) * up.
// `rows` is read from device memory (the count of valid rows is known only on the device).
__global__ void swiglu_split_fwd_kernel(const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ out,
                                        const int* __restrict__ rows, int inter) {
  const long long n = (long long)(*rows) * (inter / 8);
  const int iv = inter / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / iv, c = i % iv;
    float g[8], u[8];
    unpack8(reinterpret_cast<const Bf8*>(h + r * 2 * inter)[c], g);
    unpack8(reinterpret_cast<const Bf8*>(h + r * 2 * inter + inter)[c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
    reinterpret_cast<Bf8*>(out + r * inter)[c] = pack8(g);
  }
}

// dh[:, :I] = da * u * s * (1 + g (1 - s)),  dh[:, I:] = da * g * s,  s = sigmoid(g)
__global__ void swiglu_split_bwd_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ h,
                                        __nv_bfloat16* __restrict__ dh, const int* __restrict__ rows, int inter) {
  const long long n = (long long)(*rows) * (inter / 8);
  const int iv = inter / 8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / iv, c = i % iv;
    float d[8], g[8], u[8], og[8], ou[8];
    unpack8(reinterpret_cast<const Bf8*>(da + r * inter)[c], d);
    unpack8(reinterpret_cast<const Bf8*>(h + r * 2 * inter)[c], g);
    unpack8(reinterpret_cast<const Bf8*>(h + r * 2 * inter + inter)[c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-g[j]));
      og[j] = d[j] * u[j] * sg * (1.f + g[j] * (1.f - sg));
      ou[j] = d[j] * g[j] * sg;
    }
    reinterpret_cast<Bf8*>(dh + r * 2 * inter)[c] = pack8(og);
    reinterpret_cast<Bf8*>(dh + r * 2 * inter + inter)[c] = pack8(ou);
  }
}

int grid_cap(long long work, int threads) {
  const long long b = (work + threads - 1) / threads;
  return (int)(b < 1 ? 1 : (b < 148 * 16 ? b : 148 * 16));
}

}  // namespace

bool rows_norm_supported(int cols) { return cols % 8 == 0 && cols <= 32 * 8 * 16; }

void rows_norm_fwd(const RowsNorm& a, cudaStream_t s) {
  if (a.rows <= 0) return;
  const int per = (a.cols / 8 + 31) / 32;
  if (per <= 1) rms_fwd_launch<1>(a, s);
  else if (per <= 2) rms_fwd_launch<2>(a, s);
  else if (per <= 4) rms_fwd_launch<4>(a, s);
  else if (per <= 8) rms_fwd_launch<8>(a, s);
  else rms_fwd_launch<16>(a, s);
}

void rows_norm_bwd(const RowsNormBwd& a, cudaStream_t s) {
  if (a.rows <= 0) return;
  const int per = (a.cols / 8 + 31) / 32;
  if (per <= 1) rms_bwd_launch<1>(a, s);
  else if (per <= 2) rms_bwd_launch<2>(a, s);
  else if (per <= 4) rms_bwd_launch<4>(a, s);
  else if (per <= 8) rms_bwd_launch<8>(a, s);
  else rms_bwd_launch<16>(a, s);
}

void rope(const RopeArgs& a, bool inverse, cudaStream_t s) {
  const int per_token = (a.hq + a.hk) * (a.head_dim / 16);
  if ((long long)a.batch * a.seq * per_token <= 0) return;
  const int threads = ((per_token + 31) / 32) * 32;
  rope_kernel<<<dim3((a.seq + kTok - 1) / kTok, a.batch), threads, 0, s>>>(a, inverse ? -1.f : 1.f);
}

bool rope_supported(int head_dim, int heads) { return head_dim % 16 == 0 && heads * (head_dim / 16) <= 1024; }

void swiglu_split(const __nv_bfloat16* h, __nv_bfloat16* out, const int* rows, int max_rows, int inter,
                  cudaStream_t s) {
  if (max_rows <= 0) return;
  swiglu_split_fwd_kernel<<<grid_cap((long long)max_rows * inter / 8, 256), 256, 0, s>>>(h, out, rows, inter);
}

void swiglu_split_bwd(const __nv_bfloat16* da, const __nv_bfloat16* h, __nv_bfloat16* dh, const int* rows,
                      int max_rows, int inter, cudaStream_t s) {
  if (max_rows <= 0) return;
  swiglu_split_bwd_kernel<<<grid_cap((long long)max_rows * inter / 8, 256), 256, 0, s>>>(da, h, dh, rows, inter);
}

void adam_direction(const float* g, const float* m0, const float* v0, float* out, long long rows, long long p,
                    float b1, float b2, float inv_bc1, float inv_sqrt_bc2, float eps, cudaStream_t s) {
  const long long p4 = p / 4;
  if (rows <= 0 || p4 <= 0) return;
  adam_dir_kernel<<<grid_cap(rows * p4, 256), 256, 0, s>>>(
      reinterpret_cast<const float4*>(g), reinterpret_cast<const float4*>(m0), reinterpret_cast<const float4*>(v0),
      reinterpret_cast<float4*>(out), rows, p4, b1, b2, inv_bc1, inv_sqrt_bc2, eps);
}

namespace {

// 64 x 64 tiles through shared memory: each thread moves two 16-byte vectors in (row-major
// reads of the source) and two out (row-major writes of the destination); the 8-element
// transpose happens on the shared tile (row pitch 65 elements, conflict-light).
__global__ void __launch_bounds__(256) transpose_bf16_kernel(const __nv_bfloat16* __restrict__ src, long long lds,
                                                             __nv_bfloat16* __restrict__ dst, long long ldd, int R,
                                                             int C) {
  __shared__ __nv_bfloat16 tile[64][66];
  const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
  const long long zs = (long long)blockIdx.z * R * lds, zd = (long long)blockIdx.z * C * ldd;
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int v = threadIdx.x + q * 256;  // 512 vectors: 64 rows x 8
    const int r = v >> 3, c = (v & 7) * 8;
    const int gr = r0 + r, gc = c0 + c;
    __nv_bfloat16 e[8];
    if (gr < R && gc + 8 <= C) {
      *reinterpret_cast<uint4*>(e) = *reinterpret_cast<const uint4*>(src + zs + (long long)gr * lds + gc);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = (gr < R && gc + k < C) ? src[zs + (long long)gr * lds + gc + k] : __nv_bfloat16();
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[c + k][r] = e[k];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int v = threadIdx.x + q * 256;
    const int r = v >> 3, c = (v & 7) * 8;  // r: destination row (source column), c: source row
    const int gr = c0 + r, gc = r0 + c;
    if (gr >= C) continue;
    __nv_bfloat16 e[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = tile[r][c + k];
    if (gc + 8 <= R) {
      *reinterpret_cast<uint4*>(dst + zd + (long long)gr * ldd + gc) = *reinterpret_cast<const uint4*>(e);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (gc + k < R) dst[zd + (long long)gr * ldd + gc + k] = e[k];
    }
  }
}

}  // namespace

void transpose_bf16(const __nv_bfloat16* src, long long lds, __nv_bfloat16* dst, long long ldd, int batch, int R,
                    int C, cudaStream_t s) {
  if (R <= 0 || C <= 0 || batch <= 0) return;
  dim3 grid((C + 63) / 64, (R + 63) / 64, batch);
  transpose_bf16_kernel<<<grid, 256, 0, s>>>(src, lds, dst, ldd, R, C);
}

namespace {

// One row of a split operand: the logical (R, K) fp32 matrix element (r, k) sits at
// src[r * ld_row + k * ld_col]; dst row r holds three K-wide bf16 segments (each padded to
// Kp with zeros): pattern 0 = [hi, hi, lo], pattern 1 = [hi, lo, hi], where hi = bf16(x)
// rounded to nearest and lo = bf16(x - hi).  A K-concatenated product of a pattern-0 A and
// a pattern-1 B is hi_a hi_b + hi_a lo_b + lo_a hi_b: the bf16x3 splitting of Henry, Tang
// and Heinecke (2019), accurate to about 2^-16 relative before the fp32 accumulation.
__global__ void split3_bf16_kernel(const float* __restrict__ src, long long ld_row, long long ld_col,
                                   __nv_bfloat16* __restrict__ dst, int R, int K, int Kp, int pattern) {
  const long long total = (long long)R * Kp;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / Kp;
    const int k = (int)(i - r * Kp);
    const float x = k < K ? src[r * ld_row + (long long)k * ld_col] : 0.f;
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    const __nv_bfloat16 lo = __float2bfloat16_rn(x - __bfloat162float(hi));
    __nv_bfloat16* row = dst + r * 3LL * Kp;
    row[k] = hi;
    row[Kp + k] = pattern == 0 ? hi : lo;
    row[2 * Kp + k] = pattern == 0 ? lo : hi;
  }
}

}  // namespace

void split3_bf16(const float* src, long long ld_row, long long ld_col, __nv_bfloat16* dst, int R, int K, int Kp,
                 int pattern, cudaStream_t s) {
  if (R <= 0 || Kp <= 0) return;
  const long long total = (long long)R * Kp;
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 148LL * 16);
  split3_bf16_kernel<<<(unsigned)blocks, threads, 0, s>>>(src, ld_row, ld_col, dst, R, K, Kp, pattern);
}

}  // namespace bw
