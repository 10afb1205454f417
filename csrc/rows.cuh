// Host interface of the warp-per-row decoder kernels (rows.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bw {

// y = rmsnorm(x [+ delta]) * w; with delta, h receives the bf16 sum x + delta.
struct RowsNorm {
  const __nv_bfloat16* x;
  const __nv_bfloat16* delta;  // nullable
  __nv_bfloat16* h;            // written iff delta != nullptr
  const __nv_bfloat16* w;
  __nv_bfloat16* y;
  float* rstd;
  int rows, cols;
  float eps;
};

// dx = rmsnorm_bwd(dy; x, w, rstd) [+ dres]
struct RowsNormBwd {
  const __nv_bfloat16* dy;
  const __nv_bfloat16* x;
  const __nv_bfloat16* w;
  const float* rstd;
  const __nv_bfloat16* dres;  // nullable
  __nv_bfloat16* dx;
  int rows, cols;
};

// One rotated tensor: element (b, t, h, d) at in[b*in_sb + t*in_st + h*in_sh + d].
struct RopeTensor {
  const __nv_bfloat16* in;
  __nv_bfloat16* out;
  long long in_sb, in_st, in_sh;
  long long out_sb, out_st, out_sh;
};

struct RopeArgs {
  RopeTensor q, k;
  const float* cos;  // (seq, head_dim / 2) fp32
  const float* sin;
  int batch, seq, hq, hk, head_dim;
};

bool rows_norm_supported(int cols);
void rows_norm_fwd(const RowsNorm& a, cudaStream_t s);
void rows_norm_bwd(const RowsNormBwd& a, cudaStream_t s);
void rope(const RopeArgs& a, bool inverse, cudaStream_t s);
bool rope_supported(int head_dim, int heads);  // heads = q heads + k heads
// SwiGLU over [gate | up] rows (rows read from device memory; max_rows sizes the grid).
void swiglu_split(const __nv_bfloat16* h, __nv_bfloat16* out, const int* rows, int max_rows, int inter, cudaStream_t s);
void swiglu_split_bwd(const __nv_bfloat16* da, const __nv_bfloat16* h, __nv_bfloat16* dh, const int* rows,
                      int max_rows, int inter, cudaStream_t s);
void adam_direction(const float* g, const float* m0, const float* v0, float* out, long long rows, long long p,
                    float b1, float b2, float inv_bc1, float inv_sqrt_bc2, float eps, cudaStream_t s);

// dst[z] (C x R, row stride ldd) = src[z]^T (src: R x C, row stride lds), bf16; batch z.
// Row strides and base pointers 16-byte aligned (8 elements) for the vector path.
void transpose_bf16(const __nv_bfloat16* src, long long lds, __nv_bfloat16* dst, long long ldd, int batch, int R,
                    int C, cudaStream_t s);

// bf16x3 split of a strided fp32 (R, K) matrix into a (R, 3 Kp) bf16 K-major operand:
// pattern 0 = [hi | hi | lo], pattern 1 = [hi | lo | hi] (see rows.cu).
void split3_bf16(const float* src, long long ld_row, long long ld_col, __nv_bfloat16* dst, int R, int K, int Kp,
                 int pattern, cudaStream_t s);

}  // namespace bw
