// Host interface of the gated RMSNorm kernels (gated_norm.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bw {

constexpr int kGatedNormMaxCols = 8192;

// out (bf16, rows x cols, contiguous) = w * rmsnorm(y * silu(g)), with y fp32 contiguous and
// g bf16 of row stride ldg; rstd (rows) receives 1 / sqrt(mean((y silu(g))^2) + eps).
void gated_rms_fwd(const float* y, const __nv_bfloat16* g, long long ldg, const __nv_bfloat16* w,
                   __nv_bfloat16* out, float* rstd, int rows, int cols, float eps, cudaStream_t s);

// Rows of the fp32 (parts x cols) partial-sum workspace gated_rms_bwd needs for `rows` rows.
int gated_rms_bwd_parts(int rows);

// Backward of gated_rms_fwd from dout (bf16, contiguous): dy (fp32, contiguous), dg (bf16,
// contiguous) and dw (fp32, cols), through dw_part (gated_rms_bwd_parts(rows) x cols fp32).
void gated_rms_bwd(const __nv_bfloat16* dout, const float* y, const __nv_bfloat16* g, long long ldg,
                   const __nv_bfloat16* w, const float* rstd, float* dy, __nv_bfloat16* dg, float* dw_part, float* dw,
                   int rows, int cols, cudaStream_t s);

}  // namespace bw
