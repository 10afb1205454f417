// Host interface of the causal depthwise convolution + SiLU kernels (conv1d.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bw {

constexpr int kConvTaps = 4;  // the Mamba2 convolution width (d_conv)

// out[b, t, c] = silu(bias[c] + sum_k w[c, k] x[b, t - 3 + k, c]) (zero before t = 0): x bf16
// with row stride ldx and batch stride sbx (elements; unit channel stride), w (C, 4) and bias
// (C) bf16 (bias may be null), out (B, L, C) bf16 contiguous.  C even, x 4-byte aligned.
void causal_conv_silu_fwd(const __nv_bfloat16* x, long long ldx, long long sbx, const __nv_bfloat16* w,
                          const __nv_bfloat16* bias, __nv_bfloat16* out, int B, int L, int C, cudaStream_t s);

// Rows of the fp32 partial-sum workspaces the backward needs: (parts, C, 4) and (parts, C).
int causal_conv_bwd_parts(int B, int L);

// Backward from dout (B, L, C) bf16 contiguous: dx (B, L, C) bf16 contiguous, dw (C, 4) and
// dbias (C) fp32 (through the partial-sum workspaces).
void causal_conv_silu_bwd(const __nv_bfloat16* dout, const __nv_bfloat16* x, long long ldx, long long sbx,
                          const __nv_bfloat16* w, const __nv_bfloat16* bias, __nv_bfloat16* dx, float* dw_part,
                          float* db_part, float* dw, float* db, int B, int L, int C, cudaStream_t s);

}  // namespace bw
