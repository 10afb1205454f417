// Host interface of the mask-projection gather-contract kernel (mask_gather.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bw {

// out[b][m] = sum_t R[b][t][rows[m]] * C[b][t][cols[m]] for b < B, m < M (fp32 out).
// R is (B, T, KR) and C is (B, T, KC), bf16, contiguous and 16-byte aligned; KR and KC
// multiples of 8.  A bounded wait that gives up sets *err (the kernel's error word).
void mask_gather(const __nv_bfloat16* R, const __nv_bfloat16* C, const int* rows, const int* cols, float* out,
                 int B, int T, int KR, int KC, int M, int* err, cudaStream_t s);

}  // namespace bw
