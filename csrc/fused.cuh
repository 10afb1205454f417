// Host interface of the fused elementwise / row-reduction kernels (fused.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace bw {

void rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, float* rstd, int rows,
                 int cols, float eps, cudaStream_t s);
void rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w, const float* rstd,
                 __nv_bfloat16* dx, int rows, int cols, cudaStream_t s);
void swiglu_fwd(const __nv_bfloat16* g, const __nv_bfloat16* u, __nv_bfloat16* h, long long n, cudaStream_t s);
void swiglu_bwd(const __nv_bfloat16* dh, const __nv_bfloat16* g, const __nv_bfloat16* u, __nv_bfloat16* dg,
                __nv_bfloat16* du, long long n, cudaStream_t s);
void ce_fwd(const __nv_bfloat16* logits, const int64_t* target, float* loss, float* lse, int rows, int cols,
            long long ld, cudaStream_t s);
void ce_bwd_inplace(__nv_bfloat16* logits, const float* lse, const int64_t* target, const float* gscale,
                    int rows, int cols, long long ld, cudaStream_t s);

}  // namespace bw
