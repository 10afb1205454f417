// Host interface of the per-sample norm-parameter gradient kernel (norm_grad.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace bw {

// dw, db: (B, d) fp32, zeroed by the caller (db may be null); d a multiple of 8, <= 16384.
void norm_per_sample_grad(const __nv_bfloat16* x, const __nv_bfloat16* g, float* dw, float* db, int B, int T, int d,
                          float eps, bool layer_norm, cudaStream_t s);

}  // namespace bw
