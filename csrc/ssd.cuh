// Host interface of the intra-chunk SSD kernels (ssd.cu).
#pragma once

#include <cuda_runtime.h>

namespace bw {

// Shapes (fp32, contiguous): cb (B, G, C, S, S) = C_s . B_t per group; cum (B, H, C, S), the
// cumulative log-decay inside each chunk; x and y (B, C, S, H, P).  Head h reads group
// h / (H / G).  S a multiple of 64, P == 64.
//
// y[b, c, s, h, :] = sum_{t <= s} cb[b, g, c, s, t] * exp(cum[b, h, c, s] - cum[b, h, c, t]) * x[b, c, t, h, :]
void ssd_intra_fwd(const float* cb, const float* cum, const float* x, float* y, int B, int C, int S, int H, int G,
                   cudaStream_t s);

// Its backward from dy: dx (written), dcb and dcum (accumulated: pass zeroed buffers).
void ssd_intra_bwd(const float* cb, const float* cum, const float* x, const float* dy, float* dx, float* dcb,
                   float* dcum, int B, int C, int S, int H, int G, cudaStream_t s);

}  // namespace bw
