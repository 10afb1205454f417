// Dense per-sample embedding gradients:
//
//     out[b * vocab + v, :] = sum over tokens t of sample b with id v of g[b, t, :]
//
// The output (B * vocab rows of E) is far larger than the token gradients, so the kernel is
// bound by writing it.  Every output row is written exactly once -- zeros where the sample
// never saw that id, the fp32 sum of its token rows otherwise -- with 16-byte streaming
// stores, instead of a separate zero fill followed by a scatter-add that rewrites the hit
// rows.  The caller passes the tokens sorted by key b * vocab + id (stable, so the sum runs
// in token order and the result is deterministic) and where each output row's tokens start in
// that order; each warp owns a short run of consecutive output rows.
#include <cuda_bf16.h>

#include "embed_grad.cuh"

namespace bw {
namespace {

constexpr int kWarps = 8;
constexpr int kRowsPerWarp = 4;  // short runs: thousands of warps keep the stores in flight

template <bool kBF16>
__device__ __forceinline__ void add16(float* acc, const uint4& q) {
  if constexpr (kBF16) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      acc[2 * e] += f.x;
      acc[2 * e + 1] += f.y;
    }
  } else {
    acc[0] += __uint_as_float(q.x);
    acc[1] += __uint_as_float(q.y);
    acc[2] += __uint_as_float(q.z);
    acc[3] += __uint_as_float(q.w);
  }
}

template <bool kBF16>
__device__ __forceinline__ uint4 pack16(const float* acc) {
  uint4 q;
  if constexpr (kBF16) {
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&q);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
  } else {
    q = make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                   __float_as_uint(acc[3]));
  }
  return q;
}

template <bool kBF16>
__global__ void __launch_bounds__(kWarps * 32)
    embed_dense_kernel(const long long* __restrict__ starts, const long long* __restrict__ order,
                       const uint4* __restrict__ g, uint4* __restrict__ out, long long R, int nv) {
  constexpr int kPer = kBF16 ? 8 : 4;
  const int lane = threadIdx.x & 31;
  const long long r0 = ((long long)blockIdx.x * kWarps + (threadIdx.x >> 5)) * kRowsPerWarp;
  if (r0 >= R) return;
  const long long r1 = r0 + kRowsPerWarp < R ? r0 + kRowsPerWarp : R;
  for (long long r = r0; r < r1; ++r) {
    const long long c = __ldg(starts + r), e = __ldg(starts + r + 1);  // row r's sorted tokens
    uint4* orow = out + r * nv;
    if (e == c) {
      for (int v = lane; v < nv; v += 32) __stcs(orow + v, make_uint4(0u, 0u, 0u, 0u));
      continue;
    }
    for (int v = lane; v < nv; v += 32) {
      float acc[kPer];
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc[i] = 0.f;
      for (long long j = c; j < e; ++j) add16<kBF16>(acc, __ldg(g + __ldg(order + j) * nv + v));
      __stcs(orow + v, pack16<kBF16>(acc));
    }
  }
}

}  // namespace

void embedding_dense_grad(const int64_t* starts, const int64_t* order, const void* g, void* out, long long R,
                          int E, int elem_bytes, cudaStream_t s) {
  if (R <= 0) return;
  const int nv = E * elem_bytes / 16;
  const long long rows_per_cta = (long long)kWarps * kRowsPerWarp;
  const unsigned grid = (unsigned)((R + rows_per_cta - 1) / rows_per_cta);
  const long long* k = reinterpret_cast<const long long*>(starts);
  const long long* o = reinterpret_cast<const long long*>(order);
  if (elem_bytes == 2)
    embed_dense_kernel<true><<<grid, kWarps * 32, 0, s>>>(k, o, static_cast<const uint4*>(g),
                                                          static_cast<uint4*>(out), R, nv);
  else
    embed_dense_kernel<false><<<grid, kWarps * 32, 0, s>>>(k, o, static_cast<const uint4*>(g),
                                                           static_cast<uint4*>(out), R, nv);
}

}  // namespace bw
