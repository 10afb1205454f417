// Counter-based random projection matrices, generated on the device.
//
// Entry (i, j) of a (d_in x k) projection is a pure function of
// (seed, d_in, k, i, j): a SplitMix64 finalizer (Steele, Lea & Flood 2014) of the
// counter  key(seed, d_in, k) + i*k + j.  Rademacher entries take the sign of bit
// 63 and are scaled by 1/sqrt(k) so that E[<Pa, Pb>] = <a, b>; Gaussian entries
// use the Box-Muller transform of two 24-bit uniforms drawn from the same hash.
// The matrix is written transposed, (k x d_in) and K-major, which is the B operand
// layout of the tcgen05 GEMM:  x . P  ==  gemm_tn(x, P^T).
// The identical generator in pure PyTorch lives in
// dattri_llm_b200/gradient/ops/projection.py (`counter_projection_matrix`).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>

#include "projector.cuh"

namespace bw {
namespace {

__host__ __device__ __forceinline__ unsigned long long splitmix64(unsigned long long x) {
  x += 0x9E3779B97F4A7C15ull;
  unsigned long long z = x;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ unsigned long long proj_key(long long seed, long long d_in,
                                                                long long k) {
  return splitmix64(splitmix64((unsigned long long)seed) ^
                    ((unsigned long long)d_in * 0x100000001B3ull) ^ (unsigned long long)k);
}

__device__ __forceinline__ void store_val(float* p, double v) { *p = (float)v; }
__device__ __forceinline__ void store_val(__nv_bfloat16* p, double v) {
  *p = __float2bfloat16((float)v);
}

// out[j][i] = P[i][j]; kind 0 = Rademacher, 1 = Gaussian.
template <typename T>
__global__ void projection_kernel(T* out, long long d_in, long long k, unsigned long long key,
                                  int kind, double scale) {
  const long long total = d_in * k;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long j = e / d_in;  // output row (projection coordinate)
    const long long i = e % d_in;  // input feature
    const unsigned long long h = splitmix64(key + (unsigned long long)(i * k + j));
    double v;
    if (kind == 0) {
      v = (h >> 63) ? -1.0 : 1.0;
    } else {
      const double u1 = ((double)(h >> 40) + 0.5) * (1.0 / 16777216.0);
      const double u2 = ((double)((h >> 16) & 0xFFFFFFull) + 0.5) * (1.0 / 16777216.0);
      v = sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
    }
    store_val(out + e, v * scale);
  }
}

torch::Tensor projection_matrix_t(int64_t d_in, int64_t k, int64_t seed, int64_t kind,
                                  double scale, torch::ScalarType dtype, torch::Device device) {
  TORCH_CHECK(device.is_cuda(), "projection_matrix_t generates on a CUDA device");
  const c10::cuda::CUDAGuard guard(device);
  auto out = torch::empty({k, d_in}, torch::TensorOptions().dtype(dtype).device(device));
  const unsigned long long key = proj_key(seed, d_in, k);
  const long long total = d_in * k;
  const int threads = 256;
  const int blocks = (int)std::min<long long>((total + threads - 1) / threads, 148 * 16);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (dtype == torch::kBFloat16)
    projection_kernel<<<blocks, threads, 0, stream>>>(
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), d_in, k, key, (int)kind, scale);
  else if (dtype == torch::kFloat32)
    projection_kernel<<<blocks, threads, 0, stream>>>(out.data_ptr<float>(), d_in, k, key,
                                                      (int)kind, scale);
  else
    TORCH_CHECK(false, "projection dtype must be bfloat16 or float32");
  return out;
}

}  // namespace

void register_projector(pybind11::module& m) {
  m.def("projection_matrix_t", &projection_matrix_t,
        "(k, d_in) transposed counter-based random projection matrix");
  m.def("projection_key", [](int64_t seed, int64_t d_in, int64_t k) {
    return (int64_t)proj_key(seed, d_in, k);
  });
}

}  // namespace bw
