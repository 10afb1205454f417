// No-allocation entry point: split-K bf16 GEMM through a static fp32 scratch accumulator.
//
// This entry point has no counterpart in the reference framework; it exists for callers
// that cannot allocate device memory at call time:
//   * host code that links this library through its C symbols, without PyTorch and
//     therefore without PyTorch's caching allocator;
//   * runtimes that forbid cudaMalloc/cudaFree once they are serving, because those
//     calls synchronise the device and can fail under memory pressure mid-request;
//   * code that runs while the caller holds a lock or a stream recording that must not
//     trigger an allocator (the caller decides what that means for its own case).
//
// What it computes: C (bf16, M x N, row stride ldc) = alpha * A @ B^T, with A (M x K) and
// B (N x K) bf16, K-major.  K is split over `splits` CTAs per output tile; their fp32
// partial sums meet in a scratch accumulator by atomics, and a second kernel rounds the
// finished sums to bf16.  The tcgen05 GEMM kernel is the same one the PyTorch entry
// point `gemm_tn` launches (mode kAtomicF32); only where its output lands differs.
//
// Scratch: one file-scope device array per device (`g_scratch`), 8 MiB + 256 B.  Its
// first 256 B hold the kernels' error word; the rest holds up to kMaxOutput fp32 sums,
// so M * N must not exceed 2,097,152 (calls above that are rejected, nothing launched).
// Every call clears the error word and the M * N accumulator on the caller's stream
// before the GEMM (cudaMemsetAsync, which allocates nothing), so sums never leak from
// one call into the next.
//
// Concurrency: the scratch is shared by every call on a device.  Two calls that can
// overlap in time -- on different streams, or from different host threads without an
// ordering between their streams -- race on it and corrupt each other's results.
// Serialise calls on one device (one stream, or events between streams).
//
// Setup: the first call on each device does one-time host work -- it looks up the
// scratch address (cudaGetSymbolAddress, return code checked) and, the first time each
// GEMM tile width runs there, raises that kernel's shared-memory limit
// (cudaFuncSetAttribute).  Do that first call outside any stream capture: make one
// ordinary call with the same N on each device before capturing a stream.
// dattri_b200_noalloc_setup() performs the scratch lookup alone.
//
// Return value: a cudaError_t as int (0 = launched).  Device-side wait timeouts land in
// the error word, read with dattri_b200_noalloc_status(), which is ordered after the
// caller's stream.  The prototypes, with these limits, are in noalloc.cuh.
#include "noalloc.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "gemm_tc.cuh"

namespace {

constexpr long long kHeaderFloats = 64;            // 256 B: the error word and padding
constexpr long long kMaxOutput = 1ll << 21;        // fp32 sums: 8 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_scratch[kHeaderFloats + kMaxOutput];

float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_setup_mutex;

__global__ void round_to_bf16(const float* __restrict__ acc, __nv_bfloat16* __restrict__ c, int M, int N,
                              long long ldc) {
  const long long total = (long long)M * N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / N, n = i - m * N;
    c[m * ldc + n] = __float2bfloat16(acc[i]);
  }
}

// The scratch base of the current device, looked up once per device.
cudaError_t scratch_base(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 256 != 0) return cudaErrorInvalidSymbol;
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

// Look up the current device's scratch address (idempotent).
extern "C" __attribute__((visibility("default"))) int dattri_b200_noalloc_setup() {
  float* base = nullptr;
  return static_cast<int>(scratch_base(&base));
}

// Largest M * N one call accepts.
extern "C" __attribute__((visibility("default"))) long long dattri_b200_noalloc_max_output() {
  return kMaxOutput;
}

// C (bf16) = alpha * A @ B^T with K split over `splits` CTAs; see the file comment.
extern "C" __attribute__((visibility("default"))) int dattri_b200_gemm_bf16_splitk_noalloc(
    const void* a, const void* b, void* c, int M, int N, int K, long long lda, long long ldb,
    long long ldc, float alpha, int splits, cudaStream_t stream) {
  if (a == nullptr || b == nullptr || c == nullptr) return cudaErrorInvalidValue;
  if (M <= 0 || N <= 0 || K <= 0 || K % 8 != 0) return cudaErrorInvalidValue;
  if (lda < K || ldb < K || lda % 8 != 0 || ldb % 8 != 0 || ldc < N) return cudaErrorInvalidValue;
  if (!aligned16(a) || !aligned16(b) || reinterpret_cast<uintptr_t>(c) % 2 != 0)
    return cudaErrorInvalidValue;
  if ((long long)M * N > kMaxOutput) return cudaErrorInvalidValue;
  const int k_blocks = (K + 63) / 64;
  if (splits < 1) splits = 1;
  if (splits > k_blocks) splits = k_blocks;
  const int per_split = (k_blocks + splits - 1) / splits;
  splits = (k_blocks + per_split - 1) / per_split;  // every split owns at least one K block

  float* base = nullptr;
  cudaError_t e = scratch_base(&base);
  if (e != cudaSuccess) return e;
  float* acc = base + kHeaderFloats;
  int* err = reinterpret_cast<int*>(base);
  e = cudaMemsetAsync(base, 0, (kHeaderFloats + (long long)M * N) * sizeof(float), stream);
  if (e != cudaSuccess) return e;

  bw::GemmOperand A{a, M, K, lda, 1, (long long)M * lda};
  bw::GemmOperand B{b, N, K, ldb, 1, (long long)N * ldb};
  bw::GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.batch = 1;
  p.splits = splits;
  p.b_shared = 1;
  p.c_mode = bw::kAtomicF32;
  p.beta_accumulate = 0;
  p.alpha = alpha;
  p.C = acc;
  p.ldc = N;
  p.batch_stride_c = (long long)M * N;
  p.err = err;
  try {
    bw::gemm_tn_launch(A, B, p, bw::pick_bn(N), stream);
  } catch (...) {
    return cudaErrorInvalidValue;  // tensor-map encoding rejected the operands
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const long long total = (long long)M * N;
  const int threads = 256;
  const int blocks = (int)((total + threads - 1) / threads < 148 * 8 ? (total + threads - 1) / threads : 148 * 8);
  round_to_bf16<<<blocks, threads, 0, stream>>>(acc, static_cast<__nv_bfloat16*>(c), M, N, ldc);
  return static_cast<int>(cudaGetLastError());
}

// Copy the current device's error word to *out once every call queued on `stream` has
// finished (0 = no device error).  The copy is queued on `stream` itself, so it is ordered
// after the GEMM even when `stream` does not synchronise with the legacy default stream.
extern "C" __attribute__((visibility("default"))) int dattri_b200_noalloc_status(int* out,
                                                                                  cudaStream_t stream) {
  if (out == nullptr) return cudaErrorInvalidValue;
  int word = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&word, g_scratch, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  *out = word;
  return cudaSuccess;
}
