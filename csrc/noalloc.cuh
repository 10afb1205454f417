// C interface of the no-allocation split-K GEMM (defined in noalloc.cu).
//
// This interface has no counterpart in the reference framework.  It serves callers that
// cannot allocate device memory when they call in: C or C++ hosts that link this library
// without PyTorch (and so without PyTorch's caching allocator), and serving runtimes that
// forbid cudaMalloc/cudaFree once requests are in flight, because those calls synchronise
// the device and can fail under memory pressure.  The GEMM's fp32 split-K accumulator
// lives in a fixed file-scope device array instead of an allocation.
//
// Limits and rules:
//   * M * N <= dattri_b200_noalloc_max_output() (2,097,152 fp32 sums, 8 MiB of scratch per
//     device, held by every device that loads the library until the process exits).
//     Larger calls return cudaErrorInvalidValue and launch nothing.
//   * A (M x K) and B (N x K) are bf16, K-major, 16-byte aligned, K and both row strides
//     multiples of 8 elements; C is bf16 (M x N, row stride ldc >= N).
//   * Every call on a device shares the one scratch array and keeps the last call's sums
//     there.  Each call clears what it uses on the caller's stream first, but calls that
//     overlap on the GPU (different streams with no ordering between them, or several host
//     threads) race on the array and corrupt each other's results: order them.
//   * The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) and raises the GEMM kernel's shared-memory limit.  Make that
//     first call (or dattri_b200_noalloc_setup()) on each device, with that device current,
//     before any stream capture.
//
// Return values are cudaError_t codes as int (0 = success).
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Looks up the current device's scratch address once (idempotent).
int dattri_b200_noalloc_setup(void);

// Largest M * N that one call accepts.
long long dattri_b200_noalloc_max_output(void);

// C (bf16) = alpha * A @ B^T on `stream`, K split over `splits` CTAs per output tile whose
// fp32 partial sums meet in the static scratch; a second kernel rounds them to bf16.
int dattri_b200_gemm_bf16_splitk_noalloc(const void* a, const void* b, void* c, int M, int N, int K,
                                          long long lda, long long ldb, long long ldc, float alpha,
                                          int splits, cudaStream_t stream);

// Reads the current device's error word into *out (0 = no device-side error) after every
// call queued on `stream` so far has finished: the read is queued on `stream` and the
// function waits for that stream.  A nonzero word means a bounded wait inside the GEMM gave
// up; the result of that call is not valid.
int dattri_b200_noalloc_status(int* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
