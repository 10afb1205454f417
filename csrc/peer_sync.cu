// Cross-GPU barrier over NVLink peer memory, with a bounded wait.
//
// Every rank owns a small int32 flag array in symmetric memory (one slot per rank), mapped
// into every peer.  Barrier `epoch` (monotonic, never reused): rank r stores `epoch` into
// slot r of every rank's array (st.release.sys, after a system-scope fence so the rank's
// earlier writes -- e.g. its train block -- are visible to peers first), then waits until
// every slot of its own array holds >= epoch (ld.acquire.sys).  A wait that runs past 2 s
// writes kErrWaitPeer into the error word and returns, so a lost peer surfaces on the host
// instead of hanging the GPU.  One launch per rank per barrier, one rank per GPU.
#include <cuda_runtime.h>

#include "tc_common.cuh"
#include "peer_sync.cuh"

namespace bw {
namespace {

__global__ void peer_barrier_kernel(int* const* __restrict__ flags, int rank, int world, int epoch, int* err) {
  const int t = threadIdx.x;
  if (t < world) {
    __threadfence_system();
    int* slot = flags[t] + rank;
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(slot), "r"(epoch) : "memory");
  }
  __syncthreads();
  if (t < world) {
    const int* mine = flags[rank] + t;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if (v >= epoch) break;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        report_error(err, kErrWaitPeer);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace

void peer_barrier(int* const* flags_dev, int rank, int world, int epoch, int* err, cudaStream_t s) {
  const int threads = ((world + 31) / 32) * 32;
  peer_barrier_kernel<<<1, threads, 0, s>>>(flags_dev, rank, world, epoch, err);
}

}  // namespace bw
