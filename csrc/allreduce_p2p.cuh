// Host interface of the NVLink peer-memory all-reduce (allreduce_p2p.cu).  `peers[r]` is
// rank r's symmetric buffer as mapped in this process; n is a multiple of 4 floats.
#pragma once

#include <cuda_runtime.h>

namespace bw {

int allreduce_max_peers();
void allreduce_oneshot(const float* const* peers, int world, float* out, long long n, cudaStream_t s);
void allreduce_reduce_scatter(const float* const* peers, int world, int rank, float* own, long long n,
                              cudaStream_t s);
// out[0, n) (+)= sum_s slots[s * slot + (0, n)] (slot and n multiples of 4 floats).
void slot_reduce(const float* slots, int world, long long slot, float* out, long long n, bool accumulate,
                 cudaStream_t s);
void allreduce_all_gather(const float* const* peers, int world, float* out, long long n, cudaStream_t s);

}  // namespace bw
