// Host interface of the cross-GPU barrier (peer_sync.cu).
#pragma once

#include <cuda_runtime.h>

namespace bw {

// flags_dev: device array of `world` pointers, entry r = rank r's flag array (peer-mapped).
void peer_barrier(int* const* flags_dev, int rank, int world, int epoch, int* err, cudaStream_t s);

}  // namespace bw
