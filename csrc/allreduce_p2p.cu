// Sum all-reduce of fp32 buffers over NVLink peer memory (one process per GPU).
//
// Every rank's input sits in a symmetric-memory buffer mapped into all peers.  Two forms:
//   * one-shot  (small buffers): every rank reads every peer's whole buffer and writes the
//     sum into its own output -- one pass, latency-bound sizes;
//   * two-shot  (large buffers): reduce-scatter then all-gather.  Rank r sums slice r of all
//     peers' buffers into slice r of its OWN buffer (no other rank reads that slice in this
//     phase); after a barrier every rank copies each reduced slice from its owner.
// Loads and stores are 16-byte vectors through plain peer pointers (no TMA, no multicast).
// The callers bracket the phases with the bounded cross-GPU barrier (peer_sync.cu).
#include <cuda_runtime.h>

#include "allreduce_p2p.cuh"

namespace bw {
namespace {

constexpr int kMaxPeers = 16;

struct PeerPtrs {
  const float4* p[kMaxPeers];
};

__global__ void sum_slice_kernel(PeerPtrs in, int world, float4* out, long long begin4, long long end4) {
  for (long long i = begin4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < end4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = in.p[0][i];
    for (int r = 1; r < world; ++r) {
      const float4 v = in.p[r][i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    out[i] = acc;
  }
}

__global__ void gather_slices_kernel(PeerPtrs src, int world, float4* out, long long n4) {
  const long long per = (n4 + world - 1) / world;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    const int owner = (int)(i / per);
    out[i] = src.p[owner][i];
  }
}

// out[i] (+)= sum over s of slots[s * slot4 + i]: the owner's half of a reduce-scatter whose
// sources stored their partials into this rank's slots (local memory only).
__global__ void slot_reduce_kernel(const float4* __restrict__ slots, int world, long long slot4, float4* out,
                                   long long n4, int accumulate) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
       i += (long long)gridDim.x * blockDim.x) {
    float4 acc = accumulate ? out[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 v = slots[r * slot4 + i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    out[i] = acc;
  }
}

int grid_for(long long n4) {
  const long long b = (n4 + 255) / 256;
  return (int)(b < 1 ? 1 : (b < 148 * 8 ? b : 148 * 8));
}

PeerPtrs pack(const float* const* ptrs, int world) {
  PeerPtrs p{};
  for (int r = 0; r < world && r < kMaxPeers; ++r) p.p[r] = reinterpret_cast<const float4*>(ptrs[r]);
  return p;
}

}  // namespace

int allreduce_max_peers() { return kMaxPeers; }

void allreduce_oneshot(const float* const* peers, int world, float* out, long long n, cudaStream_t s) {
  const long long n4 = n / 4;
  if (n4 <= 0) return;
  sum_slice_kernel<<<grid_for(n4), 256, 0, s>>>(pack(peers, world), world, reinterpret_cast<float4*>(out), 0, n4);
}

void allreduce_reduce_scatter(const float* const* peers, int world, int rank, float* own, long long n,
                              cudaStream_t s) {
  const long long n4 = n / 4;
  const long long per = (n4 + world - 1) / world;
  const long long b = per * rank, e = b + per < n4 ? b + per : n4;
  if (e <= b) return;
  sum_slice_kernel<<<grid_for(e - b), 256, 0, s>>>(pack(peers, world), world, reinterpret_cast<float4*>(own), b, e);
}

void allreduce_all_gather(const float* const* peers, int world, float* out, long long n, cudaStream_t s) {
  const long long n4 = n / 4;
  if (n4 <= 0) return;
  gather_slices_kernel<<<grid_for(n4), 256, 0, s>>>(pack(peers, world), world, reinterpret_cast<float4*>(out), n4);
}

void slot_reduce(const float* slots, int world, long long slot, float* out, long long n, bool accumulate,
                 cudaStream_t s) {
  const long long n4 = n / 4;
  if (n4 <= 0) return;
  slot_reduce_kernel<<<grid_for(n4), 256, 0, s>>>(reinterpret_cast<const float4*>(slots), world, slot / 4,
                                                  reinterpret_cast<float4*>(out), n4, accumulate ? 1 : 0);
}

}  // namespace bw
