// Host-side interface of the generic tcgen05 GEMM (gemm_tc.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace bw {

// Epilogue modes.
enum GemmStore : int {
  kStoreF32 = 0,    // C (fp32) = alpha * AB^T            (or += with beta_accumulate)
  kStoreBF16 = 1,   // C (bf16) = alpha * AB^T
  kAtomicF32 = 2,   // C (fp32) += alpha * AB^T with atomics (split-K / cross-CTA sums)
  kStoreBF16T = 3,  // C^T (bf16): element (m, n) lands at C[z][n * ldc + m]
  kStoreBF16TB = 4, // per-segment C^T (bf16): rows are (s, t) with T = ldc rows per segment;
                    // element (m, n) lands at C[z][m / T][n][m % T] (a (S, N, T) block)
  // 5: unused (an earlier peer-atomic reduce; replaced by kPeerSlotF32)
  kStoreBF16Scatter = 6,  // bf16 row m stored into rank scatter[m].x's C at row scatter[m].y
                          // (peer pointers; expert outputs returned to their source ranks)
  kSqAccF32 = 8,     // C (fp32, one matrix) += (alpha * AB^T)^2 summed over the batch (atomics)
  kPeerSlotF32 = 7,  // reduce-scatter: element i (owner o = (i / 4) / per4) is STORED into
                     // peers[o][self_rank * 4 * per4 + i - o * 4 * per4] (the owner's slot for
                     // this rank); the owner sums its slots afterwards (splits must be 1)
  kStoreBF16Tail = 9,  // columns n < n_main: bf16 C[m][n] (row stride ldc); columns n >= n_main
                       // (the tail, from a second B operand): token-major bf16 C2, element
                       // (m, n) at C2[m / seg2][n - n_main][m % seg2] (a (S, N - n_main, seg2) block)
};

// A K-major bf16 operand: `batch` matrices of rows x cols (cols = K, contiguous).
struct GemmOperand {
  const void* ptr;
  long long rows;
  long long cols;
  long long row_stride;    // elements between consecutive rows (>= cols, multiple of 8)
  long long batch;         // 1 for a single matrix
  long long batch_stride;  // elements between consecutive matrices
};

struct GemmParams {
  int M, N, K;
  int batch;       // number of (A, C) batches; grid.z = batch * splits
  int splits;      // split-K factor
  int b_shared;    // 1: every batch uses B[0]
  int c_mode;      // GemmStore
  int beta_accumulate;
  float alpha;
  void* C;
  long long ldc;
  long long batch_stride_c;
  int* err;
  int cluster_k;   // >1: the split-K CTAs of a tile form a cluster and sum over DSMEM (set by the launcher)
  float* const* peers;  // kPeerSlotF32 / kStoreBF16Scatter: device array of every rank's buffer (peer-mapped)
  int world;
  long long per4;       // kPeerSlotF32: float4 elements owned by each rank
  int self_rank;        // kPeerSlotF32: this rank (selects its slot in the owners' buffers)
  const int2* scatter;  // kStoreBF16Scatter: (rank, row) of every output row
  int n_main;           // kStoreBF16Tail: columns that come from B (a multiple of 256)
  void* C2;             // kStoreBF16Tail: the tail's token-major output
  long long seg2;       // kStoreBF16Tail: tokens per segment (sample) of C2
};

// One job of a grouped launch (tensor maps in global memory, 64-byte aligned).
struct GroupJob {
  const CUtensorMap* ta;
  const CUtensorMap* tb;
  void* C;
  long long pad;
};

constexpr int kMaxPeerMaps = 8;  // single node

// A staged launch: copy the remote peers' shards of B into the local staging matrix `dst`
// (every remote byte once, over NVLink) inside the GEMM launch that consumes it.
struct StageArgs {
  const void* src[kMaxPeerMaps];  // each rank's shard (peer-mapped), bf16
  long long src_stride;           // elements between shard rows
  int src_rows;                   // rows of a shard
  long long row_elems;            // elements copied per row (multiple of 8)
  void* dst;                      // local staging matrix, bf16
  long long dst_stride;           // elements between staging rows
  long long dst_row0[kMaxPeerMaps];  // where owner r's rows start in dst
  long long dst_col0[kMaxPeerMaps];  // where owner r's columns start in dst (multiple of 8)
  int piece_rows, pieces_per_owner;
  int* flags;                     // per owner, monotonic
  int expect;                     // per-owner flag value once this launch's copy is complete
  int world, self, mode, shard, copiers;
};

CUtensorMap make_tmap_kmajor_bf16(const GemmOperand& op, int box_rows);
// B sharded over the peers; pm: device array of their tensor maps (64-byte aligned).
// mode 0: B rows sharded (shard rows each); mode 1: B's K sharded (shard columns each).
void gemm_peers_launch(const GemmOperand& A, const CUtensorMap* pm, GemmParams p, int mode, int shard, int bn,
                       cudaStream_t stream);
void gemm_grouped_launch(const GroupJob* jobs, int n_jobs, GemmParams p, int bn, cudaStream_t stream);
// Ragged grouped GEMM: A (rows, K) with per-job row segments, B3 (jobs, N, K); device arrays
// tile_prefix[jobs + 1], base[jobs], len[jobs]; grid height max_tiles (an upper bound).
void gemm_ragged_launch(const GemmOperand& A, const GemmOperand& B3, GemmParams p, const int* tile_prefix,
                        const int* base, const int* len, int jobs, int max_tiles, int bn, cudaStream_t stream);
// mode 0: B rows sharded (stage_op = the (N, K) staging matrix, own = this rank's (shard, K));
// mode 1: B's K sharded (stage_op = the (N, K) staging matrix, own = this rank's (N, shard)).
void gemm_staged_launch(const GemmOperand& A, const GemmOperand& stage_op, const GemmOperand& own, GemmParams p,
                        StageArgs sa, int bn, cudaStream_t stream);
int pick_bn(int N);
void gemm_tn_launch(const GemmOperand& A, const GemmOperand& B, GemmParams p, int bn,
                    cudaStream_t stream);
// C (fp32, M x M, row stride p.ldc) += p.alpha * At @ At^T (At: M x K, K-major) -- a
// covariance / Gram accumulation.  Only tiles on and above the diagonal are computed (each
// off-diagonal one also adds its transpose), split along K over the CTA pairs, atomic fp32
// epilogue.  p.M = p.N = At's rows, p.K = its columns.
void gram_acc_launch(const GemmOperand& At, GemmParams p, cudaStream_t stream);
// C = A @ [B; Btail]^T in one CTA-pair launch with the kStoreBF16Tail store: the main columns
// (B's rows, p.n_main of them, a multiple of 256) in row-major bf16 and the tail (Btail's rows,
// at most 256) token-major -- e.g. a layer's output and its projected activation from one pass
// over the activation.  p.N = n_main + Btail's rows.  Returns false when CTA pairs cannot run
// here (nothing launched).
bool gemm_tn_tail_launch(const GemmOperand& A, const GemmOperand& B, const GemmOperand& Btail, GemmParams p,
                         cudaStream_t stream);

}  // namespace bw
