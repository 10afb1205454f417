// Python bindings of the native kernels (module dattri_llm_b200._C).
//
// Every entry point validates dtype, device, contiguity and the 16-byte alignment
// that TMA needs, then launches on the current PyTorch stream.  Kernels report
// bounded-wait timeouts into the int32 `err` tensor the caller passes in.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <cstring>
#include <string>
#include <mutex>
#include <unordered_map>

#include "gemm_tc.cuh"
#include "ghost_gram.cuh"
#include "fused.cuh"
#include "projector.cuh"
#include "rows.cuh"
#include "score_ag.cuh"
#include "peer_sync.cuh"
#include "allreduce_p2p.cuh"
#include "mask_gather.cuh"
#include "moe_ep.cuh"
#include "norm_grad.cuh"
#include "embed_grad.cuh"
#include "gated_norm.cuh"
#include "ssd.cuh"
#include "conv1d.cuh"

namespace {

using torch::Tensor;

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

void check_err(const Tensor& err) {
  check_cuda(err, "err");
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && err.numel() >= 1, "err must be int32[>=1]");
}

bw::GemmOperand operand(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK(t.dim() == 2 || t.dim() == 3, name, " must be 2-D or 3-D");
  TORCH_CHECK(t.stride(-1) == 1, name, " must be contiguous along K");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned");
  bw::GemmOperand op;
  op.ptr = t.data_ptr();
  op.rows = t.size(-2);
  op.cols = t.size(-1);
  op.row_stride = t.dim() >= 2 ? t.stride(-2) : t.size(-1);
  if (op.rows == 1) op.row_stride = ((op.cols + 7) / 8) * 8;
  TORCH_CHECK(op.row_stride % 8 == 0, name, " row stride must be a multiple of 8 elements");
  TORCH_CHECK(op.cols % 8 == 0, name, " K must be a multiple of 8");
  op.batch = t.dim() == 3 ? t.size(0) : 1;
  op.batch_stride = t.dim() == 3 ? t.stride(0) : op.rows * op.row_stride;
  if (op.batch > 1) TORCH_CHECK(op.batch_stride % 8 == 0, name, " batch stride must be 8-aligned");
  return op;
}

// C (op)= alpha * A @ B^T, see bw::GemmStore for `mode`.
void gemm_tn(Tensor A, Tensor B, Tensor C, double alpha, int64_t mode, int64_t splits,
             bool accumulate, Tensor err) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  auto b = operand(B, "B");
  TORCH_CHECK(a.cols == b.cols, "A and B disagree on K");
  check_cuda(C, "C");
  TORCH_CHECK(mode == bw::kStoreF32 || mode == bw::kStoreBF16 || mode == bw::kAtomicF32 || mode == bw::kStoreBF16T ||
                  mode == bw::kSqAccF32,
              "mode: fp32, bf16, fp32 atomic, transposed bf16 or squared-sum store");
  const bool bf16_out = mode == bw::kStoreBF16 || mode == bw::kStoreBF16T;
  TORCH_CHECK(C.scalar_type() == (bf16_out ? torch::kBFloat16 : torch::kFloat32),
              "C dtype does not match the store mode");
  TORCH_CHECK(C.stride(-1) == 1, "C must be contiguous along its last axis");
  const int z = static_cast<int>(a.batch);
  TORCH_CHECK(b.batch == 1 || b.batch == a.batch, "B batch must be 1 or equal A's");
  bw::GemmParams p{};
  p.M = static_cast<int>(a.rows);
  p.N = static_cast<int>(b.rows);
  p.K = static_cast<int>(a.cols);
  p.batch = z;
  p.splits = static_cast<int>(std::max<int64_t>(1, splits));
  p.b_shared = b.batch == 1 ? 1 : 0;
  p.c_mode = static_cast<int>(mode);
  p.beta_accumulate = accumulate ? 1 : 0;
  p.alpha = static_cast<float>(alpha);
  p.C = C.data_ptr();
  p.ldc = C.dim() >= 2 ? C.stride(-2) : 0;
  p.batch_stride_c = (C.dim() == 3) ? C.stride(0) : 0;
  if (mode == bw::kSqAccF32) {
    TORCH_CHECK(C.dim() == 2 && p.splits == 1, "the squared-sum store takes one (M, N) matrix and no split-K");
  } else if (z > 1) {
    TORCH_CHECK(C.dim() == 3 && C.size(0) == z, "C must be (Z, ., .) for batched A");
  }
  if (mode == bw::kStoreBF16T) {
    TORCH_CHECK(C.size(-2) == p.N && C.size(-1) == p.M, "C^T must be (N, M)");
  } else {
    TORCH_CHECK(C.size(-2) == p.M && C.size(-1) == p.N, "C must be (M, N)");
  }
  TORCH_CHECK(p.splits == 1 || mode == bw::kAtomicF32, "split-K needs the atomic fp32 store");
  p.err = err.data_ptr<int>();
  if (p.M == 0 || p.N == 0) return;
  bw::gemm_tn_launch(a, b, p, bw::pick_bn(p.N), at::cuda::getCurrentCUDAStream());
}

// C (bf16) = alpha * A @ B^T stored per segment: C is (S, N, T) with S * T = M rows of A.
void gemm_tn_seg(Tensor A, Tensor B, Tensor C, double alpha, int64_t seg, Tensor err) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  auto b = operand(B, "B");
  TORCH_CHECK(a.batch == 1 && b.batch == 1, "gemm_tn_seg takes 2-D operands");
  TORCH_CHECK(a.cols == b.cols, "A and B disagree on K");
  TORCH_CHECK(seg > 0 && a.rows % seg == 0, "rows of A must be a multiple of the segment length");
  TORCH_CHECK(C.scalar_type() == torch::kBFloat16 && C.is_contiguous() && C.dim() == 3 &&
                  C.size(0) == a.rows / seg && C.size(1) == b.rows && C.size(2) == seg,
              "C must be a contiguous (M / seg, N, seg) bf16 tensor");
  bw::GemmParams p{};
  p.M = (int)a.rows;
  p.N = (int)b.rows;
  p.K = (int)a.cols;
  p.batch = 1;
  p.splits = 1;
  p.b_shared = 1;
  p.c_mode = bw::kStoreBF16TB;
  p.alpha = (float)alpha;
  p.C = C.data_ptr();
  p.ldc = seg;
  p.batch_stride_c = 0;
  p.err = err.data_ptr<int>();
  if (p.M == 0 || p.N == 0) return;
  bw::gemm_tn_launch(a, b, p, bw::pick_bn(p.N), at::cuda::getCurrentCUDAStream());
}

// C (bf16, M x N_main) = A @ B^T and C2 (bf16, token-major (M / seg, N_tail, seg)) =
// A @ Btail^T in ONE CTA-pair launch over A: a layer's output and its projected input (or,
// in the backward, its input gradient and projected output gradient) from one read of A.
void gemm_tn_tail(Tensor A, Tensor B, Tensor Btail, Tensor C, Tensor C2, int64_t seg, Tensor err) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  auto b = operand(B, "B");
  auto t = operand(Btail, "Btail");
  TORCH_CHECK(a.batch == 1 && b.batch == 1 && t.batch == 1, "gemm_tn_tail takes 2-D operands");
  TORCH_CHECK(a.cols == b.cols && a.cols == t.cols, "A, B and Btail disagree on K");
  TORCH_CHECK(b.rows % 256 == 0, "B's rows (the main output width) must be a multiple of 256");
  TORCH_CHECK(t.rows >= 1 && t.rows <= 256, "Btail must have 1..256 rows");
  TORCH_CHECK(seg > 0 && a.rows % seg == 0, "rows of A must be a multiple of the segment length");
  check_cuda(C, "C");
  check_cuda(C2, "C2");
  TORCH_CHECK(C.scalar_type() == torch::kBFloat16 && C.dim() == 2 && C.size(0) == a.rows && C.size(1) == b.rows &&
                  C.stride(1) == 1,
              "C must be a (M, N_main) bf16 matrix, contiguous along its rows");
  TORCH_CHECK(C2.scalar_type() == torch::kBFloat16 && C2.is_contiguous() && C2.dim() == 3 &&
                  C2.size(0) == a.rows / seg && C2.size(1) == t.rows && C2.size(2) == seg,
              "C2 must be a contiguous (M / seg, N_tail, seg) bf16 tensor");
  bw::GemmParams p{};
  p.M = (int)a.rows;
  p.N = (int)(b.rows + t.rows);
  p.K = (int)a.cols;
  p.alpha = 1.0f;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.n_main = (int)b.rows;
  p.C2 = C2.data_ptr();
  p.seg2 = seg;
  p.err = err.data_ptr<int>();
  if (p.M == 0) return;
  TORCH_CHECK(bw::gemm_tn_tail_launch(a, b, t, p, at::cuda::getCurrentCUDAStream()),
              "gemm_tn_tail: CTA pairs cannot run on this device");
}

// bf16x3 split operand of a 2-D fp32 matrix (any strides): (R, 3 Kp) bf16, Kp = K rounded up to 8.
Tensor split3_bf16(Tensor x, int64_t pattern) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.dim() == 2, "x: 2-D fp32");
  TORCH_CHECK(pattern == 0 || pattern == 1, "pattern 0 ([hi|hi|lo]) or 1 ([hi|lo|hi])");
  const long long R = x.size(0), K = x.size(1), Kp = (K + 7) / 8 * 8;
  Tensor out = torch::empty({R, 3 * Kp}, x.options().dtype(torch::kBFloat16));
  bw::split3_bf16(x.data_ptr<float>(), x.stride(0), x.stride(1), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                  (int)R, (int)K, (int)Kp, (int)pattern, at::cuda::getCurrentCUDAStream());
  return out;
}

// Transpose of the last two axes of a bf16 tensor ((..., R, C) -> (..., C, R), contiguous).
Tensor transpose_last2(Tensor x) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && x.dim() >= 2, "x: bf16 with at least two axes");
  Tensor xc = x.stride(-1) == 1 && x.stride(-2) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                      (x.dim() == 2 || x.is_contiguous())
                  ? x
                  : x.contiguous();
  const long long R = xc.size(-2), C = xc.size(-1);
  std::vector<int64_t> shape(xc.sizes().begin(), xc.sizes().end());
  std::swap(shape[shape.size() - 1], shape[shape.size() - 2]);
  Tensor out = torch::empty(shape, xc.options());
  const long long batch = R * C == 0 ? 0 : xc.numel() / (R * C);
  TORCH_CHECK(R < (1LL << 31) && C < (1LL << 31) && batch < 65536, "transpose_last2: extent too large");
  const bool vec_ok = (C % 8 == 0) && (R % 8 == 0);
  if (!vec_ok) return xc.transpose(-1, -2).contiguous();
  bw::transpose_bf16(reinterpret_cast<const __nv_bfloat16*>(xc.data_ptr()), xc.stride(-2),
                     reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), R, (int)batch, (int)R, (int)C,
                     at::cuda::getCurrentCUDAStream());
  return out;
}

// C (fp32, M x M) += alpha * At @ At^T: a covariance / Gram accumulation over the rows' K
// samples (At is M x K, K-major), upper-triangle tiles mirrored, split-K atomic epilogue.
void gram_acc(Tensor At, Tensor C, double alpha, Tensor err) {
  const c10::cuda::CUDAGuard guard(At.device());
  check_err(err);
  auto a = operand(At, "At");
  TORCH_CHECK(a.batch == 1, "gram_acc takes a 2-D operand");
  check_cuda(C, "C");
  TORCH_CHECK(C.scalar_type() == torch::kFloat32 && C.dim() == 2 && C.size(0) == a.rows && C.size(1) == a.rows &&
                  C.stride(1) == 1,
              "C must be a (M, M) fp32 matrix, contiguous along its rows");
  bw::GemmParams p{};
  p.M = p.N = (int)a.rows;
  p.K = (int)a.cols;
  p.alpha = (float)alpha;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.err = err.data_ptr<int>();
  if (p.M == 0 || p.K == 0) return;
  bw::gram_acc_launch(a, p, at::cuda::getCurrentCUDAStream());
}

// ---- grouped GEMM: one launch for many same-shaped batched problems --------------------
struct MapKey {
  const void* ptr;
  long long rows, cols, row_stride, batch, batch_stride;
  int box;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && row_stride == o.row_stride &&
           batch == o.batch && batch_stride == o.batch_stride && box == o.box;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<const void*>()(k.ptr);
    for (long long v : {k.rows, k.cols, k.row_stride, k.batch, k.batch_stride, (long long)k.box})
      h = h * 1000003u ^ std::hash<long long>()(v);
    return h;
  }
};

// Per-device job-table state: encoded maps, the device table, a pinned staging buffer.
struct GroupState {
  std::unordered_map<MapKey, CUtensorMap, MapKeyHash> maps;
  std::vector<uint8_t> last;
  Tensor dev;
  uint8_t* host = nullptr;
  size_t host_cap = 0;
  cudaEvent_t copied = nullptr;
  std::vector<Tensor> graph_tables;  // tables captured into CUDA graphs (kept for their replays)
  uint8_t* graph_arena = nullptr;    // pinned copy sources of captured tables (never rewritten)
  size_t graph_arena_used = 0;
};
constexpr size_t kGraphArena = 8u << 20;
std::mutex g_group_mutex;
std::unordered_map<int, GroupState> g_group;

const CUtensorMap& cached_map(GroupState& st, const bw::GemmOperand& op, int box) {
  MapKey k{op.ptr, op.rows, op.cols, op.row_stride, op.batch, op.batch_stride, box};
  auto it = st.maps.find(k);
  if (it != st.maps.end()) return it->second;
  if (st.maps.size() > 8192) st.maps.clear();
  return st.maps.emplace(k, bw::make_tmap_kmajor_bf16(op, box)).first->second;
}

// For every job i: C_i (op)= alpha * A_i @ B_i^T (batched over the leading axis; B_i may be
// shared by the batch).  All jobs share M, N, K, batch and the store mode.  The job table is
// re-uploaded (stream-ordered, same stream as the launch) only when it changed.
void gemm_grouped(std::vector<Tensor> As, std::vector<Tensor> Bs, std::vector<Tensor> Cs, int64_t mode,
                  double alpha, Tensor err) {
  TORCH_CHECK(!As.empty() && As.size() == Bs.size() && As.size() == Cs.size(), "one A, B and C per job");
  const c10::cuda::CUDAGuard guard(As[0].device());
  check_err(err);
  TORCH_CHECK(mode == bw::kStoreF32 || mode == bw::kStoreBF16, "grouped GEMM stores fp32 or bf16");
  const int n = (int)As.size();
  auto a0 = operand(As[0], "A");
  auto b0 = operand(Bs[0], "B");
  TORCH_CHECK(a0.cols == b0.cols, "A and B disagree on K");
  TORCH_CHECK(b0.batch == 1 || b0.batch == a0.batch, "B batch must be 1 or equal A's");
  const auto cdt = mode == bw::kStoreBF16 ? torch::kBFloat16 : torch::kFloat32;
  bw::GemmParams p{};
  p.M = (int)a0.rows;
  p.N = (int)b0.rows;
  p.K = (int)a0.cols;
  p.batch = (int)a0.batch;
  p.splits = 1;
  p.b_shared = b0.batch == 1 ? 1 : 0;
  p.c_mode = (int)mode;
  p.alpha = (float)alpha;
  p.ldc = Cs[0].stride(-2);
  p.batch_stride_c = Cs[0].dim() == 3 ? Cs[0].stride(0) : 0;
  p.err = err.data_ptr<int>();
  const int bn = bw::pick_bn(p.N);
  const int dev_idx = As[0].get_device();
  std::lock_guard<std::mutex> lock(g_group_mutex);
  GroupState& st = g_group[dev_idx];
  // table: n jobs (32 B each), padded to 128 B, then 2n maps (128 B each)
  const size_t jobs_bytes = ((size_t)n * sizeof(bw::GroupJob) + 127) / 128 * 128;
  const size_t bytes = jobs_bytes + (size_t)2 * n * sizeof(CUtensorMap);
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  C10_CUDA_CHECK(cudaStreamIsCapturing(at::cuda::getCurrentCUDAStream(), &capturing));
  if (capturing == cudaStreamCaptureStatusNone && (!st.dev.defined() || (size_t)st.dev.numel() < bytes)) {
    st.dev = torch::empty({(long long)(bytes * 2)}, As[0].options().dtype(torch::kUInt8));
    st.last.clear();
  }
  uint8_t* dbase = st.dev.defined() ? st.dev.data_ptr<uint8_t>() : nullptr;
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dbase) % 128 == 0, "job table must be 128-byte aligned");
  std::vector<uint8_t> table(bytes, 0);
  auto* jobs = reinterpret_cast<bw::GroupJob*>(table.data());
  auto* maps = reinterpret_cast<CUtensorMap*>(table.data() + jobs_bytes);
  for (int i = 0; i < n; ++i) {
    auto a = operand(As[i], "A");
    auto b = operand(Bs[i], "B");
    TORCH_CHECK(a.rows == a0.rows && a.cols == a0.cols && a.batch == a0.batch && b.rows == b0.rows &&
                    b.cols == b0.cols && b.batch == b0.batch, "grouped jobs must share their shapes");
    TORCH_CHECK(As[i].get_device() == dev_idx && Bs[i].get_device() == dev_idx && Cs[i].get_device() == dev_idx,
                "grouped jobs must be on one device");
    const Tensor& C = Cs[i];
    TORCH_CHECK(C.scalar_type() == cdt && C.stride(-1) == 1 && C.size(-2) == p.M && C.size(-1) == p.N &&
                    C.stride(-2) == p.ldc && (C.dim() == 3 ? C.stride(0) : 0) == p.batch_stride_c &&
                    (p.batch == 1 || (C.dim() == 3 && C.size(0) == p.batch)),
                "every C must be (batch, M, N) with the same strides and the store mode's dtype");
    maps[2 * i] = cached_map(st, a, 128);
    maps[2 * i + 1] = cached_map(st, b, bn);
    jobs[i].ta = reinterpret_cast<const CUtensorMap*>(dbase + jobs_bytes + (size_t)(2 * i) * sizeof(CUtensorMap));
    jobs[i].tb = reinterpret_cast<const CUtensorMap*>(dbase + jobs_bytes + (size_t)(2 * i + 1) * sizeof(CUtensorMap));
    jobs[i].C = C.data_ptr();
    jobs[i].pad = 0;
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  if (capturing != cudaStreamCaptureStatusNone) {
    // Inside a CUDA-graph capture: the graph gets its own table (device memory from the
    // graph's pool, kept alive with the graph's lifetime by this process) uploaded by a
    // captured copy from a pinned host buffer that is never rewritten.
    Tensor dev = torch::empty({(long long)bytes}, As[0].options().dtype(torch::kUInt8));
    uint8_t* gbase = dev.data_ptr<uint8_t>();
    for (int i = 0; i < n; ++i) {
      jobs[i].ta = reinterpret_cast<const CUtensorMap*>(gbase + jobs_bytes + (size_t)(2 * i) * sizeof(CUtensorMap));
      jobs[i].tb = reinterpret_cast<const CUtensorMap*>(gbase + jobs_bytes + (size_t)(2 * i + 1) * sizeof(CUtensorMap));
    }
    // Pinned memory cannot be allocated while a stream captures: carve the graph's copy
    // source from the pinned arena reserved by an earlier (eager) call on this device.
    TORCH_CHECK(st.graph_arena != nullptr && st.graph_arena_used + bytes <= kGraphArena,
                "gemm_grouped: make one eager call on this device before capturing a CUDA graph "
                "(its pinned staging arena is reserved outside capture)");
    uint8_t* host = st.graph_arena + st.graph_arena_used;
    st.graph_arena_used += (bytes + 127) / 128 * 128;
    std::memcpy(host, table.data(), bytes);
    C10_CUDA_CHECK(cudaMemcpyAsync(gbase, host, bytes, cudaMemcpyHostToDevice, stream));
    st.graph_tables.push_back(dev);
    if (p.M == 0 || p.N == 0) return;
    bw::gemm_grouped_launch(reinterpret_cast<const bw::GroupJob*>(gbase), n, p, bn, stream);
    return;
  }
  if (st.graph_arena == nullptr)
    C10_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&st.graph_arena), kGraphArena, cudaHostAllocDefault));
  if (st.last != table) {
    if (st.copied == nullptr) C10_CUDA_CHECK(cudaEventCreateWithFlags(&st.copied, cudaEventDisableTiming));
    else C10_CUDA_CHECK(cudaEventSynchronize(st.copied));  // the staging buffer is free again
    if (st.host_cap < bytes) {
      if (st.host != nullptr) C10_CUDA_CHECK(cudaFreeHost(st.host));
      C10_CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&st.host), bytes * 2, cudaHostAllocDefault));
      st.host_cap = bytes * 2;
    }
    std::memcpy(st.host, table.data(), bytes);
    C10_CUDA_CHECK(cudaMemcpyAsync(dbase, st.host, bytes, cudaMemcpyHostToDevice, stream));
    C10_CUDA_CHECK(cudaEventRecord(st.copied, stream));
    st.last.swap(table);
  }
  if (p.M == 0 || p.N == 0) return;
  bw::gemm_grouped_launch(reinterpret_cast<const bw::GroupJob*>(dbase), n, p, bn, stream);
}

// ---- fused all-gather + score GEMM ------------------------------------------------------
// Device copies of the peers' tensor maps, keyed by the peers' buffer addresses (symmetric
// buffers are allocated once, so each distinct table is encoded and uploaded once).
struct PeerTables {
  std::mutex mu;
  std::unordered_map<std::string, Tensor> tables;
};
PeerTables g_peer_tables;

// out (M, world * R) += alpha * test @ [X_0; ...; X_{world-1}]^T, where X_r = peers[r] is rank
// r's (R, K) bf16 block read over NVLink (peer-mapped symmetric memory).  out is fp32 and
// accumulated (the caller zeroes it).
void ag_score(Tensor test, std::vector<Tensor> peers, Tensor out, double alpha, int64_t splits, Tensor err) {
  const c10::cuda::CUDAGuard guard(test.device());
  check_err(err);
  auto t = operand(test, "test");
  TORCH_CHECK(t.batch == 1, "test must be 2-D");
  TORCH_CHECK(!peers.empty(), "at least one peer block");
  const int world = (int)peers.size();
  std::string key;
  std::vector<bw::GemmOperand> ops;
  for (int r = 0; r < world; ++r) {
    auto o = operand(peers[r], "peer block");
    TORCH_CHECK(o.batch == 1 && o.cols == t.cols, "peer blocks must be (R, K) with the test's K");
    TORCH_CHECK(o.rows == operand(peers[0], "peer block").rows, "peer blocks must have one row count");
    TORCH_CHECK(o.rows % 8 == 0, "peer blocks need a multiple of 8 rows");
    ops.push_back(o);
    key += std::to_string(reinterpret_cast<uintptr_t>(o.ptr)) + ":" + std::to_string(o.rows) + ":" +
           std::to_string(o.cols) + ":" + std::to_string(o.row_stride) + ";";
  }
  const int R = (int)ops[0].rows;
  TORCH_CHECK(bw::ag_score_tile_n(world * R) > 0, "world * rows per peer must be <= 128");
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.dim() == 2 && out.stride(1) == 1 &&
                  out.size(0) == t.rows && out.size(1) == (long long)world * R,
              "out must be (M, world * R) fp32 with contiguous rows");
  Tensor table;
  {
    std::lock_guard<std::mutex> lock(g_peer_tables.mu);
    key += "dev" + std::to_string(test.get_device());
    auto it = g_peer_tables.tables.find(key);
    if (it == g_peer_tables.tables.end()) {
      std::vector<CUtensorMap> maps;
      for (auto& o : ops) maps.push_back(bw::make_tmap_kmajor_bf16(o, R));
      auto host = torch::empty({(long long)(maps.size() * sizeof(CUtensorMap))}, torch::kUInt8);
      std::memcpy(host.data_ptr(), maps.data(), maps.size() * sizeof(CUtensorMap));
      table = host.to(test.device());  // synchronous upload, once per distinct table
      TORCH_CHECK(reinterpret_cast<uintptr_t>(table.data_ptr()) % 64 == 0, "tensor-map table must be 64-byte aligned");
      g_peer_tables.tables.emplace(key, table);
    } else {
      table = it->second;
    }
  }
  const int kblocks = (int)((t.cols + 63) / 64);
  int sp = (int)std::max<int64_t>(1, std::min<int64_t>(splits, kblocks));
  const int per = (kblocks + sp - 1) / sp;
  sp = (kblocks + per - 1) / per;  // every split owns at least one K block
  bw::AgScoreParams p{};
  p.M = (int)t.rows;
  p.K = (int)t.cols;
  p.world = world;
  p.rows_per_peer = R;
  p.splits = sp;
  p.alpha = (float)alpha;
  p.out = out.data_ptr<float>();
  p.ldo = out.stride(0);
  p.err = err.data_ptr<int>();
  if (p.M == 0) return;
  const CUtensorMap tmT = bw::make_tmap_kmajor_bf16(t, 128);
  bw::ag_score_launch(tmT, reinterpret_cast<const CUtensorMap*>(table.data_ptr()), p,
                      at::cuda::getCurrentCUDAStream());
}

// Cross-GPU barrier: flag_ptrs is a device int64 tensor of the ranks' flag-array addresses.
void peer_barrier(Tensor flag_ptrs, int64_t rank, int64_t world, int64_t epoch, Tensor err) {
  const c10::cuda::CUDAGuard guard(flag_ptrs.device());
  check_err(err);
  TORCH_CHECK(flag_ptrs.is_cuda() && flag_ptrs.scalar_type() == torch::kInt64 && flag_ptrs.numel() == world,
              "flag_ptrs must be a CUDA int64 tensor with one address per rank");
  TORCH_CHECK(world >= 1 && world <= 1024 && rank >= 0 && rank < world, "bad rank / world");
  bw::peer_barrier(reinterpret_cast<int* const*>(flag_ptrs.data_ptr<int64_t>()), (int)rank, (int)world,
                   (int)epoch, err.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

// GEMM -> reduce-scatter in one launch: every element of alpha * A @ B^T is stored (16-byte
// peer stores) into its owner rank's slot for this rank; owner = float4 index / per4.
// slot_ptrs[r] is rank r's slot buffer (world * 4 * per4 fp32) as mapped here.  The owners
// sum their slots with `slot_reduce` after a cross-GPU barrier.
void gemm_tn_rs(Tensor A, Tensor B, Tensor slot_ptrs, int64_t world, int64_t per4, int64_t M, int64_t N,
                int64_t ldc, double alpha, Tensor err, int64_t self_rank) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  auto b = operand(B, "B");
  TORCH_CHECK(a.batch == 1 && b.batch == 1 && a.cols == b.cols, "2-D operands with one K");
  TORCH_CHECK(a.rows == M && b.rows == N, "M / N disagree with the operands");
  TORCH_CHECK(slot_ptrs.is_cuda() && slot_ptrs.scalar_type() == torch::kInt64 && slot_ptrs.numel() == world,
              "slot_ptrs: one device address per rank");
  TORCH_CHECK(per4 > 0 && world >= 1 && self_rank >= 0 && self_rank < world, "bad partition");
  TORCH_CHECK((M - 1) * ldc + N <= 4 * per4 * world, "the partition does not cover C");
  bw::GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)a.cols;
  p.batch = 1;
  p.splits = 1;  // one writer per element and rank: plain stores, no atomics
  p.b_shared = 1;
  p.c_mode = bw::kPeerSlotF32;
  p.alpha = (float)alpha;
  p.ldc = ldc;
  p.peers = reinterpret_cast<float* const*>(slot_ptrs.data_ptr<int64_t>());
  p.world = (int)world;
  p.per4 = per4;
  p.self_rank = (int)self_rank;
  p.err = err.data_ptr<int>();
  if (M == 0 || N == 0) return;
  bw::gemm_tn_launch(a, b, p, bw::pick_bn(p.N), at::cuda::getCurrentCUDAStream());
}

// out[0, n) (+)= sum over the world slots of this rank's slot buffer.
void slot_reduce(Tensor slots, int64_t world, int64_t slot, Tensor out, int64_t n, bool accumulate) {
  const c10::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == torch::kFloat32 && slots.is_contiguous() &&
                  slots.numel() >= world * slot, "slots: contiguous fp32 (world * slot)");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.numel() >= n,
              "out: contiguous fp32");
  TORCH_CHECK(slot % 4 == 0 && n % 4 == 0 && n <= slot, "slot and n: multiples of 4 floats, n <= slot");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(slots.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "16-byte aligned buffers");
  bw::slot_reduce(slots.data_ptr<float>(), (int)world, slot, out.data_ptr<float>(), n, accumulate,
                  at::cuda::getCurrentCUDAStream());
}

// C (op)= alpha * A @ B^T where B lives sharded on the peers (read over NVLink inside the
// GEMM).  mode 0: peers[r] is (shard, K), B = [peers[0]; peers[1]; ...] by rows;
// mode 1: peers[r] is (N, shard), B = [peers[0] | peers[1] | ...] along K.
void gemm_tn_peers(Tensor A, std::vector<Tensor> peers, Tensor C, int64_t mode, int64_t store, double alpha,
                   Tensor err) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  TORCH_CHECK(a.batch == 1, "A must be 2-D");
  const int world = (int)peers.size();
  TORCH_CHECK(world >= 1 && world <= bw::kMaxPeerMaps, "1..8 peers");
  TORCH_CHECK(mode == 0 || mode == 1, "mode must be 0 (row shards) or 1 (K shards)");
  TORCH_CHECK(store == bw::kStoreF32 || store == bw::kStoreBF16, "store must be fp32 or bf16");
  std::vector<bw::GemmOperand> ops;
  for (auto& t : peers) ops.push_back(operand(t, "peer shard"));
  for (auto& o : ops)
    TORCH_CHECK(o.batch == 1 && o.rows == ops[0].rows && o.cols == ops[0].cols, "peer shards must match");
  const int shard = mode == 0 ? (int)ops[0].rows : (int)ops[0].cols;
  const int n_out = mode == 0 ? shard * world : (int)ops[0].rows;
  const long long k = mode == 0 ? ops[0].cols : (long long)shard * world;
  TORCH_CHECK(a.cols == k, "A's K does not match the sharded B");
  int bn = bw::pick_bn(n_out);
  if (mode == 0) {
    while (bn > 16 && shard % bn != 0) bn /= 2;  // a CTA's rows must come from one owner
  }
  if (mode == 0) {
    TORCH_CHECK(shard % bn == 0, "row shards must be a multiple of the ", bn, "-row tile");
  } else {
    TORCH_CHECK(shard % 64 == 0, "K shards must be a multiple of 64");
  }
  const bool bf16_out = store == bw::kStoreBF16;
  TORCH_CHECK(C.is_cuda() && C.scalar_type() == (bf16_out ? torch::kBFloat16 : torch::kFloat32) && C.dim() == 2 &&
                  C.size(0) == a.rows && C.size(1) == n_out && C.stride(1) == 1,
              "C must be (M, N) with contiguous rows and the store's dtype");
  Tensor table;
  {
    std::string key = "peers:" + std::to_string(bn) + ":" + std::to_string(A.get_device()) + ";";
    for (auto& o : ops)
      key += std::to_string(reinterpret_cast<uintptr_t>(o.ptr)) + ":" + std::to_string(o.rows) + ":" +
             std::to_string(o.cols) + ":" + std::to_string(o.row_stride) + ";";
    std::lock_guard<std::mutex> lock(g_peer_tables.mu);
    auto it = g_peer_tables.tables.find(key);
    if (it == g_peer_tables.tables.end()) {
      std::vector<CUtensorMap> maps;
      for (auto& o : ops) maps.push_back(bw::make_tmap_kmajor_bf16(o, bn));
      auto host = torch::empty({(long long)(maps.size() * sizeof(CUtensorMap))}, torch::kUInt8);
      std::memcpy(host.data_ptr(), maps.data(), maps.size() * sizeof(CUtensorMap));
      table = host.to(A.device());  // synchronous upload, once per distinct set of shards
      TORCH_CHECK(reinterpret_cast<uintptr_t>(table.data_ptr()) % 64 == 0, "tensor-map table must be 64-byte aligned");
      g_peer_tables.tables.emplace(key, table);
    } else {
      table = it->second;
    }
  }
  bw::GemmParams p{};
  p.M = (int)a.rows;
  p.N = n_out;
  p.K = (int)k;
  p.batch = 1;
  p.splits = 1;
  p.b_shared = 1;
  p.c_mode = (int)store;
  p.alpha = (float)alpha;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.err = err.data_ptr<int>();
  if (p.M == 0 || p.N == 0) return;
  bw::gemm_peers_launch(a, reinterpret_cast<const CUtensorMap*>(table.data_ptr()), p, (int)mode, shard, bn,
                        at::cuda::getCurrentCUDAStream());
}

// C (op)= alpha * A @ B^T with B sharded over the peers, all-gathered INSIDE the launch into
// the local staging matrix `stage` (each remote byte crosses NVLink once) while the GEMM
// tiles consume it.  mode 0: peers[r] is (shard, K) and B = rows; mode 1: peers[r] is
// (N, shard) and B = K columns.  `flags` (int32, one per rank, zeroed once) and `epoch`
// (1, 2, ... per launch on this staging buffer) gate the tiles.
void gemm_tn_staged(Tensor A, std::vector<Tensor> peers, Tensor stage, Tensor C, Tensor flags, int64_t epoch,
                    int64_t mode, int64_t self_rank, int64_t store, double alpha, Tensor err) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  TORCH_CHECK(a.batch == 1, "A must be 2-D");
  const int world = (int)peers.size();
  TORCH_CHECK(world >= 1 && world <= bw::kMaxPeerMaps, "1..8 peers");
  TORCH_CHECK(mode == 0 || mode == 1, "mode must be 0 (row shards) or 1 (K shards)");
  TORCH_CHECK(self_rank >= 0 && self_rank < world, "bad self rank");
  TORCH_CHECK(store == bw::kStoreF32 || store == bw::kStoreBF16, "store must be fp32 or bf16");
  std::vector<bw::GemmOperand> ops;
  for (auto& t : peers) ops.push_back(operand(t, "peer shard"));
  for (auto& o : ops)
    TORCH_CHECK(o.batch == 1 && o.rows == ops[0].rows && o.cols == ops[0].cols && o.row_stride == ops[0].row_stride,
                "peer shards must match");
  auto st = operand(stage, "stage");
  const int shard = mode == 0 ? (int)ops[0].rows : (int)ops[0].cols;
  const int n_out = mode == 0 ? shard * world : (int)ops[0].rows;
  const long long k = mode == 0 ? ops[0].cols : (long long)shard * world;
  TORCH_CHECK(st.batch == 1 && st.rows == n_out && st.cols == k, "stage must be the gathered (N, K) matrix");
  TORCH_CHECK(a.cols == k, "A's K does not match the sharded B");
  int bn = bw::pick_bn(n_out);
  if (mode == 0) {
    while (bn > 64 && shard % bn != 0) bn /= 2;
    TORCH_CHECK(shard % bn == 0 && bn >= 64, "row shards must be a multiple of 64 rows");
  } else {
    if (bn < 64) bn = 64;
    TORCH_CHECK(shard % 64 == 0, "K shards must be a multiple of 64");
  }
  TORCH_CHECK(flags.is_cuda() && flags.scalar_type() == torch::kInt32 && flags.numel() >= world, "flags: int32[world]");
  const bool bf16_out = store == bw::kStoreBF16;
  TORCH_CHECK(C.is_cuda() && C.scalar_type() == (bf16_out ? torch::kBFloat16 : torch::kFloat32) && C.dim() == 2 &&
                  C.size(0) == a.rows && C.size(1) == n_out && C.stride(1) == 1,
              "C must be (M, N) with contiguous rows and the store's dtype");
  bw::StageArgs sa{};
  const int src_rows = (int)ops[0].rows;
  const long long row_elems = ops[0].cols;
  TORCH_CHECK(row_elems % 8 == 0 && ops[0].row_stride % 8 == 0 && st.row_stride % 8 == 0, "rows must be 16-byte multiples");
  for (int r = 0; r < world; ++r) {
    sa.src[r] = ops[r].ptr;
    sa.dst_row0[r] = mode == 0 ? (long long)r * shard : 0;
    sa.dst_col0[r] = mode == 0 ? 0 : (long long)r * shard;
  }
  sa.src_stride = ops[0].row_stride;
  sa.src_rows = src_rows;
  sa.row_elems = row_elems;
  sa.dst = const_cast<void*>(st.ptr);
  sa.dst_stride = st.row_stride;
  int pieces = (2 * 148 + world - 1) / world;
  if (pieces > src_rows / 8) pieces = std::max(1, src_rows / 8);
  sa.piece_rows = (src_rows + pieces - 1) / pieces;
  sa.pieces_per_owner = (src_rows + sa.piece_rows - 1) / sa.piece_rows;
  sa.flags = flags.data_ptr<int>();
  sa.expect = (int)(epoch * sa.pieces_per_owner);
  sa.world = world;
  sa.self = (int)self_rank;
  sa.mode = (int)mode;
  sa.shard = shard;
  bw::GemmParams p{};
  p.M = (int)a.rows;
  p.N = n_out;
  p.K = (int)k;
  p.batch = 1;
  p.splits = 1;
  p.b_shared = 1;
  p.c_mode = (int)store;
  p.alpha = (float)alpha;
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.err = err.data_ptr<int>();
  if (p.M == 0 || p.N == 0) return;
  bw::gemm_staged_launch(a, st, ops[self_rank], p, sa, bn, at::cuda::getCurrentCUDAStream());
}

// A device array of the given tensors' addresses, cached by the address list (symmetric
// buffers are allocated once).
Tensor device_ptr_table(const std::vector<Tensor>& ts, const c10::Device& dev) {
  std::string key = "ptrs:" + std::to_string(dev.index()) + ";";
  for (auto& t : ts) key += std::to_string(reinterpret_cast<uintptr_t>(t.data_ptr())) + ";";
  std::lock_guard<std::mutex> lock(g_peer_tables.mu);
  auto it = g_peer_tables.tables.find(key);
  if (it != g_peer_tables.tables.end()) return it->second;
  auto host = torch::empty({(long long)ts.size()}, torch::kInt64);
  for (size_t i = 0; i < ts.size(); ++i) host[i] = (int64_t) reinterpret_cast<uintptr_t>(ts[i].data_ptr());
  Tensor table = host.to(dev);
  g_peer_tables.tables.emplace(key, table);
  return table;
}

// Expert-parallel dispatch: row r of src (token r / k) into rank dst_rank[r]'s receive
// buffer at row dst_row[r], with its origin (self, r) into that rank's origin table.
void moe_dispatch(Tensor src, int64_t rows_per_token, Tensor dst_rank, Tensor dst_row, std::vector<Tensor> peer_rows,
                  std::vector<Tensor> peer_meta, int64_t self) {
  const c10::cuda::CUDAGuard guard(src.device());
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kBFloat16 && src.dim() == 2 && src.stride(1) == 1 &&
                  src.stride(0) % 8 == 0 && src.size(1) % 8 == 0, "src must be (T, H) bf16 with 16-byte rows");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(src.data_ptr()) % 16 == 0, "src must be 16-byte aligned");
  const int world = (int)peer_rows.size();
  TORCH_CHECK(world >= 1 && world <= 8 && (peer_meta.empty() || (int)peer_meta.size() == world),
              "1..8 ranks, one origin table per rank or none");
  const long long rows = src.size(0) * rows_per_token;
  TORCH_CHECK(dst_rank.scalar_type() == torch::kInt32 && dst_row.scalar_type() == torch::kInt32 &&
                  dst_rank.numel() == rows && dst_row.numel() == rows && dst_rank.is_contiguous() && dst_row.is_contiguous(),
              "dst_rank / dst_row: int32 per (token, slot)");
  std::vector<void*> pr;
  std::vector<int2*> pm;
  for (int r = 0; r < world; ++r) {
    TORCH_CHECK(peer_rows[r].scalar_type() == torch::kBFloat16 && peer_rows[r].size(-1) == src.size(1) &&
                    peer_rows[r].is_contiguous(), "receive buffers must be (R, H) bf16");
    pr.push_back(peer_rows[r].data_ptr());
    if (peer_meta.empty()) continue;
    TORCH_CHECK(peer_meta[r].scalar_type() == torch::kInt32 && peer_meta[r].is_contiguous(), "origin tables: int32");
    pm.push_back(reinterpret_cast<int2*>(peer_meta[r].data_ptr<int>()));
  }
  bw::moe_dispatch(src.data_ptr(), src.stride(0), dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(), pr.data(),
                   pm.empty() ? nullptr : pm.data(), world, (int)rows, (int)src.size(1), (int)self, (int)rows_per_token,
                   at::cuda::getCurrentCUDAStream());
}

// Mask projection of factorized gradients: out (B, M) fp32 = sum_t R[b, t, rows] * C[b, t, cols].
void mask_gather(Tensor R, Tensor C, Tensor rows, Tensor cols, Tensor out, Tensor err) {
  const c10::cuda::CUDAGuard guard(R.device());
  check_err(err);
  for (auto* t : {&R, &C})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kBFloat16 && t->is_contiguous() && t->dim() == 3 &&
                    t->size(2) % 8 == 0 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "factors: contiguous 16-byte aligned (B, T, K) bf16 with K % 8 == 0");
  TORCH_CHECK(R.size(0) == C.size(0) && R.size(1) == C.size(1), "factors disagree on (B, T)");
  for (auto* t : {&rows, &cols})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous(), "coordinates: int32 CUDA");
  TORCH_CHECK(rows.numel() == cols.numel(), "one row and one column per coordinate");
  const long long M = rows.numel();
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.dim() == 2 &&
                  out.size(0) == R.size(0) && out.size(1) == M, "out: (B, M) fp32");
  bw::mask_gather(reinterpret_cast<const __nv_bfloat16*>(R.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(C.data_ptr()),
                  rows.data_ptr<int>(), cols.data_ptr<int>(), out.data_ptr<float>(), (int)R.size(0), (int)R.size(1),
                  (int)R.size(2), (int)C.size(2), (int)M, err.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

// MoE routing histogram (int32 counts, accumulated) of int64 expert ids.
void moe_count(Tensor topi, Tensor counts) {
  const c10::cuda::CUDAGuard guard(topi.device());
  TORCH_CHECK(topi.scalar_type() == torch::kInt64 && topi.is_contiguous(), "topi: contiguous int64");
  TORCH_CHECK(counts.scalar_type() == torch::kInt32 && counts.is_contiguous(), "counts: int32");
  bw::moe_count(reinterpret_cast<const long long*>(topi.data_ptr<int64_t>()), (int)topi.numel(),
                counts.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

// MoE receive layout (see moe_ep.cu): fills dest / dst_row per routed row and this rank's
// ragged-GEMM tables (tile_prefix, base, len) and received-row total.
void moe_place(Tensor topi, Tensor all_counts, int64_t rank, int64_t e_l, Tensor cursor, Tensor dest, Tensor dst_row,
               Tensor tile_prefix, Tensor base, Tensor len, Tensor total) {
  const c10::cuda::CUDAGuard guard(topi.device());
  TORCH_CHECK(topi.scalar_type() == torch::kInt64 && topi.is_contiguous(), "topi: contiguous int64");
  TORCH_CHECK(all_counts.scalar_type() == torch::kInt32 && all_counts.is_contiguous() && all_counts.dim() == 2,
              "all_counts: (world, experts) int32");
  const int world = (int)all_counts.size(0);
  TORCH_CHECK(all_counts.size(1) == world * e_l, "experts = world * e_l");
  for (auto* t : {&cursor, &dest, &dst_row, &tile_prefix, &base, &len, &total})
    TORCH_CHECK(t->scalar_type() == torch::kInt32 && t->is_contiguous() && t->is_cuda(), "int32 CUDA tables");
  TORCH_CHECK(cursor.numel() >= world * e_l && dest.numel() == topi.numel() && dst_row.numel() == topi.numel() &&
                  tile_prefix.numel() == e_l + 1 && base.numel() == e_l && len.numel() == e_l && total.numel() >= 1,
              "table sizes");
  bw::moe_place(reinterpret_cast<const long long*>(topi.data_ptr<int64_t>()), (int)topi.numel(),
                all_counts.data_ptr<int>(), world, (int)rank, (int)e_l, cursor.data_ptr<int>(), dest.data_ptr<int>(),
                dst_row.data_ptr<int>(), tile_prefix.data_ptr<int>(), base.data_ptr<int>(), len.data_ptr<int>(),
                total.data_ptr<int>(), at::cuda::getCurrentCUDAStream());
}

// MoE combine: y (T, H) = sum over the k slots of w (T, k) fp32 * slots (T * k, H) bf16.
void moe_combine(Tensor slots, Tensor w, Tensor y) {
  const c10::cuda::CUDAGuard guard(slots.device());
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.dim() == 2, "w: (T, k) fp32");
  const long long T = w.size(0), k = w.size(1);
  TORCH_CHECK(slots.scalar_type() == torch::kBFloat16 && slots.is_contiguous() && slots.dim() == 2 &&
                  slots.size(0) >= T * k && slots.size(1) % 8 == 0, "slots: contiguous (>= T * k, H) bf16");
  TORCH_CHECK(y.scalar_type() == torch::kBFloat16 && y.is_contiguous() && y.size(0) == T &&
                  y.size(1) == slots.size(1), "y: contiguous (T, H) bf16");
  bw::moe_combine(slots.data_ptr(), w.data_ptr<float>(), y.data_ptr(), (int)T, (int)k, (int)slots.size(1),
                  at::cuda::getCurrentCUDAStream());
}

// Backward of moe_combine fused with the dispatch of the slot gradients to the owners.
void moe_combine_bwd_dispatch(Tensor dy, Tensor slots, Tensor w, Tensor dw, Tensor dst_rank, Tensor dst_row,
                              std::vector<Tensor> peer_rows, std::vector<Tensor> peer_meta, int64_t self) {
  const c10::cuda::CUDAGuard guard(dy.device());
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.dim() == 2, "w: (T, k) fp32");
  const long long T = w.size(0), k = w.size(1), rows = T * k;
  TORCH_CHECK(dw.scalar_type() == torch::kFloat32 && dw.is_contiguous() && dw.numel() == rows, "dw: (T, k) fp32");
  TORCH_CHECK(dy.scalar_type() == torch::kBFloat16 && dy.is_contiguous() && dy.size(0) == T && dy.size(1) % 8 == 0,
              "dy: contiguous (T, H) bf16");
  TORCH_CHECK(slots.scalar_type() == torch::kBFloat16 && slots.is_contiguous() && slots.size(0) >= rows &&
                  slots.size(1) == dy.size(1), "slots: contiguous (T * k, H) bf16");
  TORCH_CHECK(dst_rank.scalar_type() == torch::kInt32 && dst_row.scalar_type() == torch::kInt32 &&
                  dst_rank.numel() == rows && dst_row.numel() == rows && dst_rank.is_contiguous() &&
                  dst_row.is_contiguous(), "dst_rank / dst_row: int32 per (token, slot)");
  const int world = (int)peer_rows.size();
  TORCH_CHECK(world >= 1 && world <= 8 && (peer_meta.empty() || (int)peer_meta.size() == world),
              "1..8 ranks, one origin table per rank or none");
  std::vector<void*> pr;
  std::vector<int2*> pm;
  for (int r = 0; r < world; ++r) {
    TORCH_CHECK(peer_rows[r].scalar_type() == torch::kBFloat16 && peer_rows[r].is_contiguous() &&
                    peer_rows[r].size(-1) == dy.size(1), "receive buffers must be (R, H) bf16");
    TORCH_CHECK(peer_meta[r].scalar_type() == torch::kInt32 && peer_meta[r].is_contiguous(), "origin tables: int32");
    pr.push_back(peer_rows[r].data_ptr());
    pm.push_back(reinterpret_cast<int2*>(peer_meta[r].data_ptr<int>()));
  }
  bw::moe_combine_bwd_dispatch(dy.data_ptr(), slots.data_ptr(), w.data_ptr<float>(), dw.data_ptr<float>(),
                               dst_rank.data_ptr<int>(), dst_row.data_ptr<int>(), pr.data(), pm.data(), world, (int)rows,
                               (int)k, (int)dy.size(1), (int)self, at::cuda::getCurrentCUDAStream());
}

// Per-sample LayerNorm / RMSNorm parameter gradients from the raw input x (B, T, d) and the
// output gradient g: returns (B, d) dgamma, or (B, 2d) [dgamma | dbeta] with `bias`.
Tensor norm_per_sample_grad(Tensor x, Tensor g, double eps, bool layer_norm, bool bias) {
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && g.scalar_type() == torch::kBFloat16 &&
                  x.dim() == 3 && x.sizes() == g.sizes() && x.is_contiguous() && g.is_contiguous(),
              "x and g must be contiguous (B, T, d) bf16");
  const int d = (int)x.size(2);
  TORCH_CHECK(d % 8 == 0 && d <= 16384, "d must be a multiple of 8 and <= 16384");
  const int B = (int)x.size(0), T = (int)x.size(1);
  auto out = torch::zeros({B, bias ? 2 * d : d}, x.options().dtype(torch::kFloat32));
  float* dw = out.data_ptr<float>();
  // (B, 2d) rows interleave as [dgamma | dbeta]: write through strided views.
  Tensor wv = bias ? torch::zeros({B, d}, out.options()) : out;
  Tensor bv = bias ? torch::zeros({B, d}, out.options()) : Tensor();
  if (bias) dw = wv.data_ptr<float>();
  bw::norm_per_sample_grad(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
                           reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), dw,
                           bias ? bv.data_ptr<float>() : nullptr, B, T, d, (float)eps, layer_norm,
                           at::cuda::getCurrentCUDAStream());
  if (bias) {
    out.narrow(1, 0, d).copy_(wv);
    out.narrow(1, d, d).copy_(bv);
  }
  return out;
}

// Ragged grouped GEMM of expert layers: rows [base[j], base[j] + len[j]) of A times B3[j]^T;
// output rows stored in C (same row index) or, with `scatter`, returned to their source
// ranks' buffers peer_C.  tile_prefix / base / len are device int32 arrays (tile_prefix counts
// 256-row blocks); max_tiles bounds the number of such blocks (the persistent kernel reads
// the real count on the device).
void gemm_ragged(Tensor A, Tensor B3, c10::optional<Tensor> C, Tensor tile_prefix, Tensor base, Tensor len,
                 int64_t max_tiles, std::vector<Tensor> peer_C, c10::optional<Tensor> scatter, Tensor err,
                 int64_t bn) {
  const c10::cuda::CUDAGuard guard(A.device());
  check_err(err);
  auto a = operand(A, "A");
  auto b = operand(B3, "B3");
  TORCH_CHECK(a.batch == 1 && B3.dim() == 3 && a.cols == b.cols, "A (R, K) and B3 (J, N, K)");
  const int jobs = (int)b.batch;
  for (auto* t : {&tile_prefix, &base, &len})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous(), "job arrays: int32 CUDA");
  TORCH_CHECK(tile_prefix.numel() == jobs + 1 && base.numel() == jobs && len.numel() == jobs, "job array sizes");
  bw::GemmParams p{};
  p.M = (int)a.rows;
  p.N = (int)b.rows;
  p.K = (int)a.cols;
  p.alpha = 1.f;
  p.err = err.data_ptr<int>();
  Tensor ptrs;
  if (scatter.has_value() && scatter->defined()) {
    TORCH_CHECK(scatter->scalar_type() == torch::kInt32 && scatter->is_contiguous() && scatter->numel() >= 2 * a.rows,
                "scatter: int32 (R, 2)");
    for (auto& c : peer_C)
      TORCH_CHECK(c.scalar_type() == torch::kBFloat16 && c.is_contiguous() && c.size(-1) == b.rows &&
                      reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 == 0,
                  "peer outputs must be contiguous 16-byte aligned (R, N) bf16");
    ptrs = device_ptr_table(peer_C, A.device());
    p.c_mode = bw::kStoreBF16Scatter;
    p.peers = reinterpret_cast<float* const*>(ptrs.data_ptr<int64_t>());
    p.world = (int)peer_C.size();
    p.scatter = reinterpret_cast<const int2*>(scatter->data_ptr<int>());
    p.ldc = b.rows;
  } else {
    TORCH_CHECK(C.has_value() && C->defined() && C->scalar_type() == torch::kBFloat16 && C->dim() == 2 &&
                    C->size(0) == a.rows && C->size(1) == b.rows && C->stride(1) == 1, "C must be (R, N) bf16");
    p.c_mode = bw::kStoreBF16;
    p.C = C->data_ptr();
    p.ldc = C->stride(0);
  }
  if (max_tiles <= 0 || p.N == 0) return;
  bw::gemm_ragged_launch(a, b, p, tile_prefix.data_ptr<int>(), base.data_ptr<int>(), len.data_ptr<int>(), jobs,
                         (int)max_tiles, bn > 0 ? (int)bn : std::max(64, bw::pick_bn(p.N)),
                         at::cuda::getCurrentCUDAStream());
}

void swiglu_split(Tensor h, Tensor out, Tensor rows) {
  const c10::cuda::CUDAGuard guard(h.device());
  TORCH_CHECK(h.scalar_type() == torch::kBFloat16 && h.is_contiguous() && h.dim() == 2 && h.size(1) % 16 == 0,
              "h: contiguous (R, 2I) bf16, I % 8 == 0");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.size(0) == h.size(0) &&
                  out.size(1) * 2 == h.size(1), "out: (R, I) bf16");
  TORCH_CHECK(rows.is_cuda() && rows.scalar_type() == torch::kInt32 && rows.numel() >= 1, "rows: int32 CUDA scalar");
  bw::swiglu_split(reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                   rows.data_ptr<int>(), (int)h.size(0), (int)out.size(1),
                   at::cuda::getCurrentCUDAStream());
}

void swiglu_split_bwd(Tensor da, Tensor h, Tensor dh, Tensor rows) {
  const c10::cuda::CUDAGuard guard(h.device());
  TORCH_CHECK(h.scalar_type() == torch::kBFloat16 && h.is_contiguous() && da.is_contiguous() && dh.is_contiguous() &&
                  da.size(1) * 2 == h.size(1) && dh.sizes() == h.sizes() && da.size(1) % 8 == 0,
              "da (R, I), h and dh (R, 2I): contiguous bf16");
  bw::swiglu_split_bwd(reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()),
                       reinterpret_cast<const __nv_bfloat16*>(h.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dh.data_ptr()),
                       rows.data_ptr<int>(), (int)h.size(0), (int)da.size(1),
                       at::cuda::getCurrentCUDAStream());
}

// Peer all-reduce phases over symmetric fp32 buffers (see allreduce_p2p.cu).
std::vector<const float*> peer_floats(const std::vector<Tensor>& peers, long long n) {
  TORCH_CHECK(!peers.empty() && (int)peers.size() <= bw::allreduce_max_peers(), "1..16 peer buffers");
  std::vector<const float*> ptrs;
  for (auto& t : peers) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == torch::kFloat32 && t.is_contiguous() && t.numel() >= n,
                "peer buffers must be contiguous fp32 CUDA tensors holding n elements");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, "peer buffers must be 16-byte aligned");
    ptrs.push_back(t.data_ptr<float>());
  }
  return ptrs;
}

void allreduce_phase(std::vector<Tensor> peers, Tensor out, int64_t n, int64_t phase, int64_t rank) {
  const c10::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(n % 4 == 0, "n must be a multiple of 4");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.numel() >= n &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out must be aligned contiguous fp32");
  auto ptrs = peer_floats(peers, n);
  auto stream = at::cuda::getCurrentCUDAStream();
  const int world = (int)ptrs.size();
  if (phase == 0) bw::allreduce_oneshot(ptrs.data(), world, out.data_ptr<float>(), n, stream);
  else if (phase == 1) bw::allreduce_reduce_scatter(ptrs.data(), world, (int)rank, out.data_ptr<float>(), n, stream);
  else bw::allreduce_all_gather(ptrs.data(), world, out.data_ptr<float>(), n, stream);
}

// out[i][j] += sum over token pairs of (a1 . a2)(g1 . g2); factors flattened to rows.
void ghost_gram(Tensor a1, Tensor g1, Tensor a2, Tensor g2, int64_t S1, int64_t S2, Tensor out,
                Tensor err, bool diag_only) {
  const c10::cuda::CUDAGuard guard(a1.device());
  check_err(err);
  auto oa1 = operand(a1, "a1");
  auto oa2 = operand(a2, "a2");
  auto og1 = operand(g1, "g1");
  auto og2 = operand(g2, "g2");
  TORCH_CHECK(a1.dim() == 2 && a2.dim() == 2 && g1.dim() == 2 && g2.dim() == 2,
              "ghost_gram takes flattened (rows, width) factors");
  TORCH_CHECK(oa1.cols == oa2.cols && og1.cols == og2.cols, "factor widths disagree");
  TORCH_CHECK(oa1.rows == og1.rows && oa2.rows == og2.rows, "factor row counts disagree");
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.dim() == 2 && out.stride(1) == 1,
              "out must be a (B1, B2) fp32 matrix");
  bw::GhostParams p{};
  p.M = (int)oa1.rows;
  p.N = (int)oa2.rows;
  p.K = (int)oa1.cols;
  p.D = (int)og1.cols;
  p.S1 = (int)S1;
  p.S2 = (int)S2;
  p.B1 = (int)(p.M / p.S1);
  p.B2 = (int)(p.N / p.S2);
  TORCH_CHECK(p.B1 * p.S1 == p.M && p.B2 * p.S2 == p.N, "rows must be B*S");
  TORCH_CHECK(out.size(0) == p.B1 && out.size(1) == p.B2, "out must be (B1, B2)");
  p.out = out.data_ptr<float>();
  p.ldo = out.stride(0);
  p.diag_only = diag_only ? 1 : 0;
  p.err = err.data_ptr<int>();
  if (p.M == 0 || p.N == 0) return;
  bw::ghost_gram_launch(oa1, oa2, og1, og2, p, at::cuda::getCurrentCUDAStream());
}

// Embedding-layer cross-gram: out[i][j] += sum over token pairs with equal ids of g1 . g2
// (tok: flattened int64 ids of B*S rows; g: (B*S, E) bf16).
void ghost_gram_tokens(Tensor tok1, Tensor g1, Tensor tok2, Tensor g2, int64_t S1, int64_t S2, Tensor out,
                       Tensor err, bool diag_only) {
  const c10::cuda::CUDAGuard guard(g1.device());
  check_err(err);
  auto og1 = operand(g1, "g1");
  auto og2 = operand(g2, "g2");
  TORCH_CHECK(g1.dim() == 2 && g2.dim() == 2 && og1.cols == og2.cols, "g1 / g2: (rows, E) with one E");
  for (auto* t : {&tok1, &tok2})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt64 && t->is_contiguous(), "token ids: int64 CUDA");
  TORCH_CHECK(tok1.numel() == og1.rows && tok2.numel() == og2.rows, "one token id per gradient row");
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.dim() == 2 && out.stride(1) == 1, "out: (B1, B2) fp32");
  bw::GhostParams p{};
  p.M = (int)og1.rows;
  p.N = (int)og2.rows;
  p.K = 0;
  p.D = (int)og1.cols;
  p.S1 = (int)S1;
  p.S2 = (int)S2;
  p.B1 = (int)(p.M / p.S1);
  p.B2 = (int)(p.N / p.S2);
  TORCH_CHECK(p.B1 * p.S1 == p.M && p.B2 * p.S2 == p.N, "rows must be B*S");
  TORCH_CHECK(out.size(0) == p.B1 && out.size(1) == p.B2, "out must be (B1, B2)");
  p.out = out.data_ptr<float>();
  p.ldo = out.stride(0);
  p.err = err.data_ptr<int>();
  p.tok1 = reinterpret_cast<const long long*>(tok1.data_ptr<int64_t>());
  p.tok2 = reinterpret_cast<const long long*>(tok2.data_ptr<int64_t>());
  p.diag_only = diag_only ? 1 : 0;
  if (p.M == 0 || p.N == 0) return;
  // the activation maps are unused in token mode; the gradient operands stand in for them
  bw::ghost_gram_launch(og1, og2, og1, og2, p, at::cuda::getCurrentCUDAStream());
}

__nv_bfloat16* bf(const Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

void check_rows(const Tensor& t, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16 && t.is_contiguous(), name, " must be contiguous bf16");
  TORCH_CHECK(t.size(-1) % 8 == 0, name, " width must be a multiple of 8");
}

std::vector<Tensor> rmsnorm_fwd(Tensor x, Tensor w, double eps) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_rows(x, "x");
  check_rows(w, "w");
  const int cols = (int)x.size(-1);
  const int rows = (int)(x.numel() / cols);
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (bw::rows_norm_supported(cols)) {
    bw::RowsNorm a{bf(x), nullptr, nullptr, bf(w), bf(y), rstd.data_ptr<float>(), rows, cols, (float)eps};
    bw::rows_norm_fwd(a, at::cuda::getCurrentCUDAStream());
  } else {
    bw::rmsnorm_fwd(bf(x), bf(w), bf(y), rstd.data_ptr<float>(), rows, cols, (float)eps,
                    at::cuda::getCurrentCUDAStream());
  }
  return {y, rstd};
}

// h = x + delta (bf16), y = rmsnorm(h) * w: returns {y, h, rstd}.
std::vector<Tensor> add_rmsnorm_fwd(Tensor x, Tensor delta, Tensor w, double eps) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_rows(x, "x");
  check_rows(delta, "delta");
  check_rows(w, "w");
  TORCH_CHECK(x.sizes() == delta.sizes(), "x and delta must have the same shape");
  const int cols = (int)x.size(-1);
  const int rows = (int)(x.numel() / cols);
  TORCH_CHECK(bw::rows_norm_supported(cols), "add_rmsnorm: width must be a multiple of 8 and <= 4096");
  TORCH_CHECK(w.numel() == cols, "w must have one entry per column");
  auto y = torch::empty_like(x);
  auto h = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  bw::RowsNorm a{bf(x), bf(delta), bf(h), bf(w), bf(y), rstd.data_ptr<float>(), rows, cols, (float)eps};
  bw::rows_norm_fwd(a, at::cuda::getCurrentCUDAStream());
  return {y, h, rstd};
}

// dx = rmsnorm_bwd(dy) + dres (dres optional).
Tensor rmsnorm_bwd_acc(Tensor dy, Tensor x, Tensor w, Tensor rstd, c10::optional<Tensor> dres) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_rows(dy, "dy");
  check_rows(x, "x");
  const int cols = (int)x.size(-1);
  const int rows = (int)(x.numel() / cols);
  TORCH_CHECK(bw::rows_norm_supported(cols), "rmsnorm_bwd_acc: width must be a multiple of 8 and <= 4096");
  const __nv_bfloat16* dr = nullptr;
  if (dres.has_value() && dres->defined()) {
    check_rows(*dres, "dres");
    TORCH_CHECK(dres->numel() == x.numel(), "dres must match x");
    dr = bf(*dres);
  }
  auto dx = torch::empty_like(x);
  bw::RowsNormBwd a{bf(dy), bf(x), bf(w), rstd.data_ptr<float>(), dr, bf(dx), rows, cols};
  bw::rows_norm_bwd(a, at::cuda::getCurrentCUDAStream());
  return dx;
}

bw::RopeTensor rope_tensor(const Tensor& in, const Tensor& out, const char* name) {
  check_cuda(in, name);
  TORCH_CHECK(in.scalar_type() == torch::kBFloat16 && in.dim() == 4 && in.stride(3) == 1, name,
              " must be (B, T, H, D) bf16 with a contiguous head dim");
  for (int d = 0; d < 3; ++d)
    TORCH_CHECK(in.stride(d) % 8 == 0, name, " strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(in.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
  return bw::RopeTensor{bf(in), bf(out), in.stride(0), in.stride(1), in.stride(2),
                        out.stride(0), out.stride(1), out.stride(2)};
}

// Rotate q (B, T, Hq, D) and k (B, T, Hk, D) by position (inverse: by -theta); outputs contiguous.
std::vector<Tensor> rope(Tensor q, Tensor k, Tensor cos, Tensor sin, bool inverse) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && q.size(0) == k.size(0) && q.size(1) == k.size(1) &&
                  q.size(3) == k.size(3), "q and k must be (B, T, H, D) with matching B, T, D");
  const int D = (int)q.size(3);
  TORCH_CHECK(bw::rope_supported(D, (int)(q.size(2) + k.size(2))),
              "fused RoPE needs head_dim % 16 == 0 and (q heads + k heads) * head_dim / 16 <= 1024");
  TORCH_CHECK(cos.scalar_type() == torch::kFloat32 && sin.scalar_type() == torch::kFloat32 &&
                  cos.is_contiguous() && sin.is_contiguous() && cos.dim() == 2 && cos.size(1) == D / 2 &&
                  cos.size(0) >= q.size(1) && sin.sizes() == cos.sizes(),
              "cos/sin must be contiguous fp32 (>= T, D/2)");
  auto qo = torch::empty(q.sizes(), q.options());
  auto ko = torch::empty(k.sizes(), k.options());
  bw::RopeArgs a{rope_tensor(q, qo, "q"), rope_tensor(k, ko, "k"), cos.data_ptr<float>(), sin.data_ptr<float>(),
                 (int)q.size(0), (int)q.size(1), (int)q.size(2), (int)k.size(2), D};
  bw::rope(a, inverse, at::cuda::getCurrentCUDAStream());
  return {qo, ko};
}

// Per-sample Adam direction of g (rows, p) fp32 against moments m0, v0 (p) fp32.
Tensor adam_direction(Tensor g, Tensor m0, Tensor v0, double b1, double b2, int64_t step, double eps) {
  const c10::cuda::CUDAGuard guard(g.device());
  check_cuda(g, "g");
  TORCH_CHECK(g.scalar_type() == torch::kFloat32 && m0.scalar_type() == torch::kFloat32 &&
                  v0.scalar_type() == torch::kFloat32, "adam_direction works in fp32");
  TORCH_CHECK(g.is_contiguous() && m0.is_contiguous() && v0.is_contiguous(), "inputs must be contiguous");
  const long long p = g.size(-1);
  TORCH_CHECK(m0.numel() == p && v0.numel() == p, "moments must have one entry per column");
  TORCH_CHECK(p % 4 == 0, "width must be a multiple of 4");
  TORCH_CHECK(step >= 1, "step must be >= 1");
  auto out = torch::empty_like(g);
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  bw::adam_direction(g.data_ptr<float>(), m0.data_ptr<float>(), v0.data_ptr<float>(), out.data_ptr<float>(),
                     g.numel() / p, p, (float)b1, (float)b2, (float)(1.0 / bc1), (float)(1.0 / std::sqrt(bc2)),
                     (float)eps, at::cuda::getCurrentCUDAStream());
  return out;
}

Tensor rmsnorm_bwd(Tensor dy, Tensor x, Tensor w, Tensor rstd) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_rows(dy, "dy");
  check_rows(x, "x");
  const int cols = (int)x.size(-1);
  const int rows = (int)(x.numel() / cols);
  auto dx = torch::empty_like(x);
  if (bw::rows_norm_supported(cols)) {
    bw::RowsNormBwd a{bf(dy), bf(x), bf(w), rstd.data_ptr<float>(), nullptr, bf(dx), rows, cols};
    bw::rows_norm_bwd(a, at::cuda::getCurrentCUDAStream());
  } else {
    bw::rmsnorm_bwd(bf(dy), bf(x), bf(w), rstd.data_ptr<float>(), bf(dx), rows, cols,
                    at::cuda::getCurrentCUDAStream());
  }
  return dx;
}

Tensor swiglu_fwd(Tensor g, Tensor u) {
  const c10::cuda::CUDAGuard guard(g.device());
  check_rows(g, "g");
  check_rows(u, "u");
  auto h = torch::empty_like(g);
  bw::swiglu_fwd(bf(g), bf(u), bf(h), g.numel(), at::cuda::getCurrentCUDAStream());
  return h;
}

std::vector<Tensor> swiglu_bwd(Tensor dh, Tensor g, Tensor u) {
  const c10::cuda::CUDAGuard guard(g.device());
  check_rows(dh, "dh");
  auto dg = torch::empty_like(g);
  auto du = torch::empty_like(u);
  bw::swiglu_bwd(bf(dh), bf(g), bf(u), bf(dg), bf(du), g.numel(), at::cuda::getCurrentCUDAStream());
  return {dg, du};
}

std::vector<Tensor> ce_fwd(Tensor logits, Tensor target) {
  const c10::cuda::CUDAGuard guard(logits.device());
  check_cuda(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == torch::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1,
              "logits must be (rows, vocab) bf16, contiguous rows");
  TORCH_CHECK(logits.size(1) % 8 == 0 && logits.stride(0) % 8 == 0, "vocab must be a multiple of 8");
  TORCH_CHECK(target.scalar_type() == torch::kInt64 && target.is_contiguous(), "target must be int64");
  const int rows = (int)logits.size(0);
  auto loss = torch::empty({rows}, logits.options().dtype(torch::kFloat32));
  auto lse = torch::empty({rows}, logits.options().dtype(torch::kFloat32));
  bw::ce_fwd(bf(logits), target.data_ptr<int64_t>(), loss.data_ptr<float>(), lse.data_ptr<float>(), rows,
             (int)logits.size(1), logits.stride(0), at::cuda::getCurrentCUDAStream());
  return {loss, lse};
}

void ce_bwd_inplace(Tensor logits, Tensor lse, Tensor target, Tensor gscale) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(gscale.scalar_type() == torch::kFloat32 && gscale.is_cuda(), "gscale must be a CUDA float");
  bw::ce_bwd_inplace(bf(logits), lse.data_ptr<float>(), target.data_ptr<int64_t>(), gscale.data_ptr<float>(),
                     (int)logits.size(0), (int)logits.size(1), logits.stride(0), at::cuda::getCurrentCUDAStream());
}

}  // namespace

// Dense per-sample embedding gradients (B * vocab, E) from the token rows of g (n, E) sorted
// by key b * vocab + id (`order`) and each output row's first position in that order
// (`starts`, R + 1 entries).  bf16 or fp32, the output in g's dtype; E * elem size a multiple
// of 16 bytes.
Tensor embedding_dense_grad(Tensor starts, Tensor order, Tensor g, int64_t rows) {
  const c10::cuda::CUDAGuard guard(g.device());
  TORCH_CHECK(g.is_cuda() && g.dim() == 2 && g.is_contiguous(), "g must be a contiguous (n, E) CUDA tensor");
  TORCH_CHECK(g.scalar_type() == torch::kBFloat16 || g.scalar_type() == torch::kFloat32, "g must be bf16 or fp32");
  TORCH_CHECK(starts.is_cuda() && order.is_cuda() && starts.scalar_type() == torch::kInt64 &&
                  order.scalar_type() == torch::kInt64 && starts.is_contiguous() && order.is_contiguous() &&
                  starts.numel() == rows + 1 && order.numel() == g.size(0),
              "starts (rows + 1) and order (one per row of g) must be contiguous int64 vectors");
  const int elem = (int)g.element_size();
  const int E = (int)g.size(1);
  TORCH_CHECK((E * elem) % 16 == 0, "the embedding width must fill whole 16-byte vectors");
  auto out = torch::empty({rows, (int64_t)E}, g.options());
  bw::embedding_dense_grad(starts.data_ptr<int64_t>(), order.data_ptr<int64_t>(), g.data_ptr(), out.data_ptr(), rows,
                           E, elem, at::cuda::getCurrentCUDAStream());
  return out;
}

// Gated RMSNorm (Mamba2 mixer): y (R, D) fp32 contiguous, g (R, D) bf16 with unit column
// stride, w (D) bf16; returns (out bf16 (R, D), rstd fp32 (R)).
std::vector<Tensor> gated_rms_fwd(Tensor y, Tensor g, Tensor w, double eps) {
  const c10::cuda::CUDAGuard guard(y.device());
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == torch::kFloat32 && y.dim() == 2 && y.is_contiguous(),
              "y must be a contiguous (R, D) fp32 CUDA tensor");
  TORCH_CHECK(g.scalar_type() == torch::kBFloat16 && g.dim() == 2 && g.sizes() == y.sizes() && g.stride(1) == 1,
              "g must be (R, D) bf16 with unit column stride");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && w.numel() == y.size(1), "w: (D) bf16");
  TORCH_CHECK(y.size(1) <= bw::kGatedNormMaxCols, "D above the kernel's limit");
  auto out = torch::empty(y.sizes(), y.options().dtype(torch::kBFloat16));
  auto rstd = torch::empty({y.size(0)}, y.options());
  bw::gated_rms_fwd(y.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), g.stride(0),
                    reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                    reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), rstd.data_ptr<float>(), (int)y.size(0),
                    (int)y.size(1), (float)eps, at::cuda::getCurrentCUDAStream());
  return {out, rstd};
}

// Its backward: returns (dy fp32, dg bf16 contiguous, dw fp32).
std::vector<Tensor> gated_rms_bwd(Tensor dout, Tensor y, Tensor g, Tensor w, Tensor rstd) {
  const c10::cuda::CUDAGuard guard(y.device());
  TORCH_CHECK(dout.scalar_type() == torch::kBFloat16 && dout.is_contiguous() && dout.sizes() == y.sizes(),
              "dout must be contiguous (R, D) bf16");
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.is_contiguous() && g.scalar_type() == torch::kBFloat16 &&
                  g.sizes() == y.sizes() && g.stride(1) == 1 && w.scalar_type() == torch::kBFloat16 &&
                  w.numel() == y.size(1) && rstd.scalar_type() == torch::kFloat32 && rstd.numel() == y.size(0),
              "saved tensors of gated_rms_fwd expected");
  auto dy = torch::empty_like(y);
  auto dg = torch::empty(y.sizes(), y.options().dtype(torch::kBFloat16));
  auto dw = torch::empty({y.size(1)}, y.options());
  auto part = torch::empty({bw::gated_rms_bwd_parts((int)y.size(0)), y.size(1)}, y.options());
  bw::gated_rms_bwd(reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), y.data_ptr<float>(),
                    reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), g.stride(0),
                    reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), rstd.data_ptr<float>(), dy.data_ptr<float>(),
                    reinterpret_cast<__nv_bfloat16*>(dg.data_ptr()), part.data_ptr<float>(), dw.data_ptr<float>(),
                    (int)y.size(0), (int)y.size(1), at::cuda::getCurrentCUDAStream());
  return {dy, dg, dw};
}

// Intra-chunk SSD (Mamba2): cb (B, G, C, S, S), cum (B, H, C, S), x (B, C, S, H, 64), all fp32
// contiguous; returns y like x.
void check_ssd(const Tensor& cb, const Tensor& cum, const Tensor& x) {
  for (const Tensor* t : {&cb, &cum, &x})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kFloat32 && t->is_contiguous(),
                "SSD operands must be contiguous fp32 CUDA tensors");
  TORCH_CHECK(cb.dim() == 5 && cum.dim() == 4 && x.dim() == 5, "cb (B,G,C,S,S), cum (B,H,C,S), x (B,C,S,H,P)");
  const auto B = x.size(0), C = x.size(1), S = x.size(2), H = x.size(3), G = cb.size(1);
  TORCH_CHECK(x.size(4) == 64 && S % 64 == 0, "head dim 64 and a chunk length that is a multiple of 64");
  TORCH_CHECK(cb.size(0) == B && cb.size(2) == C && cb.size(3) == S && cb.size(4) == S && H % G == 0,
              "cb does not match x");
  TORCH_CHECK(cum.size(0) == B && cum.size(1) == H && cum.size(2) == C && cum.size(3) == S, "cum does not match x");
}

Tensor ssd_intra_fwd(Tensor cb, Tensor cum, Tensor x) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_ssd(cb, cum, x);
  auto y = torch::empty_like(x);
  bw::ssd_intra_fwd(cb.data_ptr<float>(), cum.data_ptr<float>(), x.data_ptr<float>(), y.data_ptr<float>(),
                    (int)x.size(0), (int)x.size(1), (int)x.size(2), (int)x.size(3), (int)cb.size(1),
                    at::cuda::getCurrentCUDAStream());
  return y;
}

// Its backward: returns (dcb, dcum, dx).
std::vector<Tensor> ssd_intra_bwd(Tensor cb, Tensor cum, Tensor x, Tensor dy) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_ssd(cb, cum, x);
  TORCH_CHECK(dy.sizes() == x.sizes() && dy.scalar_type() == torch::kFloat32 && dy.is_contiguous(),
              "dy must be a contiguous fp32 tensor shaped like x");
  auto dx = torch::empty_like(x);
  auto dcb = torch::zeros_like(cb);
  auto dcum = torch::zeros_like(cum);
  bw::ssd_intra_bwd(cb.data_ptr<float>(), cum.data_ptr<float>(), x.data_ptr<float>(), dy.data_ptr<float>(),
                    dx.data_ptr<float>(), dcb.data_ptr<float>(), dcum.data_ptr<float>(), (int)x.size(0),
                    (int)x.size(1), (int)x.size(2), (int)x.size(3), (int)cb.size(1), at::cuda::getCurrentCUDAStream());
  return {dcb, dcum, dx};
}

// Causal depthwise conv (4 taps) + SiLU: x (B, L, C) bf16 with unit channel stride (a column
// slice of a larger projection is fine), w (C, 1, 4) bf16, bias (C) bf16 or None.
void check_conv(const Tensor& x, const Tensor& w, const c10::optional<Tensor>& bias) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 3 && x.stride(2) == 1,
              "x must be (B, L, C) bf16 with unit channel stride");
  TORCH_CHECK(x.size(2) % 2 == 0 && x.stride(1) % 2 == 0 && x.stride(0) % 2 == 0 &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 4 == 0,
              "channel pairs must be 4-byte aligned");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && w.numel() == x.size(2) * bw::kConvTaps,
              "w must be a contiguous (C, 1, 4) bf16 tensor");
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->is_contiguous() && bias->numel() == x.size(2),
                "bias must be (C) bf16");
}

Tensor causal_conv_silu_fwd(Tensor x, Tensor w, c10::optional<Tensor> bias) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_conv(x, w, bias);
  auto out = torch::empty({x.size(0), x.size(1), x.size(2)}, x.options());
  const bool hb = bias.has_value() && bias->defined();
  bw::causal_conv_silu_fwd(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(1), x.stride(0),
                           reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                           hb ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr,
                           reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)x.size(0), (int)x.size(1),
                           (int)x.size(2), at::cuda::getCurrentCUDAStream());
  return out;
}

// Its backward: returns (dx bf16 (B, L, C) contiguous, dw fp32 (C, 4), dbias fp32 (C)).
std::vector<Tensor> causal_conv_silu_bwd(Tensor dout, Tensor x, Tensor w, c10::optional<Tensor> bias) {
  const c10::cuda::CUDAGuard guard(x.device());
  check_conv(x, w, bias);
  TORCH_CHECK(dout.scalar_type() == torch::kBFloat16 && dout.is_contiguous() && dout.sizes() == x.sizes(),
              "dout must be contiguous (B, L, C) bf16");
  const int B = (int)x.size(0), L = (int)x.size(1), C = (int)x.size(2);
  auto f32 = x.options().dtype(torch::kFloat32);
  auto dx = torch::empty({B, L, C}, x.options());
  const int parts = bw::causal_conv_bwd_parts(B, L);
  auto dw_part = torch::empty({parts, C, bw::kConvTaps}, f32);
  auto db_part = torch::empty({parts, C}, f32);
  auto dw = torch::empty({C, bw::kConvTaps}, f32);
  auto db = torch::empty({C}, f32);
  const bool hb = bias.has_value() && bias->defined();
  bw::causal_conv_silu_bwd(reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                           reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(1), x.stride(0),
                           reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
                           hb ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr,
                           reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dw_part.data_ptr<float>(),
                           db_part.data_ptr<float>(), dw.data_ptr<float>(), db.data_ptr<float>(), B, L, C,
                           at::cuda::getCurrentCUDAStream());
  return {dx, dw, db};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of dattri_llm_b200";
  m.def("gemm_tn", &gemm_tn, "C (op)= alpha * A @ B^T on tcgen05 tensor cores");
  m.def("gemm_tn_seg", &gemm_tn_seg, "A @ B^T stored per segment as (S, N, T) bf16");
  m.def("gemm_grouped", &gemm_grouped, "one launch for many same-shaped batched A @ B^T problems");
  m.def("ghost_gram_tokens", &ghost_gram_tokens, "embedding-layer cross-gram: gradient Gram masked by token equality",
        py::arg("tok1"), py::arg("g1"), py::arg("tok2"), py::arg("g2"), py::arg("S1"), py::arg("S2"), py::arg("out"),
        py::arg("err"), py::arg("diag_only") = false);
  m.def("ghost_gram", &ghost_gram, "fused factorized cross-gram of per-sample gradients", py::arg("a1"), py::arg("g1"),
        py::arg("a2"), py::arg("g2"), py::arg("S1"), py::arg("S2"), py::arg("out"), py::arg("err"),
        py::arg("diag_only") = false);
  m.def("ag_score", &ag_score, "fused NVLink all-gather of peer train blocks + score GEMM");
  m.def("peer_barrier", &peer_barrier, "cross-GPU barrier on peer-mapped flags (bounded wait)");
  m.def("gemm_tn_peers", &gemm_tn_peers, "A @ B^T with B sharded over the peers, read over NVLink in the GEMM");
  m.def("gemm_tn_staged", &gemm_tn_staged, "A @ B^T with B's peer shards all-gathered inside the launch");
  m.def("norm_per_sample_grad", &norm_per_sample_grad, "per-sample LayerNorm/RMSNorm parameter gradients");
  m.def("causal_conv_silu_fwd", &causal_conv_silu_fwd, "causal depthwise conv (4 taps) + SiLU, token-major");
  m.def("causal_conv_silu_bwd", &causal_conv_silu_bwd, "backward of causal_conv_silu_fwd: (dx, dw, dbias)");
  m.def("ssd_intra_fwd", &ssd_intra_fwd, "intra-chunk SSD: y = ((C B^T) . exp(cum_s - cum_t)) x, causal");
  m.def("ssd_intra_bwd", &ssd_intra_bwd, "backward of ssd_intra_fwd: (dcb, dcum, dx)");
  m.def("gated_rms_fwd", &gated_rms_fwd, "gated RMSNorm w * rmsnorm(y * silu(g)) (Mamba2 mixer), bf16 out");
  m.def("gated_rms_bwd", &gated_rms_bwd, "backward of gated_rms_fwd");
  m.def("embedding_dense_grad", &embedding_dense_grad, "dense per-sample embedding gradients, every row written once");
  m.def("gemm_ragged", &gemm_ragged, "ragged grouped GEMM over expert row segments (optionally scattered home)",
        py::arg("A"), py::arg("B3"), py::arg("C"), py::arg("tile_prefix"), py::arg("base"), py::arg("len"),
        py::arg("max_tiles"), py::arg("peer_C"), py::arg("scatter"), py::arg("err"), py::arg("bn") = 0);
  m.def("swiglu_split", &swiglu_split);
  m.def("swiglu_split_bwd", &swiglu_split_bwd);
  m.def("moe_dispatch", &moe_dispatch, "expert-parallel dispatch: rows stored into their experts' ranks");
  m.def("mask_gather", &mask_gather, "mask projection of factorized gradients (gather-contract)");
  m.def("moe_count", &moe_count, "MoE routing histogram");
  m.def("moe_place", &moe_place, "MoE receive layout and owner-side ragged GEMM tables");
  m.def("moe_combine", &moe_combine, "MoE combine: router-weighted sum of the k returned rows");
  m.def("moe_combine_bwd_dispatch", &moe_combine_bwd_dispatch, "combine backward fused with the gradient dispatch");
  m.def("gemm_tn_rs", &gemm_tn_rs, "GEMM with the reduce-scatter in its epilogue (peer slot stores)");
  m.def("split3_bf16", &split3_bf16, "bf16x3 split operand of an fp32 matrix (K-concatenated hi/lo segments)");
  m.def("transpose_last2", &transpose_last2, "bf16 transpose of the last two axes (tiled through shared memory)");
  m.def("gram_acc", &gram_acc, "C += alpha * At At^T (symmetric tiles, split-K, fp32 atomics)");
  m.def("gemm_tn_tail", &gemm_tn_tail, "C = A B^T (bf16 rows) and C2 = A Btail^T (token-major) in one launch");
  m.def("slot_reduce", &slot_reduce, "owner-side sum of reduce-scatter slots");
  m.def("allreduce_phase", &allreduce_phase, "NVLink peer all-reduce: 0 one-shot, 1 reduce-scatter, 2 all-gather");
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("rmsnorm_bwd_acc", &rmsnorm_bwd_acc);
  m.def("rope", &rope);
  m.def("adam_direction", &adam_direction);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd_inplace", &ce_bwd_inplace);
  bw::register_projector(m);
}
