// Prefill -> decode KV-block push over NVLink (prefill/decode disaggregation).
//
// The paged pools are [layers, blocks, kv_heads, block_size, head_dim] (K and V separately), so
// one block of one layer is a contiguous run of kv_heads * block_size * head_dim elements.  The
// kernel runs on the prefill GPU and copies the listed (source block -> destination block) pairs
// of every layer, K and V, straight into the decode GPU's pool through its peer-mapped address:
// 16-byte loads from local HBM, 16-byte stores that cross NVLink, four in flight per thread.  A
// pair whose block id is outside either pool is skipped and recorded in the status word.
//
// Ordering: the launch is on the prefill device's current stream, after the prefill step that
// wrote the blocks and before any later step that could reuse them; the caller records an event
// after it and makes the decode stream wait on that event before the decode step reads the
// blocks.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace lsb {

int* status_ptr(const at::Tensor& status);

namespace {

constexpr int kPushThreads = 256;
constexpr int kUnroll = 4;

// One CTA per (pair, layer, K|V) item, grid-strided.
__global__ void __launch_bounds__(kPushThreads) kv_push_kernel(const uint4* __restrict__ src_k,
                                                              const uint4* __restrict__ src_v,
                                                              uint4* __restrict__ dst_k, uint4* __restrict__ dst_v,
                                                              const int* __restrict__ src_ids,
                                                              const int* __restrict__ dst_ids, int n_pairs,
                                                              int layers, int64_t block_vecs, int64_t src_blocks,
                                                              int64_t dst_blocks, int* status) {
  const int64_t items = (int64_t)n_pairs * layers * 2;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int kv = (int)(it & 1);
    const int64_t rest = it >> 1;
    const int layer = (int)(rest % layers);
    const int pair = (int)(rest / layers);
    const int s = src_ids[pair], d = dst_ids[pair];
    if (s < 0 || s >= src_blocks || d < 0 || d >= dst_blocks) {
      if (threadIdx.x == 0) record_error(status, kBadIndex);
      continue;
    }
    const uint4* src = (kv ? src_v : src_k) + ((int64_t)layer * src_blocks + s) * block_vecs;
    uint4* dst = (kv ? dst_v : dst_k) + ((int64_t)layer * dst_blocks + d) * block_vecs;
    int64_t i = threadIdx.x;
    for (; i + (kUnroll - 1) * kPushThreads < block_vecs; i += kUnroll * kPushThreads) {
      uint4 r[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) r[u] = __ldg(src + i + u * kPushThreads);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) dst[i + u * kPushThreads] = r[u];
    }
    for (; i < block_vecs; i += kPushThreads) dst[i] = __ldg(src + i);
  }
}

void ensure_peer_access(int src_dev, int dst_dev) {
  if (src_dev == dst_dev) return;
  static std::mutex mu;
  static std::set<std::pair<int, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({src_dev, dst_dev})) return;
  int can = 0;
  TORCH_CHECK(cudaDeviceCanAccessPeer(&can, src_dev, dst_dev) == cudaSuccess && can,
              "llmserve_b200: GPU ", src_dev, " cannot access GPU ", dst_dev, " as a peer");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(src_dev);
  cudaError_t e = cudaDeviceEnablePeerAccess(dst_dev, 0);
  cudaSetDevice(prev);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();   // clear the sticky-free "already enabled" status
  } else {
    TORCH_CHECK(e == cudaSuccess, "llmserve_b200: enabling peer access failed: ", cudaGetErrorString(e));
  }
  done.insert({src_dev, dst_dev});
}

}  // namespace

// src_k/src_v: this GPU's pools [L, Bs, kvh, bs, hd]; dst_k/dst_v: the destination pools
// [L, Bd, kvh, bs, hd] (another GPU's or this one's); src_ids/dst_ids: int32 [n] on this GPU.
void kv_push(at::Tensor src_k, at::Tensor src_v, at::Tensor dst_k, at::Tensor dst_v, at::Tensor src_ids,
             at::Tensor dst_ids, at::Tensor status) {
  TORCH_CHECK(src_k.is_cuda() && dst_k.is_cuda(), "llmserve_b200: kv_push needs CUDA pools");
  TORCH_CHECK(src_k.dim() == 5 && dst_k.dim() == 5, "llmserve_b200: pools must be [L, blocks, kvh, bs, hd]");
  TORCH_CHECK(src_k.sizes() == src_v.sizes() && dst_k.sizes() == dst_v.sizes(), "llmserve_b200: K/V pool mismatch");
  TORCH_CHECK(src_k.size(0) == dst_k.size(0) && src_k.size(2) == dst_k.size(2) && src_k.size(3) == dst_k.size(3) &&
                  src_k.size(4) == dst_k.size(4), "llmserve_b200: source and destination block shapes differ");
  TORCH_CHECK(src_k.scalar_type() == dst_k.scalar_type() && src_v.scalar_type() == dst_v.scalar_type(),
              "llmserve_b200: pool dtypes differ");
  for (const at::Tensor* t : {&src_k, &src_v, &dst_k, &dst_v})
    TORCH_CHECK(t->is_contiguous() && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "llmserve_b200: pools must be contiguous and 16-byte aligned");
  TORCH_CHECK(src_ids.scalar_type() == at::kInt && dst_ids.scalar_type() == at::kInt &&
                  src_ids.numel() == dst_ids.numel() && src_ids.device() == src_k.device() &&
                  dst_ids.device() == src_k.device(), "llmserve_b200: block ids must be int32 on the source GPU");
  TORCH_CHECK(src_v.device() == src_k.device() && dst_v.device() == dst_k.device(), "llmserve_b200: pool devices");
  const int n = src_ids.numel();
  if (n == 0) return;
  const int64_t block_bytes = src_k.size(2) * src_k.size(3) * src_k.size(4) * src_k.element_size();
  TORCH_CHECK(block_bytes % 16 == 0, "llmserve_b200: block bytes must be a multiple of 16");
  ensure_peer_access(src_k.device().index(), dst_k.device().index());
  const at::cuda::CUDAGuard g(src_k.device());
  const int layers = src_k.size(0);
  const int64_t items = (int64_t)n * layers * 2;
  const int grid = (int)std::min<int64_t>(items, 4 * 148);
  kv_push_kernel<<<grid, kPushThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const uint4*)src_k.data_ptr(), (const uint4*)src_v.data_ptr(), (uint4*)dst_k.data_ptr(),
      (uint4*)dst_v.data_ptr(), src_ids.data_ptr<int>(), dst_ids.data_ptr<int>(), n, layers, block_bytes / 16,
      src_k.size(1), dst_k.size(1), status_ptr(status));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace lsb
