// In-kernel tensor-parallel collectives over NVLink peer memory.
//
// fused_allreduce_add_rmsnorm finishes a row-parallel projection (o_proj / down_proj) on every
// rank in ONE kernel:
//   1. signal: this rank's split-K partials (written by the GEMM just before, in a peer-mapped
//      buffer) are ready -> store `epoch` into flags[phase 1][my rank] of every peer;
//   2. wait (bounded) until every peer's phase-1 flag reached `epoch`;
//   3. reduce-scatter by rows: the CTAs of this rank read the partials of ITS rows from all ranks
//      over NVLink, round to bf16 (as a bf16 GEMM output would be), add the residual and apply
//      RMSNorm -- a row is split over a cluster of CTAs that combine their sums of squares
//      through distributed shared memory;
//   4. all-gather by push: each finished row (normalised output and new residual) is stored into
//      every rank's output buffers;
//   5. the last CTA of the rank signals phase 2 to every peer and waits (bounded) for all of them,
//      so when the kernel ends every rank holds all rows.
// `epoch` lives in device memory and is advanced by the kernel itself, so the launch can be
// captured in a CUDA graph.  Every wait gives up after a bounded number of polls (kSpinLimit unless
// lowered for a test), records
// kTimeoutPeerFlag in the status word and lets the kernel finish (no hang, no trap).
//
// One buffer of each kind suffices: a rank can only overwrite a peer's buffers after that peer
// has signalled phase 1 of the NEXT call, i.e. after it consumed everything of this one.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lsb {
namespace {

#define LSB_CHECK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

constexpr int kMaxRanks = 8;
constexpr int kCluster = 8;       // CTAs per row
constexpr int kThreads = 128;

struct PeerPtrs {
  float* part[kMaxRanks];
  bf16* out[kMaxRanks];
  bf16* res[kMaxRanks];
  uint32_t* flags[kMaxRanks];     // [0, W): phase 1, [W, 2W): phase 2, [2W]: epoch, [2W+1]: CTA counter
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_v2(bf16* p, uint2 v) {
  asm volatile("st.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

// Polls before a peer-flag wait gives up (kSpinLimit unless lowered by comm_set_spin_limit, which
// the failure-detection test uses to make a wait on a flag nothing sets end in milliseconds).
__device__ uint32_t g_flag_spin_limit = kSpinLimit;

__device__ bool wait_flags(const uint32_t* flags, int W, uint32_t epoch, int* status) {
  const uint32_t limit = *((volatile uint32_t*)&g_flag_spin_limit);
  for (int r = 0; r < W; ++r) {
    uint32_t i = 0;
    while ((int32_t)(ld_acquire_sys(flags + r) - epoch) < 0) {
      if (++i > limit) {
        record_error(status, kTimeoutPeerFlag);
        return false;
      }
    }
  }
  return true;
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    fused_allreduce_add_rmsnorm_kernel(PeerPtrs peers, const bf16* __restrict__ res_in,
                                       const bf16* __restrict__ w, int rank, int W, int S, int T, int N, float eps,
                                       int rows_per_rank, int* status) {
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float red[kThreads / 32];
  __shared__ float cta_ss;
  __shared__ uint32_t s_epoch;
  __shared__ int s_last;
  uint32_t* my_flags = peers.flags[rank];
  if (threadIdx.x == 0) s_epoch = *((volatile uint32_t*)(my_flags + 2 * W)) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int crank = (int)cluster.block_rank();
  const int row_slot = blockIdx.y;
  const bool first_cta = blockIdx.x == 0 && blockIdx.y == 0;

  // 1. phase-1 signal: our partials are complete (the GEMM kernel ended before this one began)
  if (first_cta && threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(peers.flags[threadIdx.x] + rank, epoch);
  }
  // 2. wait for every rank's partials
  if (threadIdx.x == 0) wait_flags(my_flags, W, epoch, status);
  __syncthreads();

  // 3. reduce-scatter + residual + RMSNorm for row `row` of this rank
  const int row = rank * rows_per_rank + row_slot;
  const bool have_row = row_slot < rows_per_rank && row < T;
  const int cols = N / kCluster;                // columns of this CTA (multiple of 4)
  const int c0 = crank * cols;
  const int64_t TN = (int64_t)T * N;
  float ss = 0.f;
  constexpr int kMaxPer = 4;                    // float4 chunks per thread (N <= 8192 * 2)
  float4 val[kMaxPer];
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int col = c0 + (threadIdx.x + k * kThreads) * 4;
    val[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!have_row || col >= c0 + cols) continue;
    const int64_t off = (int64_t)row * N + col;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < W; ++r)
      for (int s = 0; s < S; ++s) {
        const float4 p = __ldcv(reinterpret_cast<const float4*>(peers.part[r] + s * TN + off));
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
      }
    const uint2 rr = *reinterpret_cast<const uint2*>(res_in + off);
    const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rr.x);
    const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rr.y);
    val[k].x = to_f(to_b(acc.x)) + __low2float(r01);
    val[k].y = to_f(to_b(acc.y)) + __high2float(r01);
    val[k].z = to_f(to_b(acc.z)) + __low2float(r23);
    val[k].w = to_f(to_b(acc.w)) + __high2float(r23);
    ss += val[k].x * val[k].x + val[k].y * val[k].y + val[k].z * val[k].z + val[k].w * val[k].w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < kThreads / 32; ++i) t += red[i];
    cta_ss = t;
  }
  cluster.sync();
  float total = 0.f;
  for (int c = 0; c < kCluster; ++c) total += *cluster.map_shared_rank(&cta_ss, c);
  cluster.sync();   // peers' shared memory must stay valid until everyone has read it
  const float inv = rsqrtf(total / N + eps);

  // 4. all-gather by push
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int col = c0 + (threadIdx.x + k * kThreads) * 4;
    if (!have_row || col >= c0 + cols) continue;
    const int64_t off = (int64_t)row * N + col;
    const uint2 wr = *reinterpret_cast<const uint2*>(w + col);
    const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wr.x);
    const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wr.y);
    const float v[4] = {val[k].x, val[k].y, val[k].z, val[k].w};
    const float wv[4] = {__low2float(w01), __high2float(w01), __low2float(w23), __high2float(w23)};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = to_f(to_b(to_f(to_b(v[j] * inv)) * wv[j]));
    __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]), o23 = __floats2bfloat162_rn(o[2], o[3]);
    __nv_bfloat162 s01 = __floats2bfloat162_rn(v[0], v[1]), s23 = __floats2bfloat162_rn(v[2], v[3]);
    uint2 ov, sv;
    ov.x = *reinterpret_cast<uint32_t*>(&o01);
    ov.y = *reinterpret_cast<uint32_t*>(&o23);
    sv.x = *reinterpret_cast<uint32_t*>(&s01);
    sv.y = *reinterpret_cast<uint32_t*>(&s23);
    for (int r = 0; r < W; ++r) {
      st_v2(peers.out[r] + off, ov);
      st_v2(peers.res[r] + off, sv);
    }
  }
  // 5. last CTA of this rank: phase-2 signal, then wait for all ranks' rows
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int total_ctas = gridDim.x * gridDim.y;
    const uint32_t prev = atomicAdd(my_flags + 2 * W + 1, 1u);
    s_last = prev == (uint32_t)(total_ctas - 1);
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    my_flags[2 * W + 1] = 0u;
    __threadfence_system();
    for (int r = 0; r < W; ++r) st_release_sys(peers.flags[r] + W + rank, epoch);
    wait_flags(my_flags + W, W, epoch, status);
    *((volatile uint32_t*)(my_flags + 2 * W)) = epoch;
    __threadfence();
  }
}

}  // namespace

int* status_ptr(const at::Tensor& status);

// ---- host: symmetric buffers via CUDA IPC -------------------------------------------------------
int64_t comm_alloc(int64_t nbytes) {
  void* p = nullptr;
  auto e = cudaMalloc(&p, nbytes);
  LSB_CHECK(e == cudaSuccess, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
  cudaMemset(p, 0, nbytes);
  return reinterpret_cast<int64_t>(p);
}

void comm_free(int64_t p) { cudaFree(reinterpret_cast<void*>(p)); }

at::Tensor comm_ipc_handle(int64_t p) {
  cudaIpcMemHandle_t h;
  auto e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(p));
  LSB_CHECK(e == cudaSuccess, std::string("cudaIpcGetMemHandle failed: ") + cudaGetErrorString(e));
  auto t = at::empty({(int64_t)sizeof(h)}, at::kByte);
  memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t comm_open_handle(at::Tensor handle) {
  cudaIpcMemHandle_t h;
  LSB_CHECK(handle.numel() == (int64_t)sizeof(h), "bad IPC handle size");
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  auto e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  LSB_CHECK(e == cudaSuccess, std::string("cudaIpcOpenMemHandle failed: ") + cudaGetErrorString(e));
  return reinterpret_cast<int64_t>(p);
}

void comm_close_handle(int64_t p) { cudaIpcCloseMemHandle(reinterpret_cast<void*>(p)); }

// Spin limit of the peer-flag waits on the current device, clamped to [1024, kSpinLimit].
void comm_set_spin_limit(int64_t polls) {
  uint32_t v = (uint32_t)std::min<int64_t>(std::max<int64_t>(polls, 1024), (int64_t)kSpinLimit);
  auto e = cudaMemcpyToSymbol(g_flag_spin_limit, &v, sizeof(v));
  LSB_CHECK(e == cudaSuccess, std::string("setting the spin limit failed: ") + cudaGetErrorString(e));
}

// part/out/res/flags: W base addresses each (this rank's mapping of every rank's buffers)
void fused_allreduce_add_rmsnorm(std::vector<int64_t> part, std::vector<int64_t> out, std::vector<int64_t> res,
                                 std::vector<int64_t> flags, at::Tensor res_in, at::Tensor w, int64_t rank, int64_t S,
                                 int64_t T, int64_t N, double eps, at::Tensor status) {
  const int W = part.size();
  LSB_CHECK(W >= 1 && W <= kMaxRanks && out.size() == (size_t)W && res.size() == (size_t)W && flags.size() == (size_t)W,
            "peer pointer lists must have one entry per rank (<= 8)");
  LSB_CHECK(N % (kCluster * 4) == 0 && N / kCluster <= 4 * 4 * kThreads, "hidden size unsupported by the fused path");
  LSB_CHECK(res_in.scalar_type() == at::kBFloat16 && res_in.is_contiguous() && res_in.numel() >= T * N, "bad residual");
  PeerPtrs p;
  for (int r = 0; r < W; ++r) {
    p.part[r] = reinterpret_cast<float*>(part[r]);
    p.out[r] = reinterpret_cast<bf16*>(out[r]);
    p.res[r] = reinterpret_cast<bf16*>(res[r]);
    p.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  const int rpr = (int)((T + W - 1) / W);
  dim3 grid(kCluster, std::max(rpr, 1));
  const at::cuda::CUDAGuard g(res_in.device());
  launch_pdl(fused_allreduce_add_rmsnorm_kernel, grid, dim3(kThreads), 0, at::cuda::getCurrentCUDAStream(), p,
             (const bf16*)res_in.data_ptr(), (const bf16*)w.data_ptr(), (int)rank, W, (int)S, (int)T, (int)N,
             (float)eps, rpr, status_ptr(status));
  auto e = cudaGetLastError();
  LSB_CHECK(e == cudaSuccess, std::string("fused all-reduce launch failed: ") + cudaGetErrorString(e));
}

}  // namespace lsb
