// In-kernel tensor-parallel collectives over NVLink peer memory.
//
// Symmetric buffer of one rank (allocated per rank, mapped by every peer through CUDA IPC):
//   [0, kCtrlBytes)   control: flag words (uint32) and the argmax exchange slots
//   out   bf16 [max_tokens, N]            normalised rows of the last row-parallel layer
//   res   bf16 [max_tokens, N]            residual rows of the last row-parallel layer
//   inbox fp32 [W][S][rows][N]            split-K partial planes pushed by every rank's GEMM
// Flag words: [0, W) phase-1 arrivals, [W, 2W) phase-2 arrivals, [2W] collective epoch,
// [2W+1] CTA counter, [64, 64 + W) argmax arrivals, [64 + W] argmax epoch.
//
// A row-parallel projection (o_proj / down_proj) finishes in two kernels:
//   GEMM  (gemm_sm100.cu / awq_sm100.cu, PartDest with one inbox per rank): the epilogue stores
//         the fp32 partial planes of token row t straight into the inbox of the rank owning t
//         (rows are dealt to ranks in blocks of `rows_per_rank`), plain st.global over NVLink;
//   finish (row_parallel_finish_kernel below):
//     1. signal: the GEMM before this kernel has completed, so this rank's pushes have landed ->
//        store `epoch` into flags[phase 1][my rank] of every peer (release, system scope);
//     2. wait (bounded) until every rank's phase-1 flag reached `epoch`;
//     3. reduce this rank's rows from its OWN inbox (every source rank x split plane: local
//        reads), round to bf16 (as a bf16 GEMM output would be), add the residual and apply
//        RMSNorm -- a row is spread over a cluster of CTAs whose sums of squares meet in
//        distributed shared memory;
//     4. all-gather by push: each finished row (normalised output and new residual) is stored into
//        every rank's out / res buffers;
//     5. the last CTA of the rank signals phase 2 to every peer and waits (bounded) for all of
//        them, so when the kernel ends every rank holds all rows.
// Nothing crosses NVLink as a load: the reduce-scatter half travels as the GEMM's stores, the
// all-gather half as this kernel's stores, and each rank only ever polls its own flag words.
// `epoch` lives in device memory and is advanced by the kernel itself, so the launch can be
// captured in a CUDA graph.  Every wait gives up after a bounded number of polls (kSpinLimit unless
// lowered for a test), records kTimeoutPeerFlag in the status word and lets the kernel finish.
//
// One inbox suffices: a rank writes a peer's inbox for call k+1 only after it passed phase 2 of
// call k, i.e. after that peer had reduced (and pushed) everything of call k.
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
constexpr int kArgFlags = 64;     // first argmax flag word
constexpr int kArgSlotsOff = 1024;        // byte offset of the argmax slots in the control block
constexpr int kArgMaxRows = 512;          // rows per argmax exchange

struct PeerPtrs {
  bf16* out[kMaxRanks];
  bf16* res[kMaxRanks];
  uint32_t* flags[kMaxRanks];     // control block of every rank
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
    row_parallel_finish_kernel(PeerPtrs peers, const float* __restrict__ inbox, const bf16* __restrict__ res_in,
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

  // 1. phase-1 signal: our GEMM (the previous kernel) has completed, its inbox stores are done
  if (first_cta && threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(peers.flags[threadIdx.x] + rank, epoch);
  }
  // 2. wait for every rank's partials to have landed in our inbox
  if (threadIdx.x == 0) wait_flags(my_flags, W, epoch, status);
  __syncthreads();

  // 3. local reduce + residual + RMSNorm for row `row` of this rank
  const int row = rank * rows_per_rank + row_slot;
  const bool have_row = row_slot < rows_per_rank && row < T;
  const int cols = N / kCluster;                // columns of this CTA (multiple of 4)
  const int c0 = crank * cols;
  const size_t plane = (size_t)rows_per_rank * N;
  float ss = 0.f;
  constexpr int kMaxPer = 4;                    // float4 chunks per thread (N <= 8192 * 2)
  float4 val[kMaxPer];
#pragma unroll
  for (int k = 0; k < kMaxPer; ++k) {
    const int col = c0 + (threadIdx.x + k * kThreads) * 4;
    val[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!have_row || col >= c0 + cols) continue;
    const float* src = inbox + (size_t)row_slot * N + col;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const int planes = W * S;
    int p = 0;
    // four independent loads in flight per step (the planes are local: HBM / L2 latency)
    for (; p + 4 <= planes; p += 4) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldcg(reinterpret_cast<const float4*>(src + (size_t)(p + u) * plane));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc.x += q[u].x; acc.y += q[u].y; acc.z += q[u].z; acc.w += q[u].w;
      }
    }
    for (; p < planes; ++p) {
      const float4 q = __ldcg(reinterpret_cast<const float4*>(src + (size_t)p * plane));
      acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
    }
    const size_t off = (size_t)row * N + col;
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
    const size_t off = (size_t)row * N + col;
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

// Greedy sampling under a vocab-parallel LM head, inside the decode graph: every rank holds the
// (max logit, local index) of its vocabulary shard per row; each rank stores its pairs into slot
// [parity][my rank][row] of every rank's control block, signals, waits for all W, and picks the
// largest value (ties: lowest global index, i.e. argmax over the concatenated shards).  Slots
// alternate with the epoch's parity, so a rank that runs ahead into the next call never
// overwrites pairs a slower peer is still reading.  One CTA.
__global__ void __launch_bounds__(512) vocab_argmax_exchange_kernel(const PeerPtrs peers, const float* __restrict__ vals,
                                                                    const int64_t* __restrict__ idx,
                                                                    int64_t vocab_start, int rows, int rank, int W,
                                                                    int64_t* __restrict__ out, int* status) {
  pdl_trigger();
  pdl_wait();
  __shared__ uint32_t s_epoch;
  uint32_t* my_flags = peers.flags[rank];
  if (threadIdx.x == 0) s_epoch = *((volatile uint32_t*)(my_flags + kArgFlags + W)) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const size_t par = (size_t)(epoch & 1u) * kMaxRanks * kArgMaxRows;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    uint2 v;
    v.x = __float_as_uint(vals[i]);
    v.y = (uint32_t)(idx[i] + vocab_start);
    for (int r = 0; r < W; ++r) {
      uint2* slots = reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(peers.flags[r]) + kArgSlotsOff);
      slots[par + (size_t)rank * kArgMaxRows + i] = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < W) st_release_sys(peers.flags[threadIdx.x] + kArgFlags + rank, epoch);
  if (threadIdx.x == 0) wait_flags(my_flags + kArgFlags, W, epoch, status);
  __syncthreads();
  const uint2* mine = reinterpret_cast<const uint2*>(reinterpret_cast<const uint8_t*>(my_flags) + kArgSlotsOff) + par;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    float best = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (int r = 0; r < W; ++r) {
      const uint2 v = __ldcv(&mine[(size_t)r * kArgMaxRows + i]);
      const float f = __uint_as_float(v.x);
      if (f > best || (f == best && v.y < bi)) {
        best = f;
        bi = v.y;
      }
    }
    out[i] = (int64_t)bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) *((volatile uint32_t*)(my_flags + kArgFlags + W)) = epoch;
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

// out/res/flags: W base addresses each (this rank's mapping of every rank's buffers); inbox: this
// rank's inbox [W][S][rows_per_rank][N] (local).
void row_parallel_finish(std::vector<int64_t> out, std::vector<int64_t> res, std::vector<int64_t> flags,
                         int64_t inbox, at::Tensor res_in, at::Tensor w, int64_t rank, int64_t S, int64_t T, int64_t N,
                         int64_t rows_per_rank, double eps, at::Tensor status) {
  const int W = out.size();
  LSB_CHECK(W >= 1 && W <= kMaxRanks && res.size() == (size_t)W && flags.size() == (size_t)W,
            "peer pointer lists must have one entry per rank (<= 8)");
  LSB_CHECK(N % (kCluster * 4) == 0 && N / kCluster <= 4 * 4 * kThreads, "hidden size unsupported by the fused path");
  LSB_CHECK(res_in.scalar_type() == at::kBFloat16 && res_in.is_contiguous() && res_in.numel() >= T * N, "bad residual");
  LSB_CHECK(rows_per_rank >= 1 && rows_per_rank * W >= T && S >= 1, "bad row layout");
  PeerPtrs p = {};
  for (int r = 0; r < W; ++r) {
    p.out[r] = reinterpret_cast<bf16*>(out[r]);
    p.res[r] = reinterpret_cast<bf16*>(res[r]);
    p.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  dim3 grid(kCluster, (unsigned)rows_per_rank);
  const at::cuda::CUDAGuard g(res_in.device());
  launch_pdl(row_parallel_finish_kernel, grid, dim3(kThreads), 0, at::cuda::getCurrentCUDAStream(), p,
             reinterpret_cast<const float*>(inbox), (const bf16*)res_in.data_ptr(), (const bf16*)w.data_ptr(),
             (int)rank, W, (int)S, (int)T, (int)N, (float)eps, (int)rows_per_rank, status_ptr(status));
  auto e = cudaGetLastError();
  LSB_CHECK(e == cudaSuccess, std::string("fused row-parallel finish launch failed: ") + cudaGetErrorString(e));
}

// Global greedy token per row from every rank's (max, local index) of its vocabulary shard.
// flags: every rank's control block (this rank's mapping); out: int64 [rows] on this rank.
void vocab_argmax_exchange(std::vector<int64_t> flags, at::Tensor vals, at::Tensor idx, int64_t vocab_start,
                           at::Tensor out, int64_t rank, at::Tensor status) {
  const int W = flags.size();
  const int rows = vals.numel();
  LSB_CHECK(W >= 1 && W <= kMaxRanks && rank >= 0 && rank < W, "one control block per rank (<= 8)");
  LSB_CHECK(rows <= kArgMaxRows, "at most 512 rows per argmax exchange");
  LSB_CHECK(vals.scalar_type() == at::kFloat && idx.scalar_type() == at::kLong && out.scalar_type() == at::kLong &&
                vals.is_contiguous() && idx.is_contiguous() && out.is_contiguous() && idx.numel() == rows &&
                out.numel() == rows, "vals float32 [rows], idx / out int64 [rows]");
  if (rows == 0) return;
  PeerPtrs p = {};
  for (int r = 0; r < W; ++r) p.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  const at::cuda::CUDAGuard g(vals.device());
  launch_pdl(vocab_argmax_exchange_kernel, dim3(1), dim3(512), 0, at::cuda::getCurrentCUDAStream(), p,
             vals.data_ptr<float>(), idx.data_ptr<int64_t>(), vocab_start, rows, (int)rank, W,
             out.data_ptr<int64_t>(), status_ptr(status));
  auto e = cudaGetLastError();
  LSB_CHECK(e == cudaSuccess, std::string("argmax exchange launch failed: ") + cudaGetErrorString(e));
}

int64_t comm_control_bytes() { return kArgSlotsOff + 2 * kMaxRanks * kArgMaxRows * 8; }

}  // namespace lsb
