// In-kernel tensor-parallel collectives over NVLink peer memory.
//
// Symmetric buffer of one rank (allocated per rank, mapped by every peer through CUDA IPC):
//   [0, kCtrlBytes)   control: epoch / CTA-counter words, argmax flag words and exchange slots
//   out   bf16 [max_tokens, N]   normalised rows of the last row-parallel layer (written locally)
//   res   bf16 [max_tokens, N]   residual rows of the last row-parallel layer (written locally)
//   ag    u64  [max_tokens, N]   all-gather inbox: (out, res) bf16 pairs of rows owned by peers
//   inbox u64  [W][S][rows][N]   reduce inbox: fp32 split-K partials of this rank's rows, from every rank
// Control words: [0] collective epoch, [1] CTA counter, [64, 64 + W) argmax arrivals, [64 + W]
// argmax epoch.
//
// Every inbox entry is a low-latency word (common.cuh): 4 bytes of payload and the epoch of the call
// that wrote it, stored as one 64-bit store.  A row-parallel projection (o_proj / down_proj) of
// call e finishes in two kernels and crosses NVLink only as stores:
//   GEMM  (gemm_sm100.cu / awq_sm100.cu, PartDest with one inbox per rank): the epilogue stores the
//         fp32 partials of token row t, tagged e, into the inbox of the rank owning t (rows are dealt
//         to ranks in blocks of `rows_per_rank`);
//   finish (row_parallel_finish_kernel below), one CTA cluster per token row:
//     * a row this rank owns: poll the W x S inbox words of each column until they carry epoch e,
//       sum them, round to bf16 (as a bf16 GEMM output would be), add the residual, RMSNorm (the
//       row's sum of squares meets in distributed shared memory), write out / res locally and store
//       (out, res) words tagged e into every peer's all-gather inbox;
//     * a row a peer owns: poll this rank's all-gather inbox for the row's words tagged e and unpack
//       them into out / res.
// No fence, no flag and no barrier round: a word with the expected epoch carries its data.  The
// epoch lives in device memory; the last CTA of the finish kernel advances it, so the launches can
// be captured in a CUDA graph.  Every poll gives up after a bounded number of attempts (kSpinLimit
// unless lowered for a test), records kTimeoutPeerFlag in the status word and lets the kernel finish.
//
// Single inboxes suffice: rank A stores call e+1 partials into B's reduce inbox only after A's finish
// kernel of call e received B's rows, which B pushed after reading its whole inbox of call e; and B
// pushes call e+1 rows into A's all-gather inbox only after reading A's call e+1 partials, which A's
// GEMM e+1 wrote after A's finish e had unpacked everything of call e.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cooperative_groups.h>

#include <mutex>
#include <unordered_map>

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
  uint32_t* flags[kMaxRanks];     // control block of every rank (argmax exchange)
};
struct PeerAg {
  uint64_t* ag[kMaxRanks];        // all-gather inbox of every rank (this rank's mappings)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Polls before a wait gives up (kSpinLimit unless lowered by comm_set_spin_limit, which the
// failure-detection test uses to make a wait on a peer that never writes end in milliseconds).
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

// The four words p[0..3] once all carry `epoch` (bounded; `live` turns false after a timeout, so
// one missing peer costs one spin limit per thread, not one per word).
__device__ __forceinline__ void ll_wait4(const uint64_t* p, uint32_t epoch, uint32_t limit, bool& live, int* status,
                                         uint64_t* w) {
  uint32_t i = 0;
  while (true) {
    ll_load2(p, w[0], w[1]);
    ll_load2(p + 2, w[2], w[3]);
    if ((uint32_t)(w[0] >> 32) == epoch && (uint32_t)(w[1] >> 32) == epoch && (uint32_t)(w[2] >> 32) == epoch &&
        (uint32_t)(w[3] >> 32) == epoch)
      return;
    if (!live || ++i > limit) {
      if (live) record_error(status, kTimeoutPeerFlag);
      live = false;
      return;
    }
  }
}

constexpr int kEpochWord = 0, kCounterWord = 1;
constexpr int kMaxPer = 4;       // 4-column chunks per thread: N / kCluster <= kMaxPer * 4 * kThreads

// grid (kCluster, G <= T): the kCluster CTAs of a cluster handle rows y, y + G, ... of this rank's
// rows, then of the peers' rows, N / kCluster columns each.
// phases: 1 = rows this rank owns (reduce, norm, push), 2 = rows peers own (receive); the engine
// runs both in one launch (3); a single-GPU test runs every emulated rank's phase 1 before any
// phase 2, so no launch waits on a later one.
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    row_parallel_finish_kernel(const PeerAg peers, const uint64_t* __restrict__ inbox, uint32_t* __restrict__ ctrl,
                               bf16* __restrict__ out, bf16* __restrict__ res_out, const bf16* __restrict__ res_in,
                               const bf16* __restrict__ w, int rank, int W, int S, int T, int N, float eps,
                               int rows_per_rank, int phases, int* status) {
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float red[kThreads / 32];
  __shared__ float cta_ss;
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = ld_volatile_u32(ctrl + kEpochWord) + 1u;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const uint32_t limit = *((volatile uint32_t*)&g_flag_spin_limit);
  const int crank = (int)cluster.block_rank();
  const int cols = N / kCluster;                // columns of this CTA (multiple of 4)
  const int c0 = crank * cols;
  bool live = true;

  // Rows are dealt to the gridDim.y clusters (all co-resident: the host caps the grid at the
  // device's active-cluster capacity).  Every cluster first finishes the rows this rank owns, which
  // wait only for the GEMMs' words, then receives the peers' rows -- so no cluster waits on work of
  // a cluster that cannot run.
  const int own_lo = min(T, rank * rows_per_rank), own_hi = min(T, (rank + 1) * rows_per_rank);
  if (phases & 1) {
    for (int t = own_lo + (int)blockIdx.y; t < own_hi; t += gridDim.y) {
      const int r = t - own_lo;
      // reduce this rank's row t from its inbox, add the residual, RMSNorm, push (out, res) to peers
      const size_t plane = (size_t)rows_per_rank * N;
      float ss = 0.f;
      float4 val[kMaxPer];
#pragma unroll
      for (int k = 0; k < kMaxPer; ++k) {
        const int col = c0 + (threadIdx.x + k * kThreads) * 4;
        val[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (col >= c0 + cols) continue;
        const uint64_t* src = inbox + (size_t)r * N + col;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < W * S; ++p) {
          uint64_t wv[4];
          ll_wait4(src + (size_t)p * plane, epoch, limit, live, status, wv);
          acc.x += __uint_as_float((uint32_t)wv[0]);
          acc.y += __uint_as_float((uint32_t)wv[1]);
          acc.z += __uint_as_float((uint32_t)wv[2]);
          acc.w += __uint_as_float((uint32_t)wv[3]);
        }
        const size_t off = (size_t)t * N + col;
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
        float a = 0.f;
        for (int i = 0; i < kThreads / 32; ++i) a += red[i];
        cta_ss = a;
      }
      cluster.sync();
      float total = 0.f;
      for (int c = 0; c < kCluster; ++c) total += *cluster.map_shared_rank(&cta_ss, c);
      cluster.sync();   // peers' shared memory must stay valid until everyone has read it
      const float inv = rsqrtf(total / N + eps);
#pragma unroll
      for (int k = 0; k < kMaxPer; ++k) {
        const int col = c0 + (threadIdx.x + k * kThreads) * 4;
        if (col >= c0 + cols) continue;
        const size_t off = (size_t)t * N + col;
        const uint2 wr = *reinterpret_cast<const uint2*>(w + col);
        const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wr.x);
        const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wr.y);
        const float v[4] = {val[k].x, val[k].y, val[k].z, val[k].w};
        const float wv[4] = {__low2float(w01), __high2float(w01), __low2float(w23), __high2float(w23)};
        bf16 ob[4], sb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ob[j] = to_b(to_f(to_b(v[j] * inv)) * wv[j]);
          sb[j] = to_b(v[j]);
        }
        *reinterpret_cast<uint2*>(out + off) = *reinterpret_cast<const uint2*>(ob);
        *reinterpret_cast<uint2*>(res_out + off) = *reinterpret_cast<const uint2*>(sb);
        uint64_t word[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t pair = (uint32_t)__bfloat16_as_ushort(ob[j]) | ((uint32_t)__bfloat16_as_ushort(sb[j]) << 16);
          word[j] = ll_word(pair, epoch);
        }
        for (int q = 0; q < W; ++q) {
          if (q == rank) continue;
          uint64_t* dst = peers.ag[q] + off;
          ll_store2(dst, word[0], word[1]);
          ll_store2(dst + 2, word[2], word[3]);
        }
      }
    }
  }
  if (phases & 2) {
    const int others = T - (own_hi - own_lo);
    for (int i = (int)blockIdx.y; i < others; i += gridDim.y) {
      const int t = i < own_lo ? i : i + (own_hi - own_lo);
      // receive row t from its owner
#pragma unroll
      for (int k = 0; k < kMaxPer; ++k) {
        const int col = c0 + (threadIdx.x + k * kThreads) * 4;
        if (col >= c0 + cols) continue;
        const size_t off = (size_t)t * N + col;
        uint64_t wv[4];
        ll_wait4(peers.ag[rank] + off, epoch, limit, live, status, wv);
        uint16_t ob[4], sb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ob[j] = (uint16_t)(wv[j] & 0xffffu);
          sb[j] = (uint16_t)((wv[j] >> 16) & 0xffffu);
        }
        *reinterpret_cast<uint2*>(out + off) = *reinterpret_cast<const uint2*>(ob);
        *reinterpret_cast<uint2*>(res_out + off) = *reinterpret_cast<const uint2*>(sb);
      }
    }
  }
  // the launch that completes the call advances the epoch once every CTA has read it
  if (phases & 2) {
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t total_ctas = gridDim.x * gridDim.y;
      if (atomicAdd(ctrl + kCounterWord, 1u) == total_ctas - 1) {
        ctrl[kCounterWord] = 0u;
        *((volatile uint32_t*)(ctrl + kEpochWord)) = epoch;
      }
    }
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

namespace {
// Clusters of the finishing kernel that can be resident at once on the current device (every one
// of them must be, since clusters wait on each other's rows across GPUs); cached per device.
int64_t finish_cluster_capacity() {
  static std::mutex mu;
  static std::unordered_map<int, int64_t> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCluster, 1024);
  cfg.blockDim = dim3(kThreads);
  int n = 0;
  auto e = cudaOccupancyMaxActiveClusters(&n, row_parallel_finish_kernel, &cfg);
  LSB_CHECK(e == cudaSuccess && n > 0, std::string("cluster occupancy query failed: ") + cudaGetErrorString(e));
  const int64_t cap = std::max<int64_t>(1, n / 2);   // half: room for the kernels PDL overlaps with it
  cache.emplace(dev, cap);
  return cap;
}
}  // namespace

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

// ag: every rank's all-gather inbox (this rank's mappings); inbox: this rank's reduce inbox
// [W][S][rows_per_rank][N] (local); ctrl: this rank's control block; out / res_out: this rank's local
// [T, N] outputs.  phases: 3 in the engine (see the kernel).
void row_parallel_finish(std::vector<int64_t> ag, int64_t inbox, int64_t ctrl, int64_t out, int64_t res_out,
                         at::Tensor res_in, at::Tensor w, int64_t rank, int64_t S, int64_t T, int64_t N,
                         int64_t rows_per_rank, double eps, int64_t phases, at::Tensor status) {
  const int W = ag.size();
  LSB_CHECK(W >= 1 && W <= kMaxRanks && rank >= 0 && rank < W, "one all-gather inbox per rank (<= 8)");
  LSB_CHECK(N % (kCluster * 4) == 0 && N / kCluster <= kMaxPer * 4 * kThreads, "hidden size unsupported by the fused path");
  LSB_CHECK(res_in.scalar_type() == at::kBFloat16 && res_in.is_contiguous() && res_in.numel() >= T * N, "bad residual");
  LSB_CHECK(w.scalar_type() == at::kBFloat16 && w.numel() == N, "bad norm weight");
  LSB_CHECK(rows_per_rank >= 1 && rows_per_rank * W >= T && S >= 1 && phases >= 1 && phases <= 3, "bad row layout");
  if (T == 0) return;
  PeerAg p = {};
  for (int r = 0; r < W; ++r) p.ag[r] = reinterpret_cast<uint64_t*>(ag[r]);
  const at::cuda::CUDAGuard g(res_in.device());
  dim3 grid(kCluster, (unsigned)std::min<int64_t>(T, finish_cluster_capacity()));
  launch_pdl(row_parallel_finish_kernel, grid, dim3(kThreads), 0, at::cuda::getCurrentCUDAStream(), p,
             reinterpret_cast<const uint64_t*>(inbox), reinterpret_cast<uint32_t*>(ctrl), reinterpret_cast<bf16*>(out),
             reinterpret_cast<bf16*>(res_out), (const bf16*)res_in.data_ptr(), (const bf16*)w.data_ptr(), (int)rank,
             W, (int)S, (int)T, (int)N, (float)eps, (int)rows_per_rank, (int)phases, status_ptr(status));
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
