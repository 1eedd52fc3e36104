// Shared device helpers for the llmserve_b200 sm_100a kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace lsb {

using bf16 = __nv_bfloat16;

// Error codes a kernel records in the process-wide status word instead of trapping.
enum ErrorCode : int {
  kOk = 0,
  kTimeoutTmaFull = 1,      // MMA issuer waited too long for a TMA stage
  kTimeoutSmemEmpty = 2,    // producer waited too long for a free stage
  kTimeoutAccum = 3,        // epilogue waited too long for the accumulator
  kTimeoutPeerFlag = 4,     // fused collective waited too long for a peer
  kBadIndex = 5,            // a slot / block index outside the pool was skipped
};

// Spin limit of every bounded wait: ~2^26 polls is seconds on a B200, far above any
// legitimate wait, and still ends a wait on a flag that is never set.
constexpr uint32_t kSpinLimit = 1u << 26;

// ---- low-latency words for the tensor-parallel collective ------------------------------------------
// A 64-bit word whose low half is 4 bytes of payload and whose high half is the epoch (call number)
// of the collective that wrote it.  An aligned 64-bit store is single-copy atomic, so a reader that
// sees the expected epoch also sees that call's payload: peers poll the data itself, with no fence
// and no separate flag.
__device__ __forceinline__ uint64_t ll_word(uint32_t payload, uint32_t epoch) {
  return ((uint64_t)epoch << 32) | payload;
}
__device__ __forceinline__ void ll_store2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ll_store1(uint64_t* p, uint64_t a) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ void ll_load2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Where a GEMM writes its fp32 split-K partial planes.  Off tensor parallelism there is one owner
// (the local [planes, T, N] fp32 buffer).  Under tensor parallelism the token rows are dealt to
// the ranks in blocks of `rows` (rank o owns rows [o*rows, (o+1)*rows)) and base[o] is rank o's
// inbox (a peer pointer for o != this rank) of 64-bit low-latency words
// [source rank][plane][row][N], this rank writing the source-rank slot `slot`, each word carrying
// the value and the call's epoch (the word at `epoch` plus one).  The owner polls its own memory
// for the words of the current epoch and reduces them, so the row-parallel reduction crosses NVLink
// as stores made by the GEMM epilogue, never as loads, and needs no fence or flag.
constexpr int kMaxOwners = 8;
struct PartDest {
  float* base[kMaxOwners];
  int rows;      // token rows per owner (T with one owner)
  int slot;      // this rank's source slot in every owner's inbox (0 with one owner)
  int planes;    // split-K planes per source (the GEMM's gridDim.z)
  int owners;    // 1, or the tensor-parallel size
  int ll;        // 1: the collective's inboxes (epoch-tagged words), whatever the number of owners
  const uint32_t* epoch;   // ll: this rank's epoch word of the collective
  __device__ __forceinline__ uint32_t call_epoch() const { return ll ? ld_volatile_u32(epoch) + 1u : 0u; }
  __device__ __forceinline__ float* at(int z, int t, int N, int feat) const {   // local planes (ll == 0)
    return base[0] + ((size_t)z * rows + t) * N + feat;
  }
  __device__ __forceinline__ uint64_t* ll_at(int z, int t, int N, int feat) const {
    const int o = t / rows, r = t - o * rows;
    float* b = base[0];
#pragma unroll
    for (int i = 1; i < kMaxOwners; ++i)   // select without indexing the parameter array dynamically
      if (i == o) b = base[i];
    return reinterpret_cast<uint64_t*>(b) + ((size_t)(slot * planes + z) * rows + r) * N + feat;
  }
  // one value of plane z, token row t, feature feat
  __device__ __forceinline__ void store(int z, int t, int N, int feat, float v, uint32_t e) const {
    if (!ll) *at(z, t, N, feat) = v;
    else ll_store1(ll_at(z, t, N, feat), ll_word(__float_as_uint(v), e));
  }
  // four consecutive features feat..feat+3 (feat % 4 == 0, N % 4 == 0)
  __device__ __forceinline__ void store4(int z, int t, int N, int feat, const float* v, uint32_t e) const {
    if (!ll) {
      float* p = at(z, t, N, feat);
#pragma unroll
      for (int q = 0; q < 4; ++q) p[q] = v[q];
    } else {
      uint64_t* p = ll_at(z, t, N, feat);
      ll_store2(p, ll_word(__float_as_uint(v[0]), e), ll_word(__float_as_uint(v[1]), e));
      ll_store2(p + 2, ll_word(__float_as_uint(v[2]), e), ll_word(__float_as_uint(v[3]), e));
    }
  }
};

inline PartDest local_part_dest(float* partials, int T, int planes) {
  PartDest d = {};
  d.base[0] = partials;
  d.rows = T > 0 ? T : 1;
  d.slot = 0;
  d.planes = planes;
  d.owners = 1;
  d.ll = 0;
  d.epoch = nullptr;
  return d;
}

__device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 to_b(float v) { return __float2bfloat16(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `scratch` holds >= 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? scratch[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with `parity` to complete; false after kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- cp.async (Ampere-style, used by the attention kernels) ---------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int bytes = pred ? 16 : 0;   // src-size 0 -> zero fill
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// ---- programmatic dependent launch ------------------------------------------------------------
// Kernels of the serving path are launched with the programmatic-stream-serialization attribute:
// the next kernel may start while this one drains.  Each kernel therefore (1) lets its dependent
// launch early and (2) waits for its predecessor's completion (and memory) before touching any
// global memory that a predecessor may write -- work before the wait is limited to shared memory
// set-up and reads of data no kernel writes (weights, tensor maps).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) applies to the CURRENT device only: one process
// that drives several GPUs (prefill/decode disaggregation, tests) must set it on each of them.
// Sets it for the current device the first time `bytes` exceeds what was set there.
void ensure_dynamic_smem(const void* func, int bytes);

// cudaLaunchKernelEx with the PDL attribute (when enabled).
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace lsb
