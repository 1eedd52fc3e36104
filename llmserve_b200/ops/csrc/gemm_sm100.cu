// bf16 GEMM on the 5th-generation tensor cores: Y[T, N] = X[T, K] . W[N, K]^T.
//
// One CTA computes a 128 (weight rows) x BN (tokens) output tile over a K range:
//   warp 0, one lane : TMA producer, streams 128x64 W and BNx64 X tiles (128B swizzle) into a
//                      STAGES-deep shared-memory ring (mbarrier "full" with tx-count);
//   warp 1, one lane : MMA issuer, four tcgen05.mma (K=16 each) per stage into a TMEM
//                      accumulator, tcgen05.commit frees the stage ("empty") when its MMAs are done;
//   all 4 warps      : epilogue, tcgen05.ld 32 lanes x 16 columns at a time (warp w owns TMEM
//                      lanes 32w..32w+31 = output features), store bf16 (or fp32 split-K partials)
//                      with the feature index contiguous across the warp.
// The weight matrix is the UMMA "A" (M = 128 rows) and the tokens are "B" (N = BN), so a decode
// batch of a few dozen tokens still fills the tensor core's M dimension and the weights -- the
// bytes that bound decode -- are read once.  K is split over gridDim.z when the tile grid alone
// would leave SMs idle; the caller then reduces the fp32 partials (fused with the next op).
//
// Every mbarrier wait is bounded; a timeout records an error code in `status`, stops issuing
// work, waits (bounded) for the TMA copies already in flight, frees TMEM and returns.
// Every CTA issues its own TMA loads from this GPU's memory (the kernel runs under tensor parallelism).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <map>
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lsb {
namespace {

#define LSB_CHECK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

constexpr int BM = 128;
constexpr int BK = 64;   // 64 bf16 = 128 bytes: one 128B swizzle atom per row
constexpr int kSmemBudget = 200 * 1024;
constexpr int kGroupT = 8;   // token tiles per raster group
constexpr int kMaxClusterSplits = 16;   // K splits reduced in one (non-portable) cluster

// ---- descriptors --------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"), K-major, 128B swizzle:
// start address >> 4 in bits [0,14), leading-byte-offset (unused for swizzled K-major, 1) in
// [16,30), stride-byte-offset = 1024 B (8 rows x 128 B) >> 4 in [32,46), descriptor version 1 in
// [46,48), layout type 2 (128B swizzle) in [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor for kind::f16: fp32 accumulate (bits 4-5 = 1), A = B = bf16
// (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
template <int N>
__host__ __device__ constexpr uint32_t idesc_bf16_f32() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// ---- PTX wrappers ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kW = BM * BK * 2;           // 16 KiB
  static constexpr int kX = BN * BK * 2;
  static constexpr int kStage = kW + kX;           // multiple of 1024
  static constexpr int kBarOff = STAGES * kStage;
  static constexpr int kBytes = kBarOff + (2 * STAGES + 1) * 8 + 16 + 1024;   // + alignment slack
};

template <int BN>
constexpr int tmem_cols() {
  return BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
}

// EPI 0: bf16 output [T, N] or fp32 split-K partials; EPI 1: SiLU-mul of an interleaved gate/up
// weight (rows 128i..128i+63 gate, +64..+127 up) -> bf16 [T, N/2].
//
// cluster_red > 0: the gridDim.z = cluster_red K-split CTAs of one output tile form a thread-block
// cluster (1, 1, cluster_red) and reduce their accumulators on chip: each CTA parks its fp32 tile
// [BN tokens][128 features] in its own (now idle) stage memory, the cluster synchronises, and CTA
// z sums slice z of the tile over every CTA's copy through distributed shared memory, then writes
// the finished slice once -- bf16 output (or SiLU-mul for EPI 1), or ONE fp32 plane through `pd`
// (plane 0).  No partial plane touches HBM and, under tensor parallelism, only one plane per rank
// crosses NVLink.
template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(128, 1) gemm_bf16_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                           const __grid_constant__ CUtensorMap tm_x,
                                                           bf16* __restrict__ out, const PartDest pd,
                                                           int T, int N, int k_tiles, int k_tiles_per_split,
                                                           int packed, int cluster_red, int* __restrict__ status) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Tile order: blockIdx.x enumerates (weight tile, token tile) pairs in groups of kGroupT token
  // tiles, token tile fastest, so the CTAs resident at one time cover a ~18 x 8 block of the
  // output and re-read W and X from L2 rather than HBM.  With one token tile (decode) this is
  // the plain weight-tile order.
  const int num_m = (N + BM - 1) / BM, num_t = (T + BN - 1) / BN;
  const int per_group = kGroupT * num_m;
  const int grp = blockIdx.x / per_group, rem = blockIdx.x - grp * per_group;
  const int first_t = grp * kGroupT;
  const int gsz = min(num_t - first_t, kGroupT);
  const int m_tile = rem / gsz, t_tile = first_t + rem % gsz;
  const int n0 = m_tile * BM, t0 = t_tile * BN;
  const int kt_begin = blockIdx.z * k_tiles_per_split;
  // W tile coordinates: row-major [N, K] (tensor map with 128B swizzle), or the packed layout in
  // which tile (m, kt) is 128 consecutive pre-swizzled 128-byte rows (one contiguous 16 KiB run).
  auto w_x = [&](int kt) { return packed ? 0 : kt * BK; };
  auto w_y = [&](int kt) { return packed ? (m_tile * k_tiles + kt) * BM : n0; };
  const int kt_end = min(k_tiles, kt_begin + k_tiles_per_split);
  const int nk = max(0, kt_end - kt_begin);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols<BN>()));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  if (warp == 0) {
    if (lane == 0) {
      // Weights never depend on the previous kernel: stream the first stages of W before waiting
      // for the predecessor (programmatic dependent launch), then the activations.
      const int pre = nk < STAGES ? nk : STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], L::kStage);
        tma_load_2d(smem + i * L::kStage, &tm_w, &full[i], w_x(kt_begin + i), w_y(kt_begin + i));
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + i * L::kStage + L::kW, &tm_x, &full[i], (kt_begin + i) * BK, t0);
      int issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = s < pre ? s + 1 : 0;
      for (int i = pre; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t phase = (i / STAGES) & 1;
        if (!mbar_wait(&empty[s], phase ^ 1)) {
          record_error(status, kTimeoutSmemEmpty);
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*((volatile int*)&abort_flag)) break;
        uint8_t* st = smem + s * L::kStage;
        mbar_expect_tx(&full[s], L::kStage);
        const int kx = (kt_begin + i) * BK;
        tma_load_2d(st, &tm_w, &full[s], w_x(kt_begin + i), w_y(kt_begin + i));
        tma_load_2d(st + L::kW, &tm_x, &full[s], kx, t0);
        issued[s] = i + 1;
      }
      if (*((volatile int*)&abort_flag)) {
        // drain: wait (bounded) for every stage's most recent copy to land before leaving
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] > 0) mbar_wait(&full[s], ((issued[s] - 1) / STAGES) & 1);
      }
    } else {
      pdl_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && nk > 0) {
      constexpr uint32_t idesc = idesc_bf16_f32<BN>();
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t phase = (i / STAGES) & 1;
        if (!mbar_wait(&full[s], phase) || *((volatile int*)&abort_flag)) {
          record_error(status, kTimeoutTmaFull);
          atomicExch(&abort_flag, 1);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t wa = smem_u32(smem + s * L::kStage);
        const uint32_t xa = wa + L::kW;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma(tmem, smem_desc_sw128(wa + k * 32), smem_desc_sw128(xa + k * 32), idesc, (i | k) != 0);
        tc_commit(&empty[s]);
      }
      if (ok) tc_commit(accum);
    }
    __syncwarp();
  } else {
    pdl_wait();
  }

  // ---- epilogue ---------------------------------------------------------------------------------
  bool have = nk > 0;
  if (have) {
    if (!mbar_wait(accum, 0) || *((volatile int*)&abort_flag)) {
      record_error(status, kTimeoutAccum);
      have = false;
    }
  }
  tc_fence_after();
  // the collective's epoch of this call (0 off tensor parallelism); every thread waited for the
  // predecessor above, so the word is the previous call's final value
  const uint32_t ep = pd.call_epoch();
  const int feat = n0 + warp * 32 + lane;
  const uint32_t row_addr = tmem + ((uint32_t)(warp * 32) << 16);
  if (cluster_red > 0) {
    static_assert(BN * BM * 4 <= STAGES * L::kStage, "reduction tile must fit in the stage memory");
    cg::cluster_group cluster = cg::this_cluster();
    float* red = reinterpret_cast<float*>(smem);   // [BN][128] fp32; the stage buffers are idle now
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      if (have) {
        tc_ld16(row_addr + c0, r);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) red[(c0 + j) * BM + warp * 32 + lane] = __uint_as_float(r[j]);
    }
    cluster.sync();   // every K-slice of the tile is parked
    const int S = cluster_red;
    const int z = (int)cluster.block_rank();
    const int nvalid = max(0, min(BN, T - t0));
    // EPI 0: float4 groups (token j, features 4g..4g+3); EPI 1: (token j, gate/up pair group g < 16)
    constexpr int kGroups = EPI == 0 ? BM / 4 : BM / 8;
    const int E = nvalid * kGroups;
    const int per = (E + S - 1) / S;
    const int e_end = min(E, (z + 1) * per);
    for (int e = z * per + (int)threadIdx.x; e < e_end; e += 128) {
      const int j = e / kGroups, g = e - j * kGroups;
      const int t = t0 + j;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = make_float4(0.f, 0.f, 0.f, 0.f);
      // four distributed-shared-memory loads in flight per round (their latency, not the adds,
      // bounds this loop), then the sums in source order
      int src = 0;
      for (; src + 4 <= S; src += 4) {
        float4 x[4], y[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float* rs = cluster.map_shared_rank(red, src + u) + j * BM;
          x[u] = *reinterpret_cast<const float4*>(rs + g * 4);
          if constexpr (EPI == 1) y[u] = *reinterpret_cast<const float4*>(rs + BM / 2 + g * 4);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          a.x += x[u].x; a.y += x[u].y; a.z += x[u].z; a.w += x[u].w;
          if constexpr (EPI == 1) {
            b.x += y[u].x; b.y += y[u].y; b.z += y[u].z; b.w += y[u].w;
          }
        }
      }
      for (; src < S; ++src) {
        const float* rs = cluster.map_shared_rank(red, src) + j * BM;
        const float4 x = *reinterpret_cast<const float4*>(rs + g * 4);
        a.x += x.x; a.y += x.y; a.z += x.z; a.w += x.w;
        if constexpr (EPI == 1) {
          const float4 y = *reinterpret_cast<const float4*>(rs + BM / 2 + g * 4);
          b.x += y.x; b.y += y.y; b.z += y.z; b.w += y.w;
        }
      }
      const float va[4] = {a.x, a.y, a.z, a.w};
      if constexpr (EPI == 0) {
        const int f0 = n0 + g * 4;
        if (pd.base[0] != nullptr && (pd.ll || f0 + 3 < N)) {
          pd.store4(0, t, N, f0, va, ep);          // N % 4 == 0 for the collective's inboxes
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (f0 + q >= N) break;
            if (pd.base[0] != nullptr) *pd.at(0, t, N, f0 + q) = va[q];
            else out[(size_t)t * N + f0 + q] = to_b(va[q]);
          }
        }
      } else {
        const float vb[4] = {b.x, b.y, b.z, b.w};
        const int out_n = N / 2, c = m_tile * (BM / 2) + g * 4;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (c + q >= out_n) break;
          const float gt = to_f(to_b(va[q])), up = to_f(to_b(vb[q]));
          out[(size_t)t * out_n + c + q] = to_b(gt / (1.f + expf(-gt)) * up);
        }
      }
    }
    cluster.sync();   // keep this CTA's tile alive until every peer CTA has read it
  } else if constexpr (EPI == 0) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      if (have) {
        tc_ld16(row_addr + c0, r);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
      if (feat < N) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = t0 + c0 + j;
          if (t < T) {
            const float v = __uint_as_float(r[j]);
            if (pd.base[0] != nullptr)
              pd.store(blockIdx.z, t, N, feat, v, ep);
            else
              out[(size_t)t * N + feat] = to_b(v);
          }
        }
      }
    }
  } else {
    // warps 2-3 hold the up rows: hand them to warps 0-1 (same row offset) through shared memory
    float* xch = reinterpret_cast<float*>(smem);            // stage buffers are free now
    const int half_row = (warp & 1) * 32 + lane;             // 0..63
    const int out_n = N / 2;
    const int out_col = m_tile * (BM / 2) + half_row;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      if (have) {
        tc_ld16(row_addr + c0, r);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
      if (warp >= 2) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xch[half_row * 17 + j] = __uint_as_float(r[j]);
      }
      __syncthreads();
      if (warp < 2 && out_col < out_n) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = t0 + c0 + j;
          if (t < T) {
            const float g = to_f(to_b(__uint_as_float(r[j])));
            const float u = to_f(to_b(xch[half_row * 17 + j]));
            out[(size_t)t * out_n + out_col] = to_b(g / (1.f + expf(-g)) * u);
          }
        }
      }
      __syncthreads();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols<BN>()));
  }
}

// ---- host side ---------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  LSB_CHECK(fn != nullptr, "cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with a (box_rows x 64) box.
CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int64_t row_stride_elems, int box_rows,
                     bool swizzle = true) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LSB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

struct MapKey {
  const void* p;
  int64_t rows, cols, stride;
  int box;
  bool packed;
  bool operator==(const MapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && stride == o.stride && box == o.box && packed == o.packed;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (std::hash<int64_t>()(k.rows) * 31) ^ (std::hash<int64_t>()(k.cols) * 131) ^
           (size_t)k.box;
  }
};

}  // namespace

// Weight maps are built once per (pointer, shape); activations change every call.  A packed
// weight is a [rows, 64] bf16 tensor already in the swizzled shared-memory image, so its map
// copies 128 x 64 boxes without swizzling.
const CUtensorMap& weight_map(const at::Tensor& w, bool packed) {
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  static std::mutex mu;
  MapKey key{w.data_ptr(), w.size(0), w.size(1), w.stride(0), BM, packed};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it == cache.end())
    it = cache.emplace(key, make_map(w.data_ptr(), w.size(0), w.size(1), w.stride(0), BM, !packed)).first;
  return it->second;
}

namespace {

// Cluster sizes above 8 need the non-portable opt-in, per kernel and device.
void allow_large_clusters(const void* func) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, bool> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  bool& d = done[{func, dev}];
  if (!d) {
    cudaFuncSetAttribute(func, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    d = true;
  }
}

// reduce: the `splits` K-slices of a tile reduce in a cluster (splits <= kMaxClusterSplits) and
// write bf16 `out` (or SiLU-mul) / one fp32 plane through `pd`; otherwise every slice writes its
// own fp32 plane through `pd` (or bf16 `out` when splits == 1).
template <int BN, int STAGES, int EPI = 0>
void launch(const at::Tensor& x, const at::Tensor& w, int N, bool packed, bf16* out, const PartDest& pd, int splits,
            int* status, bool reduce = false) {
  using L = GemmSmem<BN, STAGES>;
  static_assert(L::kStage % 1024 == 0, "stage size must keep 1024-byte alignment");
  const int T = x.size(0), K = x.size(1);
  const int k_tiles = (K + BK - 1) / BK;
  const int kps = (k_tiles + splits - 1) / splits;
  const CUtensorMap mx = make_map(x.data_ptr(), T, K, x.stride(0), BN);
  const CUtensorMap& mw = weight_map(w, packed);
  auto kern = gemm_bf16_kernel<BN, STAGES, EPI>;
  ensure_dynamic_smem((const void*)kern, L::kBytes);
  dim3 grid(((N + BM - 1) / BM) * ((T + BN - 1) / BN), 1, splits);
  const int cred = reduce && splits > 1 ? splits : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  int nattr = 1;
  if (cred > 0) {
    if (cred > 8) allow_large_clusters((const void*)kern);
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = cred;
    nattr = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  cudaLaunchKernelEx(&cfg, kern, mw, mx, out, pd, T, N, k_tiles, kps, (int)packed, cred, status);
}

template <int BN>
constexpr int stages_for() {
  constexpr int st = kSmemBudget / GemmSmem<BN, 1>::kStage;
  return st > 8 ? 8 : st;
}

}  // namespace

int* status_ptr(const at::Tensor& status);

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }

// 128B-swizzled map over activations x [T, K] with (box_rows x 64) boxes.
CUtensorMap activation_map(const at::Tensor& x, int box_rows) {
  return make_map(x.data_ptr(), x.size(0), x.size(1), x.stride(0), box_rows);
}


// Token counts from which the persistent 2-SM kernel replaces the one-SM tile kernel.
static int pair_min_tokens() {
  static int v = [] {
    const char* e = std::getenv("LLMSERVE_PAIR_GEMM_MIN_T");
    return e ? std::atoi(e) : 512;
  }();
  return v;
}

// SiLU-gated projection with an interleaved gate/up weight [N, K] (N = 2 * I, interleaved per 64
// rows): out = silu(gate) * up as bf16 [T, I], in the GEMM epilogue (no split-K).
static void gemm_silu_dispatch(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, bool packed, at::Tensor status,
                               int64_t max_stages, int64_t splits = 1) {
  LSB_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
            "gemm operands must be bf16 CUDA tensors");
  LSB_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1, "gemm shape mismatch");
  if (packed) {
    const int64_t kt = (x.size(1) + BK - 1) / BK, mt = (n + 255) / 256 * 2;
    LSB_CHECK(w.size(1) == BK && w.is_contiguous() && w.size(0) == mt * kt * BM, "packed weight shape mismatch");
  } else {
    LSB_CHECK(x.size(1) == w.size(1) && w.size(0) == n, "gemm shape mismatch");
  }
  LSB_CHECK(n % BM == 0, "interleaved gate/up weight must have a multiple of 128 rows");
  const int T = x.size(0), N = (int)n;
  LSB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)T * (N / 2),
            "bad out");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  bf16* o = (bf16*)out.data_ptr();
  int* st = status_ptr(status);
  const bool shallow = max_stages > 0 && max_stages <= 4;
  const PartDest nopd = local_part_dest(nullptr, T, 1);
  LSB_CHECK(splits >= 1 && splits <= kMaxClusterSplits, "SiLU GEMM splits must be 1..16 (cluster reduction)");
  const int sp = (int)splits;
#define LSB_SILU(BNV)                                                                  \
  do {                                                                                 \
    if (shallow) launch<BNV, 4, 1>(x, w, N, packed, o, nopd, sp, st, true);            \
    else launch<BNV, stages_for<BNV>(), 1>(x, w, N, packed, o, nopd, sp, st, true);    \
  } while (0)
  if (T <= 16) LSB_SILU(16);
  else if (T <= 32) LSB_SILU(32);
  else if (T <= 64) LSB_SILU(64);
  else if (T <= 128) launch<128, stages_for<128>(), 1>(x, w, N, packed, o, nopd, sp, st, true);
  else launch<256, stages_for<256>(), 1>(x, w, N, packed, o, nopd, sp, st, true);
#undef LSB_SILU
}

void gemm_bf16_silu(at::Tensor out, at::Tensor x, at::Tensor w, at::Tensor status, int64_t max_stages) {
  LSB_CHECK(w.dim() == 2, "gemm weight must be 2-D");
  gemm_silu_dispatch(out, x, w, w.size(0), false, status, max_stages);
}

// Same with the tile-packed image (gemm.pack_weight) of an interleaved gate/up weight of n rows.
void gemm_bf16_silu_packed(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, at::Tensor status,
                           int64_t max_stages) {
  gemm_silu_dispatch(out, x, w, n, true, status, max_stages);
}

// SiLU-gated projection with K split over `splits` CTAs that reduce in a cluster (no partials).
void gemm_bf16_silu_reduced(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, bool packed, int64_t splits,
                            at::Tensor status, int64_t max_stages) {
  gemm_silu_dispatch(out, x, w, n, packed, status, max_stages, splits);
}

void gemm_bf16_pair(void* out, bool out_f32, const at::Tensor& x, const at::Tensor& w, int N, bool packed, int* status);

// The one-SM tile kernel for T tokens: a shallow 4-stage ring (two CTAs per SM) for decode-sized
// T when asked, else the deepest ring that fits.
static void tile_dispatch(const at::Tensor& x, const at::Tensor& w, int n, bool packed, bf16* o, const PartDest& pd,
                          int splits, int* st, int64_t max_stages, bool reduce = false) {
  const int T = x.size(0);
  if (max_stages > 0 && max_stages <= 4 && T <= 64) {
    // shallow ring: two CTAs fit on one SM and overlap each other's prologue / epilogue
    if (T <= 16) launch<16, 4>(x, w, n, packed, o, pd, splits, st, reduce);
    else if (T <= 32) launch<32, 4>(x, w, n, packed, o, pd, splits, st, reduce);
    else launch<64, 4>(x, w, n, packed, o, pd, splits, st, reduce);
    return;
  }
  if (T <= 16) launch<16, stages_for<16>()>(x, w, n, packed, o, pd, splits, st, reduce);
  else if (T <= 32) launch<32, stages_for<32>()>(x, w, n, packed, o, pd, splits, st, reduce);
  else if (T <= 64) launch<64, stages_for<64>()>(x, w, n, packed, o, pd, splits, st, reduce);
  else if (T <= 128) launch<128, stages_for<128>()>(x, w, n, packed, o, pd, splits, st, reduce);
  else launch<256, stages_for<256>()>(x, w, n, packed, o, pd, splits, st, reduce);
}

static void check_gemm_operands(const at::Tensor& x, const at::Tensor& w, int64_t N, bool packed) {
  LSB_CHECK(x.is_cuda() && w.is_cuda(), "gemm operands must be CUDA tensors");
  LSB_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  LSB_CHECK(x.dim() == 2 && w.dim() == 2, "gemm operands must be 2-D");
  LSB_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "gemm operands must be K-contiguous");
  LSB_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
  LSB_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
            "gemm operands must be 16-byte aligned");
  if (packed) {
    const int64_t kt = (x.size(1) + BK - 1) / BK, mt = (N + 255) / 256 * 2;
    LSB_CHECK(w.size(1) == BK && w.is_contiguous() && w.size(0) == mt * kt * BM, "packed weight shape mismatch");
  } else {
    LSB_CHECK(x.size(1) == w.size(1) && w.size(0) == N, "gemm shape mismatch");
  }
}

// K split over `splits` CTAs (1..16) whose accumulators are reduced in a cluster: bf16 out [T, n]
// when `plane` is empty, else one fp32 plane [T, n].  T < 512 (the tile kernel's range).
void gemm_bf16_reduced(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, bool packed, at::Tensor plane,
                       int64_t splits, at::Tensor status, int64_t max_stages) {
  check_gemm_operands(x, w, n, packed);
  LSB_CHECK(splits >= 1 && splits <= kMaxClusterSplits, "cluster-reduced splits must be 1..16");
  const int T = x.size(0);
  bf16* o = nullptr;
  float* p = nullptr;
  if (plane.numel() == 0) {
    LSB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)T * n, "bad out");
    o = (bf16*)out.data_ptr();
  } else {
    LSB_CHECK(plane.scalar_type() == at::kFloat && plane.is_contiguous() && plane.numel() == (int64_t)T * n,
              "bad fp32 plane");
    p = plane.data_ptr<float>();
  }
  if (T == 0 || n == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  tile_dispatch(x, w, (int)n, packed, o, local_part_dest(p, T, 1), (int)splits, status_ptr(status), max_stages, true);
}

// Shared dispatch.  w: row-major [N, K], or (packed) the [rows, 64] pre-swizzled tile image of a
// weight with N logical rows (rows padded to 256, K to 64).
static void gemm_dispatch(at::Tensor out, at::Tensor x, at::Tensor w, int64_t N, bool packed, at::Tensor partials,
                          int64_t splits, at::Tensor status, int64_t max_stages) {
  LSB_CHECK(x.is_cuda() && w.is_cuda(), "gemm operands must be CUDA tensors");
  LSB_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  LSB_CHECK(x.dim() == 2 && w.dim() == 2, "gemm operands must be 2-D");
  LSB_CHECK(x.stride(1) == 1 && w.stride(1) == 1, "gemm operands must be K-contiguous");
  LSB_CHECK((x.stride(0) * 2) % 16 == 0 && (w.stride(0) * 2) % 16 == 0, "row strides must be 16-byte multiples");
  LSB_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
            "gemm operands must be 16-byte aligned");
  const int T = x.size(0);
  if (packed) {
    const int64_t kt = (x.size(1) + BK - 1) / BK, mt = (N + 255) / 256 * 2;
    LSB_CHECK(w.size(1) == BK && w.is_contiguous() && w.size(0) == mt * kt * BM, "packed weight shape mismatch");
  } else {
    LSB_CHECK(x.size(1) == w.size(1) && w.size(0) == N, "gemm shape mismatch");
  }
  LSB_CHECK(splits >= 1 && splits <= 64, "splits out of range");
  bf16* o = nullptr;
  float* p = nullptr;
  if (splits == 1 && partials.numel() == 0) {
    LSB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)T * N, "bad out");
    o = (bf16*)out.data_ptr();
  } else {
    LSB_CHECK(partials.scalar_type() == at::kFloat && partials.is_contiguous() &&
                  partials.numel() == splits * (int64_t)T * N, "bad partials");
    p = partials.data_ptr<float>();
  }
  if (T == 0 || N == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  int* st = status_ptr(status);
  const int n = (int)N;
  if (splits == 1 && T >= pair_min_tokens() && N % 8 == 0) {
    gemm_bf16_pair(o != nullptr ? (void*)o : (void*)p, o == nullptr, x, w, n, packed, st);
    return;
  }
  tile_dispatch(x, w, n, packed, o, local_part_dest(p, T, (int)splits), (int)splits, st, max_stages);
}

// Row-parallel projection under tensor parallelism: the fp32 partial planes of token row t go to
// the inbox of the rank owning t (inboxes[o], a peer pointer for o != rank; see PartDest), as
// plain stores from the epilogue (no TMA touches peer memory).  w: row-major [n, K], or (packed)
// the tile image of a weight with n logical rows.
void gemm_bf16_to_owners(at::Tensor x, at::Tensor w, int64_t n, bool packed, std::vector<int64_t> inboxes,
                         int64_t rank, int64_t rows_per_rank, int64_t splits, bool reduce, int64_t epoch_ptr,
                         at::Tensor status, int64_t max_stages) {
  LSB_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
            "gemm operands must be bf16 CUDA tensors");
  LSB_CHECK(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x must be K-contiguous and 16-byte aligned");
  LSB_CHECK(w.stride(1) == 1 && (w.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
            "w must be K-contiguous and 16-byte aligned");
  if (packed) {
    const int64_t kt = (x.size(1) + BK - 1) / BK, mt = (n + 255) / 256 * 2;
    LSB_CHECK(w.size(1) == BK && w.is_contiguous() && w.size(0) == mt * kt * BM, "packed weight shape mismatch");
  } else {
    LSB_CHECK(x.size(1) == w.size(1) && w.size(0) == n, "gemm shape mismatch");
  }
  const int W = (int)inboxes.size(), T = x.size(0);
  LSB_CHECK(W >= 1 && W <= kMaxOwners && rank >= 0 && rank < W, "one inbox per rank (<= 8)");
  LSB_CHECK(splits >= 1 && splits <= 64 && rows_per_rank >= 1 && rows_per_rank * W >= T, "bad split / row layout");
  if (T == 0) return;
  PartDest pd = {};
  for (int r = 0; r < W; ++r) pd.base[r] = reinterpret_cast<float*>(inboxes[r]);
  LSB_CHECK(!reduce || splits <= kMaxClusterSplits, "cluster-reduced splits must be 1..16");
  pd.rows = (int)rows_per_rank;
  pd.slot = (int)rank;
  pd.planes = reduce ? 1 : (int)splits;   // a cluster-reduced projection sends one plane per rank
  pd.owners = W;
  LSB_CHECK(n % 4 == 0 && epoch_ptr != 0, "the collective's inboxes need N % 4 == 0 and an epoch word");
  pd.ll = 1;
  pd.epoch = reinterpret_cast<const uint32_t*>(epoch_ptr);
  const at::cuda::CUDAGuard g(x.device());
  tile_dispatch(x, w, (int)n, packed, nullptr, pd, (int)splits, status_ptr(status), max_stages, reduce);
}

// out: bf16 [T, N] when splits == 1; partials: fp32 [splits, T, N] otherwise.
void gemm_bf16(at::Tensor out, at::Tensor x, at::Tensor w, at::Tensor partials, int64_t splits, at::Tensor status,
               int64_t max_stages) {
  LSB_CHECK(w.dim() == 2, "gemm weight must be 2-D");
  gemm_dispatch(out, x, w, w.size(0), false, partials, splits, status, max_stages);
}

// Same with a packed weight (see gemm.pack_weight) of n logical rows.
void gemm_bf16_packed(at::Tensor out, at::Tensor x, at::Tensor w, int64_t n, at::Tensor partials, int64_t splits,
                      at::Tensor status, int64_t max_stages) {
  gemm_dispatch(out, x, w, n, true, partials, splits, status, max_stages);
}

}  // namespace lsb
