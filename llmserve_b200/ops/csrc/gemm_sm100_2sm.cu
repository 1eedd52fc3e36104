// Wide bf16 GEMM for prefill-sized token counts: Y[T, N] = X[T, K] . W[N, K]^T on CTA pairs.
//
// Blackwell 2-SM tensor-core path (tcgen05 with cta_group::2):
//   * a cluster of two CTAs (two SMs) owns a 256-token x 256-feature output tile; CTA r loads
//     tokens [128r, 128r+128) of X and features [128r, 128r+128) of W for every 64-wide K step,
//     so each SM stages 32 KiB per step instead of the 48 KiB a one-SM 128x256 tile needs;
//   * the even CTA's single MMA thread issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16),
//     which reads A from both CTAs' shared memory (split along M) and B from both (split along N)
//     and leaves rows 128r.. of the fp32 accumulator in CTA r's tensor memory;
//   * the kernel is persistent (one cluster per SM pair, tiles strided by cluster id) and the
//     accumulator is double-buffered in TMEM (2 x 256 columns = all 512), so the epilogue of one
//     tile (tcgen05.ld -> bf16/fp32 -> 16-byte global stores) overlaps the next tile's main loop.
//
// W comes either row-major (128B-swizzled tensor map) or as the packed tile image of
// ``gemm.pack_weight`` (each 128 x 64 tile one contiguous, pre-swizzled 16 KiB run: sequential
// HBM pages instead of 128-byte pieces of 128 rows).
//
// Roles per CTA (192 threads): warp 0 lane 0 = TMA producer (6-stage ring, 32 KiB per stage),
// warp 1 = TMEM allocator and, on the even CTA, the MMA issuer; warps 2..5 = epilogue (warp w
// reads TMEM lanes 32*(w%4)..+31, the restriction tcgen05.ld places on a warp).
// Both CTAs' TMA loads complete on the even CTA's "full" barrier (the cta_group::2 form of the
// bulk tensor copy addresses a barrier in the peer CTA); the MMA thread's commits arrive on the
// "empty" and "accumulator full" barriers of both CTAs (one plain commit per CTA).  Every
// wait is bounded: a timeout records an error code, stops the role, and both CTAs still meet at
// the final cluster barrier before TMEM is released.  Every CTA loads its own tiles from
// this GPU's memory (the kernel runs under tensor parallelism).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace lsb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
const CUtensorMap& weight_map(const at::Tensor& w, bool packed);

namespace {

#define LSB_CHECK2(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

constexpr int kRows = 128;                       // token rows (and feature rows) per CTA
constexpr int kTileN = 256;                      // features per pair tile
constexpr int kTileT = 256;                      // tokens per pair tile
constexpr int kBK = 64;                          // K per stage: 128-byte rows, 128B swizzle
constexpr int kStages = 6;
constexpr int kHalf = kRows * kBK * 2;           // 16 KiB: one operand half per CTA per stage
constexpr int kStageBytes = 2 * kHalf;           // X half + W half
constexpr int kBarOff = kStages * kStageBytes;   // 192 KiB
constexpr int kSmemBytes = kBarOff + 256 + 1024; // barriers + alignment slack
constexpr int kThreads = 192;
constexpr int kAccCols = 256;                    // fp32 accumulator columns per buffer
constexpr int kGroupT = 8;                       // token tiles per raster group

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  // K-major, 128B swizzle: start >> 4, LBO 1 (unused), SBO 1024 B >> 4, version 1, layout 2.
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, fp32 accumulate, A = B = bf16, K-major, N = 256 (>> 3 at bit 17), M = 256 (>> 4 at 24).
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileN >> 3) << 17) |
                            ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ bool try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool wait_cluster(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (try_wait_cluster(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

__device__ __forceinline__ void tma_load_pair(uint32_t dst, const CUtensorMap* map, uint32_t leader_bar, int x,
                                              int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(map), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tile_coords(int tile, int num_n, int num_t, int& t_tile, int& n_tile) {
  const int per_group = kGroupT * num_n;
  const int grp = tile / per_group, rem = tile - grp * per_group;
  const int first_t = grp * kGroupT;
  const int gsz = min(num_t - first_t, kGroupT);
  t_tile = first_t + rem % gsz;
  n_tile = rem / gsz;
}

template <bool kF32Out>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     void* __restrict__ out, int T, int N, int k_tiles, int packed, int* __restrict__ status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;    // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2], used on the even CTA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int abort_flag;
  volatile int* aborted = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int num_n = (N + kTileN - 1) / kTileN, num_t = (T + kTileT - 1) / kTileT;
  const int num_tiles = num_n * num_t;
  const int first_tile = (int)cluster_id_x(), tile_step = (int)num_clusters_x();

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);   // 4 epilogue warps x 2 CTAs
    }
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * kAccCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();   // barriers of both CTAs initialised before any remote arrive / complete_tx
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int it = 0, last_issued[kStages];
      for (int s = 0; s < kStages; ++s) last_issued[s] = -1;
      for (int tile = first_tile; tile < num_tiles && !*aborted; tile += tile_step) {
        int tt, nt;
        tile_coords(tile, num_n, num_t, tt, nt);
        const int x_row = tt * kTileT + (int)rank * kRows;
        const int w_row = nt * kTileN + (int)rank * kRows;
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            record_error(status, kTimeoutSmemEmpty);
            *aborted = 1;
            break;
          }
          if (rank == 0) mbar_expect_tx(&full[s], 2 * kStageBytes);   // both CTAs' halves
          const uint32_t leader_full = map_to_rank(smem_u32(&full[s]), 0);
          const uint32_t dst = smem_u32(smem + s * kStageBytes);
          tma_load_pair(dst, &tm_x, leader_full, kt * kBK, x_row);
          // W: row-major (128B-swizzled map) or packed tiles (tile m, kt = 128 rows at (m*k_tiles+kt)*128)
          if (packed)
            tma_load_pair(dst + kHalf, &tm_w, leader_full, 0, ((nt * 2 + (int)rank) * k_tiles + kt) * kRows);
          else
            tma_load_pair(dst + kHalf, &tm_w, leader_full, kt * kBK, w_row);
          last_issued[s] = it;
        }
      }
      // Tail (bounded waits): do not leave while a copy into this CTA or an MMA release of one of
      // its stages is still in flight.  The even CTA's full barrier also counts the odd CTA's copies.
      for (int s = 0; s < kStages; ++s) {
        if (last_issued[s] < 0) continue;
        const uint32_t use = (uint32_t)(last_issued[s] / kStages);
        if (rank == 0 && *aborted) mbar_wait(&full[s], use & 1);
        if (!*aborted) mbar_wait(&empty[s], use & 1);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t peer_empty0 = map_to_rank(smem_u32(&empty[0]), 1);
      const uint32_t peer_accf0 = map_to_rank(smem_u32(&acc_full[0]), 1);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = first_tile; tile < num_tiles && ok; tile += tile_step, ++local) {
        const int b = local & 1;
        const uint32_t use = local >> 1;
        if (!wait_cluster(smem_u32(&acc_empty[b]), (use & 1) ^ 1)) {
          record_error(status, kTimeoutAccum);
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(b * kAccCols);
        for (int kt = 0; kt < k_tiles; ++kt, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&full[s], ph) || *aborted) {
            record_error(status, kTimeoutTmaFull);
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t xa = smem_u32(smem + s * kStageBytes);
          const uint32_t wa = xa + kHalf;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            mma_pair(d, desc_sw128(xa + k * 32), desc_sw128(wa + k * 32), (kt | k) != 0);
          commit_pair(smem_u32(&empty[s]));
          commit_pair(peer_empty0 + (uint32_t)(s * 8));
        }
        if (!ok) break;
        commit_pair(smem_u32(&acc_full[b]));
        commit_pair(peer_accf0 + (uint32_t)(b * 8));
      }
      if (!ok) *aborted = 1;
    }
    __syncwarp();
  } else {
    // epilogue: warp w owns TMEM lanes 32*(w%4)..+31 = token rows of this CTA's half tile
    const int q = warp & 3;
    const uint32_t leader_acc_empty0 = map_to_rank(smem_u32(&acc_empty[0]), 0);
    int local = 0;
    for (int tile = first_tile; tile < num_tiles; tile += tile_step, ++local) {
      const int b = local & 1;
      const uint32_t use = local >> 1;
      if (!mbar_wait(&acc_full[b], use & 1)) {
        record_error(status, kTimeoutAccum);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int tt, nt;
      tile_coords(tile, num_n, num_t, tt, nt);
      const int tok = tt * kTileT + (int)rank * kRows + q * 32 + lane;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kAccCols);
#pragma unroll 1
      for (int c0 = 0; c0 < kAccCols; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(base + (uint32_t)c0, r);
        const int f0 = nt * kTileN + c0;
        if (tok < T && f0 < N) {
          if constexpr (kF32Out) {
            float* dst = reinterpret_cast<float*>(out) + (size_t)tok * N + f0;
            if (f0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(dst + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                  __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (f0 + j < N) dst[j] = __uint_as_float(r[j]);
            }
          } else {
            bf16* dst = reinterpret_cast<bf16*>(out) + (size_t)tok * N + f0;
            if (f0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 v;
                __nv_bfloat162 h0 = __floats2bfloat162_rn(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
                __nv_bfloat162 h1 = __floats2bfloat162_rn(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                __nv_bfloat162 h2 = __floats2bfloat162_rn(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
                __nv_bfloat162 h3 = __floats2bfloat162_rn(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
                v.x = *reinterpret_cast<uint32_t*>(&h0);
                v.y = *reinterpret_cast<uint32_t*>(&h1);
                v.z = *reinterpret_cast<uint32_t*>(&h2);
                v.w = *reinterpret_cast<uint32_t*>(&h3);
                *reinterpret_cast<uint4*>(dst + j) = v;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (f0 + j < N) dst[j] = to_b(__uint_as_float(r[j]));
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) arrive_remote(leader_acc_empty0 + (uint32_t)(b * 8));
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync();   // no CTA leaves while its peer may still signal its barriers or read its smem
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kAccCols));
  }
}

CUtensorMap make_rows_map(const void* ptr, int64_t rows, int64_t cols, int64_t stride) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kRows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LSB_CHECK2(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return m;
}

int max_pairs_resident() {
  static int pairs = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    pairs = sms / 2;
    ensure_dynamic_smem((const void*)gemm_pair_kernel<false>, kSmemBytes);
    ensure_dynamic_smem((const void*)gemm_pair_kernel<true>, kSmemBytes);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, (void*)gemm_pair_kernel<false>, &cfg) == cudaSuccess && clusters > 0)
      pairs = std::min(pairs, clusters);
    cudaGetLastError();
  });
  return pairs;
}

}  // namespace

// out: bf16 [T, N] (out_f32 false) or fp32 [T, N]; x [T, K], w [N, K] bf16, K-contiguous.
void gemm_bf16_pair(void* out, bool out_f32, const at::Tensor& x, const at::Tensor& w, int N, bool packed,
                    int* status) {
  const int T = x.size(0), K = x.size(1);
  LSB_CHECK2(N % 8 == 0, "wide GEMM needs N % 8 == 0");
  const CUtensorMap mx = make_rows_map(x.data_ptr(), T, K, x.stride(0));
  const CUtensorMap& mw = weight_map(w, packed);
  const int k_tiles = (K + kBK - 1) / kBK;
  const int tiles = ((N + kTileN - 1) / kTileN) * ((T + kTileT - 1) / kTileT);
  const int pairs = std::min(tiles, max_pairs_resident());
  // the occupancy query above ran on the first device only; the attribute is per device
  ensure_dynamic_smem((const void*)gemm_pair_kernel<false>, kSmemBytes);
  ensure_dynamic_smem((const void*)gemm_pair_kernel<true>, kSmemBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (out_f32)
    cudaLaunchKernelEx(&cfg, gemm_pair_kernel<true>, mx, mw, out, T, N, k_tiles, (int)packed, status);
  else
    cudaLaunchKernelEx(&cfg, gemm_pair_kernel<false>, mx, mw, out, T, N, k_tiles, (int)packed, status);
}

}  // namespace lsb
