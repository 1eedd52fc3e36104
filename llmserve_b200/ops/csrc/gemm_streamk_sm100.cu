// Persistent stream-K bf16 GEMM for decode-sized token counts (T <= 128) on the 5th-generation
// tensor cores: fp32 partials P[S, T, N] with sum_s P[s] = X[T, K] . W[N, K]^T.
//
// Why: a decode step is a stream of weight bytes.  Tiling the output into 128-row weight tiles
// and splitting K by a power of two leaves the grid unbalanced (QKV: 192 CTAs, gate_up: 192 CTAs
// on 148 SMs -- some SMs stream twice the bytes of others) and pays a launch/fill/drain per CTA.
// Here the grid is one or two resident CTAs per SM (8- or 4-stage ring), and the (weight tile,
// K tile) units -- m_tiles * k_tiles of them, each one 128 x 64 weight tile -- are dealt out as G
// contiguous, equal ranges: every SM streams the same number of weight bytes, once.  A range covers one or more "segments" (the part
// of one weight tile's K range that falls in it); each segment's fp32 sum goes to slot j of P,
// where j is the segment's position among the CTAs that share that tile, so the layout is the
// split-K layout every reducer of this library already consumes (residual + RMSNorm, QK-norm +
// RoPE, SiLU-mul, the TP collective).  Slots a tile does not use are zero-filled by the CTA that
// owns the tile's last segment.  The slot count S is computed on the host from (m_tiles, k_tiles,
// G) with the same arithmetic.
//
// Roles per CTA (192 threads): warp 0 lane 0 = TMA producer over the whole unit range (STAGES-deep
// ring of {128 x 64 weight tile from the tile-packed weight, BN x 64 activation tile}); warp 1 =
// TMEM allocator and, lane 0, the MMA issuer, accumulating each segment into one of two TMEM
// accumulators (BN fp32 columns each) so the epilogue of a segment overlaps the next one's MMAs;
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4).., one weight row = one output feature
// per thread, tokens along the columns), fp32 stores coalesced along the feature dimension.
// Every wait is bounded; a timeout records an error code in `status`, the roles drain (bounded)
// and TMEM is freed.  Every CTA issues its own TMA loads from this GPU's memory.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace lsb {

const CUtensorMap& weight_map(const at::Tensor& w, bool packed);
CUtensorMap activation_map(const at::Tensor& x, int box_rows);
int* status_ptr(const at::Tensor& status);

namespace {

#define LSB_CHECK_SK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreadsSK = 192;
constexpr int kMaxSlots = 8;

__device__ __forceinline__ uint64_t sk_desc_sw128(uint32_t saddr) {
  // K-major, 128B swizzle: start >> 4, LBO 1 (unused), SBO 1024 B >> 4, version 1, layout 2.
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, fp32 accumulate, A = B = bf16, K-major, N = BN, M = 128.
template <int BN>
__host__ __device__ constexpr uint32_t sk_idesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void sk_tma_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void sk_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void sk_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void sk_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void sk_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void sk_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void sk_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The CTA whose unit range [floor(c U / G), floor((c+1) U / G)) holds unit u.
__host__ __device__ __forceinline__ int owner_of(int64_t u, int64_t U, int64_t G) {
  return (int)(((u + 1) * G + U - 1) / U - 1);
}

template <int BN, int STAGES>
struct SkSmem {
  static constexpr int kW = kBM * kBK * 2;     // 16 KiB weight tile (pre-swizzled image)
  static constexpr int kX = BN * kBK * 2;      // activation tile, 128B swizzle
  static constexpr int kStage = kW + kX;
  static constexpr int kBarOff = STAGES * kStage;
  // full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], tmem slot
  static constexpr int kBytes = kBarOff + (2 * STAGES + 4) * 8 + 16 + 1024;
};

template <int BN>
constexpr uint32_t sk_tmem_cols() {
  return 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 256;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreadsSK, 1) gemm_streamk_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                     const __grid_constant__ CUtensorMap tm_x,
                                                                     float* __restrict__ part, int T, int N,
                                                                     int k_tiles, int m_tiles, int S,
                                                                     int* __restrict__ status) {
  using L = SkSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t U = (int64_t)m_tiles * k_tiles, G = gridDim.x;
  const int u0 = (int)((int64_t)blockIdx.x * U / G), u1 = (int)((int64_t)(blockIdx.x + 1) * U / G);
  const int nu = u1 - u0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);   // one arrival per epilogue warp
    }
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(sk_tmem_cols<BN>()));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  sk_fence_before();
  __syncthreads();
  sk_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0 && nu > 0) {
      // unit u -> weight tile (u / k_tiles, u % k_tiles); the packed weight keeps tile (m, kt) at
      // rows (m * k_tiles + kt) * 128 of a [rows, 64] image, so the tile's row is simply u * 128.
      const int pre = nu < STAGES ? nu : STAGES;
      for (int i = 0; i < pre; ++i) {   // weights never depend on the predecessor kernel
        mbar_expect_tx(&full[i], L::kStage);
        sk_tma_2d(smem + i * L::kStage, &tm_w, &full[i], 0, (u0 + i) * kBM);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        sk_tma_2d(smem + i * L::kStage + L::kW, &tm_x, &full[i], ((u0 + i) % k_tiles) * kBK, 0);
      int issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = s < pre ? s + 1 : 0;
      for (int i = pre; i < nu; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1)) {
          record_error(status, kTimeoutSmemEmpty);
          atomicExch(&abort_flag, 1);
          break;
        }
        if (*((volatile int*)&abort_flag)) break;
        uint8_t* st = smem + s * L::kStage;
        mbar_expect_tx(&full[s], L::kStage);
        sk_tma_2d(st, &tm_w, &full[s], 0, (u0 + i) * kBM);
        sk_tma_2d(st + L::kW, &tm_x, &full[s], ((u0 + i) % k_tiles) * kBK, 0);
        issued[s] = i + 1;
      }
      if (*((volatile int*)&abort_flag)) {
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] > 0) mbar_wait(&full[s], ((issued[s] - 1) / STAGES) & 1);
      }
    } else {
      pdl_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && nu > 0) {
      constexpr uint32_t idesc = sk_idesc<BN>();
      int i = 0, seg = 0;
      bool ok = true;
      while (i < nu && ok) {
        const int u = u0 + i;
        const int seg_end = min(u1, (u / k_tiles + 1) * k_tiles);
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[b], ((seg >> 1) - 1) & 1)) {
          record_error(status, kTimeoutAccum);
          atomicExch(&abort_flag, 1);
          ok = false;
          break;
        }
        sk_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        for (int v = u; v < seg_end; ++v, ++i) {
          const int s = i % STAGES;
          if (!mbar_wait(&full[s], (i / STAGES) & 1) || *((volatile int*)&abort_flag)) {
            record_error(status, kTimeoutTmaFull);
            atomicExch(&abort_flag, 1);
            ok = false;
            break;
          }
          sk_fence_after();
          const uint32_t wa = smem_u32(smem + s * L::kStage);
          const uint32_t xa = wa + L::kW;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            sk_mma(acc, sk_desc_sw128(wa + k * 32), sk_desc_sw128(xa + k * 32), idesc, (v != u || k != 0) ? 1u : 0u);
          sk_commit(&empty[s]);
        }
        if (ok) sk_commit(&acc_full[b]);
        ++seg;
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue: warps 2..5 ------------------------------------------------------------------
    pdl_wait();
    const int quad = warp & 3;                      // TMEM lanes 32*quad .. 32*quad+31
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const int64_t TN = (int64_t)T * N;
    int i = 0, seg = 0;
    while (i < nu) {
      const int u = u0 + i;
      const int m = u / k_tiles;
      const int seg_end = min(u1, (m + 1) * k_tiles);
      const int b = seg & 1;
      const int first = owner_of((int64_t)m * k_tiles, U, G);
      const int slot = (int)blockIdx.x - first;
      const int feat = m * kBM + quad * 32 + lane;
      bool have = !*((volatile int*)&abort_flag);
      if (have && !mbar_wait(&acc_full[b], (seg >> 1) & 1)) {
        record_error(status, kTimeoutAccum);
        atomicExch(&abort_flag, 1);
        have = false;
      }
      have = __all_sync(0xffffffffu, have);       // tcgen05.ld below is warp-collective
      sk_fence_after();
      if (have && slot < S) {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          sk_ld16(lane_base + (uint32_t)(b * BN + c0), r);
          if (feat < N) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int t = c0 + j;
              if (t < T) part[(int64_t)slot * TN + (int64_t)t * N + feat] = __uint_as_float(r[j]);
            }
          }
        }
      }
      sk_fence_before();
      __syncwarp();
      if (lane == 0) sk_arrive(&acc_empty[b]);
      // the owner of the tile's last unit clears the slots no CTA writes for this tile
      if (seg_end == (m + 1) * k_tiles && feat < N) {
        const int nseg = owner_of((int64_t)(m + 1) * k_tiles - 1, U, G) - first + 1;
        for (int z = nseg; z < S; ++z)
          for (int t = 0; t < T; ++t) part[(int64_t)z * TN + (int64_t)t * N + feat] = 0.f;
      }
      i += seg_end - u;
      ++seg;
    }
  }

  sk_fence_before();
  __syncthreads();
  if (warp == 1) {
    sk_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(sk_tmem_cols<BN>()));
  }
}

template <int BN, int STAGES>
void launch_streamk(float* part, const at::Tensor& x, const at::Tensor& w, int N, int k_tiles, int m_tiles, int S,
                    int grid, int* status) {
  using L = SkSmem<BN, STAGES>;
  static_assert(L::kStage % 1024 == 0, "stage size must keep 1024-byte alignment");
  static_assert(L::kBytes <= 227 * 1024, "shared memory budget");
  const CUtensorMap mx = activation_map(x, BN);
  const CUtensorMap& mw = weight_map(w, true);
  auto kern = gemm_streamk_kernel<BN, STAGES>;
  ensure_dynamic_smem((const void*)kern, L::kBytes);
  launch_pdl(kern, dim3(grid), dim3(kThreadsSK), L::kBytes, at::cuda::getCurrentCUDAStream(), mw, mx, part,
             (int)x.size(0), N, k_tiles, m_tiles, S, status);
}

}  // namespace

// Number of partial slots the stream-K schedule of (m_tiles x k_tiles) units over `grid` CTAs
// needs: the largest number of CTAs that share one weight tile.
int64_t streamk_slots(int64_t m_tiles, int64_t k_tiles, int64_t grid) {
  const int64_t U = m_tiles * k_tiles;
  int64_t best = 0;
  for (int64_t m = 0; m < m_tiles; ++m) {
    const int64_t n = owner_of((m + 1) * k_tiles - 1, U, grid) - owner_of(m * k_tiles, U, grid) + 1;
    best = n > best ? n : best;
  }
  return best;
}

// partials: fp32 [S, T, N]; x: bf16 [T, K] (T <= 128); w: tile-packed weight image of N logical
// rows (see gemm.pack_weight); grid: CTAs, whose schedule needs exactly S slots (streamk_slots);
// stages: ring depth, 8 (about 195 KiB: one CTA per SM) or 4 (two CTAs per SM).
void gemm_bf16_streamk(at::Tensor partials, at::Tensor x, at::Tensor w, int64_t n, int64_t grid, int64_t stages,
                       at::Tensor status) {
  LSB_CHECK_SK(x.is_cuda() && w.is_cuda() && partials.is_cuda(), "stream-K operands must be CUDA tensors");
  LSB_CHECK_SK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16, "operands must be bf16");
  LSB_CHECK_SK(x.dim() == 2 && x.stride(1) == 1 && (x.stride(0) * 2) % 16 == 0, "x must be [T, K], 16-byte rows");
  LSB_CHECK_SK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x must be 16-byte aligned");
  const int T = x.size(0), K = x.size(1), N = (int)n;
  const int k_tiles = (K + kBK - 1) / kBK, m_tiles = (N + kBM - 1) / kBM;
  const int64_t mt_pad = (n + 255) / 256 * 2;
  LSB_CHECK_SK(w.dim() == 2 && w.size(1) == kBK && w.is_contiguous() && w.size(0) == mt_pad * k_tiles * kBM,
               "packed weight shape mismatch");
  LSB_CHECK_SK(T >= 1 && T <= 128, "stream-K GEMM takes 1..128 tokens");
  LSB_CHECK_SK(partials.scalar_type() == at::kFloat && partials.is_contiguous() && partials.dim() == 3 &&
                   partials.size(1) == T && partials.size(2) == N, "partials must be fp32 [S, T, N]");
  const int S = partials.size(0);
  LSB_CHECK_SK(grid >= 1 && grid <= (int64_t)m_tiles * k_tiles && grid <= 1024, "bad stream-K grid");
  LSB_CHECK_SK(S >= 1 && S <= kMaxSlots && S == streamk_slots(m_tiles, k_tiles, grid),
               "partials slot count does not match the stream-K schedule");
  LSB_CHECK_SK(stages == 4 || stages == 8, "stream-K ring depth must be 4 (two CTAs per SM) or 8 (one)");
  const at::cuda::CUDAGuard g(x.device());
  int* st = status_ptr(status);
  float* p = partials.data_ptr<float>();
  const int G = (int)grid;
  const bool deep = stages == 8;
  if (T <= 16) {
    if (deep) launch_streamk<16, 8>(p, x, w, N, k_tiles, m_tiles, S, G, st);
    else launch_streamk<16, 4>(p, x, w, N, k_tiles, m_tiles, S, G, st);
  } else if (T <= 32) {
    if (deep) launch_streamk<32, 8>(p, x, w, N, k_tiles, m_tiles, S, G, st);
    else launch_streamk<32, 4>(p, x, w, N, k_tiles, m_tiles, S, G, st);
  } else if (T <= 64) {
    if (deep) launch_streamk<64, 8>(p, x, w, N, k_tiles, m_tiles, S, G, st);
    else launch_streamk<64, 4>(p, x, w, N, k_tiles, m_tiles, S, G, st);
  } else {
    if (deep) launch_streamk<128, 6>(p, x, w, N, k_tiles, m_tiles, S, G, st);
    else launch_streamk<128, 4>(p, x, w, N, k_tiles, m_tiles, S, G, st);
  }
}

}  // namespace lsb
