// W4A16 GEMM for AutoAWQ (4-bit, group 128, zero point) weights on the 5th-generation tensor
// cores: Y[T, N] = X[T, K] . dequant(W)[N, K]^T,  dequant(w) = (q - z) * s per group of 128 K.
//
// Same swap-AB tiling as the bf16 kernel (128 output features = UMMA M, tokens = UMMA N), with a
// dequantisation stage between the copy and the MMA:
//   warp 0, lane 0 : producer.  Per 64-wide K step it bulk-copies the 4 KiB int4 tile of 128
//                    features (load-time repacked so one feature's 64 codes are 8 consecutive
//                    words), the 1 KiB scale/zero words of the tile's group, and the activation
//                    tile (2-D tensor copy, 128B swizzle) into a ring (6 stages for decode).
//   warps 2..9     : dequantisers (two CTAs per SM).  Each thread owns half (32 K) of one feature
//                    row: each 32-bit word holds 8 codes placed
//                    so that (word >> 4i) & 0x000F000F | 0x43004300 is the bf16 pair (128+q, 128+q')
//                    (exponent 2^7, codes in the low mantissa bits, exact); (pair - (128+z)) * s in
//                    bf16x2 gives round((q - z) * s).  For decode-sized T the 16 pairs go straight
//                    into a double-buffered operand in tensor memory (tcgen05.st, the row's TMEM
//                    lane, so a warp writes the 32 rows of its lane quadrant); otherwise into a
//                    double-buffered bf16 tile in the 128B-swizzled K-major layout in shared memory.
//   warp 1, lane 0 : MMA issuer, four tcgen05.mma (K = 16) per K step into a TMEM accumulator, A
//                    from tensor memory (or shared memory), B = the activation tile; commits free
//                    the ring stage and the operand buffer.
//   warps 2..9     : epilogue (tcgen05.ld), bf16 output or fp32 split-K partials.
// Every wait is bounded (a timeout records an error code and the roles drain and return).
// Every CTA issues its own TMA loads.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <cstdlib>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lsb {

CUtensorMap activation_map(const at::Tensor& x, int box_rows);
int* status_ptr(const at::Tensor& status);

namespace {

constexpr int QBM = 128;                 // features per CTA
constexpr int QBK = 64;                  // K per step
constexpr int kQTile = QBM * QBK / 2;    // 4 KiB of int4 codes
constexpr int kSZTile = QBM * 8;         // 1 KiB: (s, s) and (128+z, 128+z) bf16 pairs per feature
constexpr int kWTile = QBM * QBK * 2;    // 16 KiB bf16 operand

template <int BN, int STAGES, int WB>
struct QSmem {
  static constexpr int kX = BN * QBK * 2;
  static constexpr int kStage = kX + kQTile + kSZTile;      // X first (1024-aligned sizes)
  static constexpr int kWOff = STAGES * kStage;             // WB bf16 operand buffers
  static constexpr int kBarOff = kWOff + WB * kWTile;
  static constexpr int kBytes = kBarOff + (2 * STAGES + 2 * WB + 1) * 8 + 16 + 1024;
};

// WB operand buffers; shared memory budget per CTA: two CTAs per SM when WB == 2, three with the
// lean ring (WB == 1: one operand buffer, ~72 KB), one otherwise.
template <int BN, int WB>
constexpr int qstages() {
  constexpr int budget = (WB == 1 ? 72 : WB == 2 ? 110 : 200) * 1024 - WB * kWTile;
  constexpr int st = budget / QSmem<BN, 1, WB>::kStage;
  return st > 8 ? 8 : st < 2 ? 2 : st;
}
constexpr int kQThreads = 320;   // producer warp, MMA warp, 8 dequant / epilogue warps

template <int BN>
constexpr int qtmem_cols() {
  return BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
}
// With the dequantised operand in TMEM (TA): the accumulator's BN columns, then WB operand buffers of
// 32 columns (128 rows x 64 K as bf16 pairs), rounded up to an allocatable power of two.
template <int BN, int WB, bool TA>
constexpr int qtmem_alloc() {
  constexpr int need = TA ? (BN < 32 ? 32 : BN) + 32 * WB : qtmem_cols<BN>();
  return need <= 32 ? 32 : need <= 64 ? 64 : need <= 128 ? 128 : need <= 256 ? 256 : 512;
}

__device__ __forceinline__ uint64_t qdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <int N>
__host__ __device__ constexpr uint32_t qidesc() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(QBM >> 4) << 24);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tma_x(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void qmma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

// A from tensor memory (the dequantised weight tile), B from shared memory (the activation tile)
__device__ __forceinline__ void qmma_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void qst16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void qcommit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void qld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t bf2_sub_mul(uint32_t w, uint32_t z2, uint32_t s2) {
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&w);
  const __nv_bfloat162 z = *reinterpret_cast<const __nv_bfloat162*>(&z2);
  const __nv_bfloat162 s = *reinterpret_cast<const __nv_bfloat162*>(&s2);
  a = __hmul2(__hsub2(a, z), s);
  return *reinterpret_cast<uint32_t*>(&a);
}

template <int BN, int STAGES, int WB, bool TA = false>
__global__ void __launch_bounds__(kQThreads, 1) awq_gemm_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                          const uint32_t* __restrict__ qtiles,
                                                          const uint2* __restrict__ sztiles, bf16* __restrict__ out,
                                                          const PartDest pd, int T, int N, int k_tiles,
                                                          int k_tiles_per_split, int cluster_red,
                                                          int* __restrict__ status) {
  using L = QSmem<BN, STAGES, WB>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* wfull = empty + STAGES;    // [WB]
  uint64_t* wempty = wfull + WB;       // [WB]
  uint64_t* accum = wempty + WB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  __shared__ int abort_flag;
  volatile int* aborted = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (N + QBM - 1) / QBM, num_t = (T + BN - 1) / BN;
  const int m_tile = blockIdx.x % num_m, t_tile = blockIdx.x / num_m;
  (void)num_t;
  const int n0 = m_tile * QBM, t0 = t_tile * BN;
  const int kt_begin = blockIdx.z * k_tiles_per_split;
  const int kt_end = min(k_tiles, kt_begin + k_tiles_per_split);
  const int nk = max(0, kt_end - kt_begin);
  const int groups = k_tiles / 2;   // group 128 = two K steps

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < WB; ++b) {
      mbar_init(&wfull[b], 8);    // one arrive per dequant warp
      mbar_init(&wempty[b], 1);
    }
    mbar_init(accum, 1);
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(qtmem_alloc<BN, WB, TA>()));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // weights and scales do not depend on the previous kernel: issue the first stages' copies
      // of them before waiting on it (programmatic dependent launch), then the activations
      const int pre = nk < STAGES ? nk : STAGES;
      for (int i = 0; i < pre; ++i) {
        const int kt = kt_begin + i;
        uint8_t* st = smem + i * L::kStage;
        mbar_expect_tx(&full[i], L::kStage);
        bulk_g2s(smem_u32(st + L::kX), qtiles + ((size_t)m_tile * k_tiles + kt) * (kQTile / 4), kQTile, &full[i]);
        bulk_g2s(smem_u32(st + L::kX + kQTile), sztiles + ((size_t)m_tile * groups + kt / 2) * QBM, kSZTile,
                 &full[i]);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) tma_x(smem_u32(smem + i * L::kStage), &tm_x, &full[i], (kt_begin + i) * QBK, t0);
      int last[STAGES];
      for (int s = 0; s < STAGES; ++s) last[s] = s < pre ? s : -1;
      for (int i = pre; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1) || *aborted) {
          record_error(status, kTimeoutSmemEmpty);
          *aborted = 1;
          break;
        }
        const int kt = kt_begin + i;
        uint8_t* st = smem + s * L::kStage;
        mbar_expect_tx(&full[s], L::kStage);
        tma_x(smem_u32(st), &tm_x, &full[s], kt * QBK, t0);
        bulk_g2s(smem_u32(st + L::kX), qtiles + ((size_t)m_tile * k_tiles + kt) * (kQTile / 4), kQTile, &full[s]);
        bulk_g2s(smem_u32(st + L::kX + kQTile), sztiles + ((size_t)m_tile * groups + kt / 2) * QBM, kSZTile,
                 &full[s]);
        last[s] = i;
      }
      // drain (bounded): every issued copy has landed before the CTA may leave
      for (int s = 0; s < STAGES; ++s)
        if (last[s] >= 0) mbar_wait(&full[s], (last[s] / STAGES) & 1);
    } else {
      pdl_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0 && nk > 0) {
      constexpr uint32_t idesc = qidesc<BN>();
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES, b = i % WB;
        // the operand buffer (dequantised by warps 2..9) and, directly, the activation tile
        if (!mbar_wait(&wfull[b], (i / WB) & 1) || !mbar_wait(&full[s], (i / STAGES) & 1) || *aborted) {
          record_error(status, kTimeoutTmaFull);
          *aborted = 1;
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t xa = smem_u32(smem + s * L::kStage);
        if constexpr (TA) {
          // operand buffer b: TMEM columns [acc + 32 b, +32), 8 columns (16 K) per MMA
          const uint32_t ta = tmem + (uint32_t)((BN < 32 ? 32 : BN) + 32 * b);
#pragma unroll
          for (int k = 0; k < QBK / 16; ++k) qmma_ta(tmem, ta + k * 8, qdesc_sw128(xa + k * 32), idesc, (i | k) != 0);
        } else {
          const uint32_t wa = smem_u32(smem + L::kWOff + b * kWTile);
#pragma unroll
          for (int k = 0; k < QBK / 16; ++k)
            qmma(tmem, qdesc_sw128(wa + k * 32), qdesc_sw128(xa + k * 32), idesc, (i | k) != 0);
        }
        qcommit(&empty[s]);
        qcommit(&wempty[b]);
      }
      if (ok) qcommit(accum);
    }
    __syncwarp();
  } else {
    // ---- dequantise: thread t owns half h = t / 128 (words 4h..4h+3) of feature row r = t % 128 ----
    pdl_wait();
    const int t = threadIdx.x - 64;
    // TA: a warp may only reach TMEM lanes 32 (warp % 4) .. +31, so row r follows the warp's lanes
    const int r = TA ? (warp & 3) * 32 + lane : t & 127;
    const int h = TA ? (warp - 2) >> 2 : t >> 7;
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES, b = i % WB;
      bool ready = mbar_wait(&full[s], (i / STAGES) & 1) && mbar_wait(&wempty[b], ((i / WB) & 1) ^ 1) && !*aborted;
      if (TA) ready = __all_sync(0xffffffffu, ready);   // tcgen05.st below is warp-collective
      if (!ready) {
        record_error(status, kTimeoutTmaFull);
        *aborted = 1;
        ok = false;
        break;
      }
      // explicit shared-space loads (a generic load of shared memory takes the slower L1 path)
      const uint32_t st = smem_u32(smem + s * L::kStage);
      uint32_t words[4];
      uint2 sz;
      asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(words[0]), "=r"(words[1]), "=r"(words[2]), "=r"(words[3])
                   : "r"(st + L::kX + r * 32 + h * 16));
      asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(sz.x), "=r"(sz.y) : "r"(st + L::kX + kQTile + r * 8));
      if constexpr (TA) {
        // 32 K elements of row r as 16 bf16 pairs -> TMEM lane r, columns [acc + 32 b + 16 h, +16)
        uint32_t d[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            d[cc * 4 + j] = bf2_sub_mul(((words[cc] >> (4 * j)) & 0x000F000Fu) | 0x43004300u, sz.y, sz.x);
        qst16(tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((BN < 32 ? 32 : BN) + 32 * b + 16 * h), d);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      } else {
        const uint32_t wbase = smem_u32(smem + L::kWOff + b * kWTile) + r * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c = h * 4 + cc;
          const uint32_t v = words[cc];
          uint32_t d[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) d[j] = bf2_sub_mul(((v >> (4 * j)) & 0x000F000Fu) | 0x43004300u, sz.y, sz.x);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(wbase + (((c ^ (r & 7))) << 4)), "r"(d[0]),
                       "r"(d[1]), "r"(d[2]), "r"(d[3])
                       : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor core reads
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&wfull[b])) : "memory");
    }

    // ---- epilogue: warp w reads TMEM lanes 32*(w%4)..+31; warps 2-5 and 6-9 split the columns ----
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int kCols = BN >= 32 ? BN / 2 : BN;
    bool have = nk > 0 && ok;
    if (have && (!mbar_wait(accum, 0) || *aborted)) {
      record_error(status, kTimeoutAccum);
      have = false;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t ep = pd.call_epoch();   // the collective's epoch of this call (0 off TP)
    if (BN >= 32 || half == 0) {
      const int feat = n0 + q * 32 + lane;
      const uint32_t row_addr = tmem + ((uint32_t)(q * 32) << 16);
      const int cbeg = BN >= 32 ? half * kCols : 0;
#pragma unroll 1
      for (int c0 = cbeg; c0 < cbeg + kCols; c0 += 16) {
        uint32_t rr[16];
        if (have) {
          qld16(row_addr + c0, rr);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) rr[j] = 0u;
        }
        if (cluster_red > 0) {
          // park this K slice's tile [token][128 features] in the (now idle) ring memory
          float* red = reinterpret_cast<float*>(smem);
#pragma unroll
          for (int j = 0; j < 16; ++j) red[(c0 + j) * QBM + q * 32 + lane] = __uint_as_float(rr[j]);
        } else if (feat < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int tok = t0 + c0 + j;
            if (tok < T) {
              const float v = __uint_as_float(rr[j]);
              if (pd.base[0] != nullptr)
                pd.store(blockIdx.z, tok, N, feat, v, ep);
              else
                out[(size_t)tok * N + feat] = to_b(v);
            }
          }
        }
      }
    }
  }
  if (cluster_red > 0) {
    // the cluster_red K-slice CTAs of this tile sum their parked tiles through distributed shared
    // memory: CTA z writes slice z of the elements once (bf16, or one fp32 plane through pd)
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const uint32_t ep = pd.call_epoch();
    float* red = reinterpret_cast<float*>(smem);
    const int S = cluster_red, z = (int)cluster.block_rank();
    const int nvalid = max(0, min(BN, T - t0));
    const int E = nvalid * (QBM / 4);   // float4 groups: token j, features 4g..4g+3
    const int per = (E + S - 1) / S;
    const int e_end = min(E, (z + 1) * per);
    if (threadIdx.x >= 64) {
      for (int e = z * per + (int)threadIdx.x - 64; e < e_end; e += kQThreads - 64) {
        const int j = e / (QBM / 4), g = e - j * (QBM / 4);
        const int tok = t0 + j;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        int src = 0;
        for (; src + 4 <= S; src += 4) {
          float4 xv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            xv[u] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(red, src + u) + j * QBM + g * 4);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            a.x += xv[u].x; a.y += xv[u].y; a.z += xv[u].z; a.w += xv[u].w;
          }
        }
        for (; src < S; ++src) {
          const float4 xv = *reinterpret_cast<const float4*>(cluster.map_shared_rank(red, src) + j * QBM + g * 4);
          a.x += xv.x; a.y += xv.y; a.z += xv.z; a.w += xv.w;
        }
        const float va[4] = {a.x, a.y, a.z, a.w};
        const int f0 = n0 + g * 4;
        if (pd.base[0] != nullptr && (pd.ll || f0 + 3 < N)) {
          pd.store4(0, tok, N, f0, va, ep);
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            if (f0 + u >= N) break;
            if (pd.base[0] != nullptr) *pd.at(0, tok, N, f0 + u) = va[u];
            else out[(size_t)tok * N + f0 + u] = to_b(va[u]);
          }
        }
      }
    }
    cluster.sync();   // keep this CTA's tile alive until every peer CTA has read it
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(qtmem_alloc<BN, WB, TA>()));
  }
}

// reduce: the `splits` K slices of a tile reduce in a thread-block cluster (splits <= 8, the tile
// [BN][128] fp32 fitting in the ring + operand memory) and write bf16 `out` or one plane via `pd`.
template <int BN, int WB, bool TA = false>
void awq_launch(const at::Tensor& x, const at::Tensor& qt, const at::Tensor& sz, int N, bf16* out,
                const PartDest& pd, int splits, int* status, bool reduce = false) {
  constexpr int ST = qstages<BN, WB>();
  using L = QSmem<BN, ST, WB>;
  static_assert(L::kStage % 1024 == 0, "stage size must keep 1024-byte alignment");
  const int T = x.size(0), K = x.size(1);
  const int k_tiles = K / QBK;
  const int kps = (k_tiles + splits - 1) / splits;
  const CUtensorMap mx = activation_map(x, BN);
  auto kern = awq_gemm_kernel<BN, ST, WB, TA>;
  ensure_dynamic_smem((const void*)kern, L::kBytes);
  dim3 grid(((N + QBM - 1) / QBM) * ((T + BN - 1) / BN), 1, splits);
  const int cred = reduce && splits > 1 ? splits : 0;
  TORCH_CHECK(cred == 0 || (cred <= 8 && BN * QBM * 4 <= L::kBarOff),
              "llmserve_b200: AWQ cluster reduction needs <= 8 splits and a tile that fits the ring");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = L::kBytes;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  int nattr = 1;
  if (cred > 0) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = cred;
    nattr = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = nattr;
  cudaLaunchKernelEx(&cfg, kern, mx, (const uint32_t*)qt.data_ptr(), (const uint2*)sz.data_ptr(), out, pd, T, N,
                     k_tiles, kps, cred, status);
}

// For decode-sized T (<= 128) with two operand buffers the dequantisers write the bf16 weight
// operand into tensor memory (the MMA's A operand): no shared-memory stores and no async-proxy
// fence per K step (Qwen3-8B AWQ decode step at C = 64: 4.73 ms against 5.02 ms through shared
// memory).  LLMSERVE_AWQ_TMEM_A=0 selects the shared-memory operand.
bool awq_tmem_a() {
  static bool v = [] {
    const char* e = std::getenv("LLMSERVE_AWQ_TMEM_A");
    return !(e && std::atoi(e) == 0);
  }();
  return v;
}

int awq_wbuf() {
  static int v = [] {
    const char* e = std::getenv("LLMSERVE_AWQ_WBUF");
    return e ? std::atoi(e) : 2;
  }();
  return v;
}

template <int BN>
void awq_launch_any(const at::Tensor& x, const at::Tensor& qt, const at::Tensor& sz, int N, bf16* out,
                    const PartDest& pd, int splits, int* status, bool reduce) {
  const int wb = awq_wbuf();
  if constexpr (BN <= 128) {
    if (wb == 2 && awq_tmem_a()) {
      awq_launch<BN, 2, true>(x, qt, sz, N, out, pd, splits, status, reduce);
      return;
    }
  }
  if (wb >= 8) awq_launch<BN, 8>(x, qt, sz, N, out, pd, splits, status, reduce);
  else if (wb >= 4) awq_launch<BN, 4>(x, qt, sz, N, out, pd, splits, status, reduce);
  else if (wb == 1) awq_launch<BN, 1>(x, qt, sz, N, out, pd, splits, status, reduce);
  else awq_launch<BN, 2>(x, qt, sz, N, out, pd, splits, status, reduce);
}

void awq_dispatch(const at::Tensor& x, const at::Tensor& qt, const at::Tensor& sz, int N, bf16* o, const PartDest& pd,
                  int splits, int* st, bool reduce = false) {
  const int T = x.size(0);
  if (T <= 16) awq_launch_any<16>(x, qt, sz, N, o, pd, splits, st, reduce);
  else if (T <= 32) awq_launch_any<32>(x, qt, sz, N, o, pd, splits, st, reduce);
  else if (T <= 64) awq_launch_any<64>(x, qt, sz, N, o, pd, splits, st, reduce);
  else if (T <= 128) awq_launch_any<128>(x, qt, sz, N, o, pd, splits, st, reduce);
  else {
    TORCH_CHECK(!reduce, "llmserve_b200: AWQ cluster reduction is for T <= 128");
    awq_launch_any<256>(x, qt, sz, N, o, pd, splits, st, false);
  }
}

void check_awq_operands(const at::Tensor& x, const at::Tensor& qtiles, const at::Tensor& sztiles, int N) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "llmserve_b200: AWQ GEMM activations must be bf16 [T, K], K-contiguous");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "llmserve_b200: AWQ GEMM activations must be 16-byte aligned");
  const int K = x.size(1);
  TORCH_CHECK(K % 128 == 0, "llmserve_b200: AWQ K must be a multiple of the group size 128");
  const int64_t mt = (N + QBM - 1) / QBM;
  TORCH_CHECK(qtiles.is_contiguous() && qtiles.scalar_type() == at::kInt && qtiles.numel() == mt * (K / QBK) * QBM * 8,
              "llmserve_b200: AWQ qtiles shape mismatch");
  TORCH_CHECK(sztiles.is_contiguous() && sztiles.scalar_type() == at::kInt &&
                  sztiles.numel() == mt * (K / 128) * QBM * 2,
              "llmserve_b200: AWQ scale/zero tiles shape mismatch");
}

}  // namespace

// x [T, K] bf16; qtiles int32 [ceil(N/128), K/64, 128, 8]; sztiles int32 [ceil(N/128), K/128, 128, 2];
// out bf16 [T, N] (splits == 1) or partials fp32 [splits, T, N].
void awq_gemm(at::Tensor out, at::Tensor x, at::Tensor qtiles, at::Tensor sztiles, int64_t n, at::Tensor partials,
              int64_t splits, at::Tensor status) {
  const int T = x.size(0), N = (int)n;
  check_awq_operands(x, qtiles, sztiles, N);
  TORCH_CHECK(splits >= 1 && splits <= 64, "llmserve_b200: splits out of range");
  bf16* o = nullptr;
  float* p = nullptr;
  if (splits == 1 && partials.numel() == 0) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)T * N,
                "llmserve_b200: bad AWQ out");
    o = (bf16*)out.data_ptr();
  } else {
    TORCH_CHECK(partials.scalar_type() == at::kFloat && partials.is_contiguous() &&
                    partials.numel() == splits * (int64_t)T * N,
                "llmserve_b200: bad AWQ partials");
    p = partials.data_ptr<float>();
  }
  if (T == 0 || N == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  awq_dispatch(x, qtiles, sztiles, N, o, local_part_dest(p, T, (int)splits), (int)splits, status_ptr(status));
}

// bf16 out [T, N] = x . dequant(W)^T with K split over `splits` CTAs that reduce in a cluster
// (T <= 128, splits 2..8): no partial planes, no reduction kernel.
void awq_gemm_reduced(at::Tensor out, at::Tensor x, at::Tensor qtiles, at::Tensor sztiles, int64_t n, int64_t splits,
                      at::Tensor status) {
  const int T = x.size(0), N = (int)n;
  check_awq_operands(x, qtiles, sztiles, N);
  TORCH_CHECK(splits >= 2 && splits <= 8 && T <= 128, "llmserve_b200: cluster-reduced AWQ needs 2..8 splits, T <= 128");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (int64_t)T * N,
              "llmserve_b200: bad AWQ out");
  if (T == 0 || N == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  awq_dispatch(x, qtiles, sztiles, N, (bf16*)out.data_ptr(), local_part_dest(nullptr, T, 1), (int)splits,
               status_ptr(status), true);
}

// Row-parallel W4A16 projection under tensor parallelism: partial planes of token row t go to the
// inbox of the rank owning t (see PartDest) as epoch-tagged words stored by the epilogue.
void awq_gemm_to_owners(at::Tensor x, at::Tensor qtiles, at::Tensor sztiles, int64_t n, std::vector<int64_t> inboxes,
                        int64_t rank, int64_t rows_per_rank, int64_t splits, bool reduce, int64_t epoch_ptr,
                        at::Tensor status) {
  const int T = x.size(0), N = (int)n, W = (int)inboxes.size();
  check_awq_operands(x, qtiles, sztiles, N);
  TORCH_CHECK(W >= 1 && W <= kMaxOwners && rank >= 0 && rank < W, "llmserve_b200: one inbox per rank (<= 8)");
  TORCH_CHECK(splits >= 1 && splits <= 64 && rows_per_rank >= 1 && rows_per_rank * W >= T,
              "llmserve_b200: bad split / row layout");
  if (T == 0 || N == 0) return;
  PartDest pd = {};
  for (int r = 0; r < W; ++r) pd.base[r] = reinterpret_cast<float*>(inboxes[r]);
  pd.rows = (int)rows_per_rank;
  pd.slot = (int)rank;
  TORCH_CHECK(!reduce || (splits >= 2 && splits <= 8 && T <= 128 && N % 4 == 0),
              "llmserve_b200: cluster-reduced AWQ needs 2..8 splits, T <= 128, N % 4 == 0");
  pd.planes = reduce ? 1 : (int)splits;   // a cluster-reduced projection sends one plane per rank
  pd.owners = W;
  TORCH_CHECK(epoch_ptr != 0, "llmserve_b200: the collective's inboxes need an epoch word");
  pd.ll = 1;
  pd.epoch = reinterpret_cast<const uint32_t*>(epoch_ptr);
  const at::cuda::CUDAGuard g(x.device());
  awq_dispatch(x, qtiles, sztiles, N, nullptr, pd, (int)splits, status_ptr(status), reduce);
}

}  // namespace lsb
