// Tile helpers of the paged attention kernels and the split-KV decode kernel.
//
// Shared by attention.cu (the entry points that take a caller-provided workspace) and
// decode_noalloc.cu (the entry point whose scratch is a static device array).
#pragma once

#include "common.cuh"

namespace lsb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int KT = 64;          // keys per tile
constexpr int NTHREADS = 128;   // 4 warps

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Byte offset of 16-byte chunk `c` of row `r` in a tile whose rows are HD bf16 long.
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * HD * 2 + ((c ^ (r & 7)) << 4));
}

// Stage KT keys [kstart, kstart+KT) of one KV head (rows >= kend are zero-filled).  A block id
// outside [0, nblk) is never dereferenced: its rows are zero-filled and kBadIndex is recorded
// (status may be null).
template <int HD>
__device__ __forceinline__ void load_kv_tile(bf16* sk, bf16* sv, const bf16* kc, const bf16* vc, const int* bt,
                                             int kstart, int kend, int kvh, int nkv, int bs, int nblk, int* status) {
  constexpr int CH = HD / 8;   // 16-byte chunks per row
  for (int q = threadIdx.x; q < KT * CH; q += NTHREADS) {
    const int r = q / CH, c = q % CH;
    const int pos = kstart + r;
    bool ok = pos < kend;
    size_t off = 0;
    if (ok) {
      const int blk = bt[pos / bs];
      if ((unsigned)blk < (unsigned)nblk) {
        off = (((size_t)blk * nkv + kvh) * bs + pos % bs) * HD + c * 8;
      } else {
        ok = false;
        if (c == 0) record_error(status, kBadIndex);
      }
    }
    cp_async16(reinterpret_cast<char*>(sk) + swz<HD>(r, c), kc + off, ok);
    cp_async16(reinterpret_cast<char*>(sv) + swz<HD>(r, c), vc + off, ok);
  }
}

// Online-softmax update for this warp's 16x16 score block (two n8 tiles) and PV accumulation.
// s0/s1: C fragments of keys [0,8) and [8,16) of the warp's 16-key slice.  Returns nothing;
// updates m (2 rows), l (2 rows, per-lane partial), o (HD/8 n-tiles).
template <int HD>
__device__ __forceinline__ void softmax_pv(float* s0, float* s1, float* m, float* l, float (*o)[4], uint32_t sv_base,
                                           int key0_in_tile) {
  const int lane = threadIdx.x & 31;
  float mx[2];
  mx[0] = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
  mx[1] = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
    mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
  }
  float corr[2], mu[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const float mn = fmaxf(m[r], mx[r]);
    mu[r] = mn == -INFINITY ? 0.f : mn;
    corr[r] = exp2f(m[r] - mu[r]);
    m[r] = mn;
    l[r] *= corr[r];
  }
  float p[8];
  p[0] = exp2f(s0[0] - mu[0]); p[1] = exp2f(s0[1] - mu[0]);
  p[2] = exp2f(s0[2] - mu[1]); p[3] = exp2f(s0[3] - mu[1]);
  p[4] = exp2f(s1[0] - mu[0]); p[5] = exp2f(s1[1] - mu[0]);
  p[6] = exp2f(s1[2] - mu[1]); p[7] = exp2f(s1[3] - mu[1]);
  l[0] += p[0] + p[1] + p[4] + p[5];
  l[1] += p[2] + p[3] + p[6] + p[7];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) {
    o[n][0] *= corr[0]; o[n][1] *= corr[0];
    o[n][2] *= corr[1]; o[n][3] *= corr[1];
  }
  uint32_t a[4];
  a[0] = pack_bf16(p[0], p[1]);
  a[1] = pack_bf16(p[2], p[3]);
  a[2] = pack_bf16(p[4], p[5]);
  a[3] = pack_bf16(p[6], p[7]);
  const int key = key0_in_tile + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
  for (int dt = 0; dt < HD / 16; ++dt) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(b0, b1, b2, b3, sv_base + swz<HD>(key, dt * 2 + (lane >> 4)));
    mma16816(o[2 * dt], a, b0, b1);
    mma16816(o[2 * dt + 1], a, b2, b3);
  }
}

// S (16 rows x 16 keys at key0_in_tile) = Qfrag . K^T
template <int HD>
__device__ __forceinline__ void qk16(float* s0, float* s1, const uint32_t (*qa)[4], uint32_t sk_base, int key0_in_tile) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 4; ++i) s0[i] = s1[i] = 0.f;
  const int key = key0_in_tile + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4(b0, b1, b2, b3, sk_base + swz<HD>(key, kk * 2 + ((lane >> 3) & 1)));
    mma16816(s0, qa[kk], b0, b1);
    mma16816(s1, qa[kk], b2, b3);
  }
}

// ------------------------------------------------------------------------------------------
// Decode
// ------------------------------------------------------------------------------------------
// grid (B, kv_heads, Z): CTA z handles splits z, z+Z, ... of `partition` keys each.  A split's
// result is written straight to `out` when the context has one split; otherwise it goes to the
// workspace and the CTA that finishes the last split of (b, kv head) -- detected with a per-pair
// counter that it resets afterwards -- merges all splits.
template <int HD>
__global__ void __launch_bounds__(NTHREADS) decode_kernel(
    bf16* __restrict__ out, const bf16* __restrict__ q, const bf16* __restrict__ kc, const bf16* __restrict__ vc,
    const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ context_lens, float scale_log2,
    float* __restrict__ part_o, float* __restrict__ part_ml, int* __restrict__ counters, int max_splits,
    int partition, int nh, int nkv, int bs, int nblk, int* __restrict__ status) {
  pdl_trigger();
  extern __shared__ __align__(128) char smem[];
  __shared__ int is_last;
  bf16* sk[2] = {reinterpret_cast<bf16*>(smem), reinterpret_cast<bf16*>(smem + 2 * KT * HD * 2)};
  bf16* sv[2] = {reinterpret_cast<bf16*>(smem + KT * HD * 2), reinterpret_cast<bf16*>(smem + 3 * KT * HD * 2)};
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int G = nh / nkv;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Context lengths and block tables are written by the host before the step's first kernel, and
  // only the newest position's K/V (ctx - 1) is written by the kernel just before this one.  So
  // the first tile, when it ends before that position, is streamed before waiting on the
  // predecessor (programmatic dependent launch), overlapping it with the QKV projection.
  // a context longer than the block table row is clamped to it: every block-table read and every
  // split slot (b, h, split < max_splits) then stays inside what the caller sized
  const int ctx = max(0, min(context_lens[b], bt_stride * bs));
  const int nsplits = (ctx + partition - 1) / partition;
  const int* bt = block_tables + (size_t)b * bt_stride;
  bool prefetched = false;
  if ((int)blockIdx.z < nsplits) {
    const int ks = blockIdx.z * partition;
    const int ke = min(ks + partition, ctx);
    if (min(ks + KT, ke) <= ctx - 1) {
      load_kv_tile<HD>(sk[0], sv[0], kc, vc, bt, ks, ke, kvh, nkv, bs, nblk, status);
      cp_async_commit();
      prefetched = true;
    }
  }
  pdl_wait();
  if (nsplits == 0) {
    if (blockIdx.z == 0)
      for (int i = threadIdx.x; i < G * HD; i += NTHREADS) out[((size_t)b * nh + kvh * G) * HD + i] = to_b(0.f);
    return;
  }
  uint32_t qa[HD / 16][4];
  {
    const int r0 = lane >> 2, c = (lane & 3) * 2;
    const bf16* qb = q + ((size_t)b * nh + kvh * G) * HD;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      const int col = kk * 16 + c;
      auto ld = [&](int r, int cc) -> uint32_t {
        if (r >= G) return 0u;
        return *reinterpret_cast<const uint32_t*>(qb + (size_t)r * HD + cc);
      };
      qa[kk][0] = ld(r0, col);
      qa[kk][1] = ld(r0 + 8, col);
      qa[kk][2] = ld(r0, col + 8);
      qa[kk][3] = ld(r0 + 8, col + 8);
    }
  }
  float* so = reinterpret_cast<float*>(smem);   // [4 warps][16 rows][HD] once the tiles are consumed
  float* sm = so + 4 * 16 * HD;
  float* sl = sm + 64;
  const int g = lane >> 2, c2 = (lane & 3) * 2;
  for (int split = blockIdx.z; split < nsplits; split += gridDim.z) {
    const int kstart = split * partition;
    const int kend = min(kstart + partition, ctx);
    const int ntiles = (kend - kstart + KT - 1) / KT;
    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    __syncthreads();   // shared memory is reused across splits
    if (!prefetched) {
      load_kv_tile<HD>(sk[0], sv[0], kc, vc, bt, kstart, kend, kvh, nkv, bs, nblk, status);
      cp_async_commit();
    }
    prefetched = false;
    for (int t = 0; t < ntiles; ++t) {
      if (t + 1 < ntiles) {
        load_kv_tile<HD>(sk[(t + 1) & 1], sv[(t + 1) & 1], kc, vc, bt, kstart + (t + 1) * KT, kend, kvh, nkv, bs,
                         nblk, status);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      const int key0 = warp * 16;
      float s0[4], s1[4];
      qk16<HD>(s0, s1, qa, smem_u32(sk[t & 1]), key0);
      const int kbase = kstart + t * KT + key0 + (lane & 3) * 2;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kp = kbase + (i & 1);
        s0[i] = kp < kend ? s0[i] * scale_log2 : -INFINITY;
        s1[i] = kp + 8 < kend ? s1[i] * scale_log2 : -INFINITY;
      }
      softmax_pv<HD>(s0, s1, m, l, o, smem_u32(sv[t & 1]), key0);
      __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
      l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
    }
    __syncthreads();
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) {
      so[(warp * 16 + g) * HD + n * 8 + c2] = o[n][0];
      so[(warp * 16 + g) * HD + n * 8 + c2 + 1] = o[n][1];
      so[(warp * 16 + g + 8) * HD + n * 8 + c2] = o[n][2];
      so[(warp * 16 + g + 8) * HD + n * 8 + c2 + 1] = o[n][3];
    }
    if ((lane & 3) == 0) {
      sm[warp * 16 + g] = m[0];
      sm[warp * 16 + g + 8] = m[1];
      sl[warp * 16 + g] = l[0];
      sl[warp * 16 + g + 8] = l[1];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * HD; idx += NTHREADS) {
      const int r = idx / HD, d = idx % HD;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w * 16 + r]);
      const float Mu = M == -INFINITY ? 0.f : M;
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm[w * 16 + r] - Mu);
        L += sl[w * 16 + r] * f;
        O += so[(w * 16 + r) * HD + d] * f;
      }
      const int h = kvh * G + r;
      if (nsplits == 1) {
        out[((size_t)b * nh + h) * HD + d] = to_b(L > 0.f ? O / L : 0.f);
      } else {
        const size_t base = ((size_t)b * nh + h) * max_splits + split;
        part_o[base * HD + d] = O;
        if (d == 0) {
          part_ml[base * 2] = M;
          part_ml[base * 2 + 1] = L;
        }
      }
    }
    if (nsplits == 1) continue;
    // publish this split; the CTA that completes the last one merges them all
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      int* cnt = counters + (size_t)b * nkv + kvh;
      const int prev = atomicAdd(cnt, 1);
      is_last = prev == nsplits - 1;
      if (is_last) *cnt = 0;
    }
    __syncthreads();
    if (!is_last) continue;
    __threadfence();
    for (int idx = threadIdx.x; idx < G * HD; idx += NTHREADS) {
      const int r = idx / HD, d = idx % HD;
      const int h = kvh * G + r;
      const size_t base = ((size_t)b * nh + h) * max_splits;
      float M = -INFINITY;
      for (int sp = 0; sp < nsplits; ++sp) M = fmaxf(M, __ldcg(&part_ml[(base + sp) * 2]));
      const float Mu = M == -INFINITY ? 0.f : M;
      float L = 0.f, O = 0.f;
      for (int sp = 0; sp < nsplits; ++sp) {
        const float f = exp2f(__ldcg(&part_ml[(base + sp) * 2]) - Mu);
        L += __ldcg(&part_ml[(base + sp) * 2 + 1]) * f;
        O += __ldcg(&part_o[(base + sp) * HD + d]) * f;
      }
      out[((size_t)b * nh + h) * HD + d] = to_b(L > 0.f ? O / L : 0.f);
    }
  }
}

// Dynamic shared memory of decode_kernel<hd>: two K/V tile stages, or the cross-warp merge buffer.
constexpr int decode_smem(int hd) { return 4 * KT * hd * 2 > (4 * 16 * hd + 128) * 4 ? 4 * KT * hd * 2 : (4 * 16 * hd + 128) * 4; }

}  // namespace
}  // namespace lsb
