// Paged decode attention fed by TMA: persistent CTAs (two per SM) stream K/V pages through a
// shared-memory ring while four consumer warps each run the GQA score / online-softmax / PV math.
//
// Work items are (chunk of `partition` keys, sequence, kv head), enumerated chunk-major and dealt
// round-robin to the CTAs; the producer's ring runs straight across item boundaries, so the HBM
// stream never drains between items (the earlier one-CTA-per-item kernel paid a pipeline fill
// per CTA and a partial last wave).
//
//   warp 4, lane 0 : producer (3-stage ring of 32 KiB for head_dim 128).  For each 64-key stage it issues 2-D tensor copies (128-byte
//                    swizzle, box 64 dims x min(block_size, 64) keys) of K and V straight out of
//                    the paged pool [blocks, kv_heads, block_size, head_dim], completing on the
//                    stage's "full" mbarrier.  Stages whose keys all precede the newest position
//                    are issued before griddepcontrol.wait, overlapping the QKV kernel.
//   warps 0..3     : consumers.  Warp w owns keys [16w, 16w+16) of each stage: S = Q K^T and
//                    O += P V on mma.sync m16n8k16 (the G query heads of one kv head fill rows of
//                    the 16-row A tile), online softmax in registers, then release the stage.
//                    At an item's end the four warps merge through shared memory; a context
//                    with several chunks writes fp32 partials and the CTA that finishes its last
//                    chunk (per-pair counter, reset by that CTA) combines them.
// Keys past the context inside the last stage are masked in S and their V rows are zeroed in
// shared memory (the copy brings whatever the page holds there).  Every wait is bounded and
// records an error code in `status` on timeout; no named barrier is used (the consumer warps
// synchronise through an mbarrier), so a timed-out role cannot strand the others.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "attention_tiles.cuh"

namespace lsb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
int* status_ptr(const at::Tensor& status);

namespace {

constexpr int kDecKeys = 64;       // keys per stage
constexpr int kDecThreads = 160;   // 4 consumer warps + 1 producer warp

// Shared memory: [stages x (K tile | V tile)] [barriers] [merge buffer: o (4 warps x G rows x HD)
// + m, l (4 warps x 16 rows)].  Sized so two CTAs fit on one SM for G <= 8 (8 consumer warps per
// SM hide each other's mma / global latency).
// ST: ring depth (default 96 KiB of ring for either head dim); a verify chunk (up to 16 tile rows)
// has a 4x larger merge buffer and takes one stage less so that two CTAs still fit per SM.
template <int HD, int ST = (HD == 128 ? 3 : 6)>
struct DecLayout {
  static constexpr int kHalves = HD / 64;                    // 128-byte column halves
  static constexpr int kHalfBytes = kDecKeys * 128;          // 8 KiB
  static constexpr int kTileBytes = kHalves * kHalfBytes;    // K (or V) of one stage
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kStages = ST;
  static constexpr int kBarOff = kStages * kStageBytes;
  static constexpr int kMergeOff = kBarOff + 128;
  static int smem_bytes(int G) { return kMergeOff + (4 * G * HD + 2 * 64) * 4 + 1024; }
};

// Byte offset of 16-byte chunk c of key row r in a stage tile written by a 128B-swizzled copy:
// column halves are separate 64-row x 128-byte regions; chunk bits are XORed with row bits.
template <int HD>
__device__ __forceinline__ uint32_t tsw(int r, int c) {
  return (uint32_t)((c >> 3) * DecLayout<HD>::kHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

template <int HD>
__device__ __forceinline__ void qk16_t(float* s0, float* s1, const uint32_t (*qa)[4], uint32_t sk, int key0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 4; ++i) s0[i] = s1[i] = 0.f;
  const int key = key0 + ((lane >> 4) << 3) + (lane & 7);
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4(b0, b1, b2, b3, sk + tsw<HD>(key, kk * 2 + ((lane >> 3) & 1)));
    mma16816(s0, qa[kk], b0, b1);
    mma16816(s1, qa[kk], b2, b3);
  }
}

template <int HD>
__device__ __forceinline__ void softmax_pv_t(float* s0, float* s1, float* m, float* l, float (*o)[4], uint32_t sv,
                                             int key0) {
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
  const int key = key0 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
  for (int dt = 0; dt < HD / 16; ++dt) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(b0, b1, b2, b3, sv + tsw<HD>(key, dt * 2 + (lane >> 4)));
    mma16816(o[2 * dt], a, b0, b1);
    mma16816(o[2 * dt + 1], a, b2, b3);
  }
}

__device__ __forceinline__ void tma2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Consumer-group barrier (4 warps) on an mbarrier: bounded, unlike a named barrier.
__device__ __forceinline__ bool group_sync(uint64_t* bar, uint32_t& phase, int* status) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_local(bar);
  const bool ok = mbar_wait(bar, phase);
  phase ^= 1u;
  __syncwarp();
  if (!ok) record_error(status, kTimeoutAccum);
  return ok;
}

template <int HD, int ST>
__global__ void __launch_bounds__(kDecThreads, 2) decode_tma_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, bf16* __restrict__ out,
    const bf16* __restrict__ q, const int* __restrict__ block_tables, int bt_stride,
    const int* __restrict__ context_lens, float scale_log2, float* __restrict__ part_o, float* __restrict__ part_ml,
    int* __restrict__ counters, int max_splits, int partition, int max_chunks, int B, int nh, int nkv, int bs,
    int box_rows, int nblk, int nq, int* __restrict__ status) {
  using LY = DecLayout<HD, ST>;
  constexpr int S = LY::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + LY::kBarOff);
  uint64_t* empty = full + S;
  uint64_t* group = empty + S;
  __shared__ int is_last;
  __shared__ int abort_flag;
  volatile int* aborted = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = nh / nkv;
  const int pairs = B * nkv;
  const int n_items = max_chunks * pairs;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    mbar_init(group, 4);
    fence_barrier_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_k) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_v) : "memory");
  }
  __syncthreads();
  pdl_trigger();

  if (warp == 4) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int it = 0, last[S];
      for (int s = 0; s < S; ++s) last[s] = -1;
      bool waited = false;
      for (int item = blockIdx.x; item < n_items && !*aborted; item += gridDim.x) {
        const int chunk = item / pairs, pair = item - chunk * pairs;
        const int b = pair / nkv, kvh = pair - b * nkv;
        const int ctx = max(0, min(context_lens[b], bt_stride * bs));   // clamped to the table row
        const int ks = chunk * partition;
        if (ks >= ctx) continue;
        const int ke = min(ks + partition, ctx);
        const int* bt = block_tables + (size_t)b * bt_stride;
        for (int st = ks; st < ke; st += kDecKeys, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1)) {
            record_error(status, kTimeoutSmemEmpty);
            *aborted = 1;
            break;
          }
          // the previous kernel writes the newest nq positions' K/V: wait for it before those stages
          if (!waited && st + kDecKeys > ctx - nq) {
            pdl_wait();
            waited = true;
          }
          const int nsub = (min(kDecKeys, ke - st) + box_rows - 1) / box_rows;
          mbar_expect_tx(&full[s], (uint32_t)(nsub * box_rows * 128 * LY::kHalves * 2));
          const uint32_t kt = smem_u32(smem + s * LY::kStageBytes);
          const uint32_t vt = kt + LY::kTileBytes;
          for (int j = 0; j < nsub; ++j) {
            const int pos = st + j * box_rows;
            int blk = bt[pos / bs];
            if ((unsigned)blk >= (unsigned)nblk) {
              // never dereferenced: a row past the pool is outside the tensor map, so the copy
              // delivers zeros (and still completes its transaction bytes)
              record_error(status, kBadIndex);
              blk = nblk;
            }
            const int row = (blk * nkv + kvh) * bs + pos % bs;
#pragma unroll
            for (int h = 0; h < LY::kHalves; ++h) {
              tma2d(kt + h * LY::kHalfBytes + j * box_rows * 128, &tm_k, &full[s], h * 64, row);
              tma2d(vt + h * LY::kHalfBytes + j * box_rows * 128, &tm_v, &full[s], h * 64, row);
            }
          }
          last[s] = it;
        }
      }
      if (!waited) pdl_wait();
      // tail (bounded): leave only after every issued stage has landed and been consumed
      for (int s = 0; s < S; ++s) {
        if (last[s] < 0) continue;
        const uint32_t use = (uint32_t)(last[s] / S);
        if (*aborted) mbar_wait(&full[s], use & 1);
        else mbar_wait(&empty[s], use & 1);
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();
  float* so = reinterpret_cast<float*>(smem + LY::kMergeOff);   // [4 warps][nq * G rows][HD]
  float* sm = so + 4 * nq * G * HD;
  float* sl = sm + 64;
  const int g = lane >> 2, c2 = (lane & 3) * 2;
  const int R = nq * G;            // tile rows: (query i, head gg) at row i * G + gg
  uint32_t gphase = 0;
  int it = 0;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int chunk = item / pairs, pair = item - chunk * pairs;
    const int b = pair / nkv, kvh = pair - b * nkv;
    const int ctx = max(0, min(context_lens[b], bt_stride * bs));
    const int ks = chunk * partition;
    if (ks >= ctx) {
      if (chunk == 0 && warp == 0)   // empty context: defined output
        for (int i = lane; i < R * HD; i += 32) {
          const int r = i / HD, qi = nq == 1 ? 0 : r / G;
          out[((size_t)(b * nq + qi) * nh + kvh * G + r - qi * G) * HD + i % HD] = to_b(0.f);
        }
      continue;
    }
    const int ke = min(ks + partition, ctx);
    const int nchunks = (ctx + partition - 1) / partition;

    // this lane's two tile rows g and g + 8: (query, head) pairs and their query-row pointers,
    // worked out once per item (no division in the loops; nq = 1 is plain decode)
    const int qA = nq == 1 ? 0 : g / G, qB = nq == 1 ? 0 : (g + 8) / G;
    const bf16* qrA = g < R ? q + ((size_t)(b * nq + qA) * nh + kvh * G + (g - qA * G)) * HD : nullptr;
    const bf16* qrB = g + 8 < R ? q + ((size_t)(b * nq + qB) * nh + kvh * G + (g + 8 - qB * G)) * HD : nullptr;
    // query i of sequence b at absolute position ctx - nq + i sees keys [0, ctx - nq + i]
    const int limA = min(ke, ctx - nq + qA + 1), limB = min(ke, ctx - nq + qB + 1);
    uint32_t qa[HD / 16][4];
    {
      const int c = (lane & 3) * 2;
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const int col = kk * 16 + c;
        qa[kk][0] = qrA ? *reinterpret_cast<const uint32_t*>(qrA + col) : 0u;
        qa[kk][1] = qrB ? *reinterpret_cast<const uint32_t*>(qrB + col) : 0u;
        qa[kk][2] = qrA ? *reinterpret_cast<const uint32_t*>(qrA + col + 8) : 0u;
        qa[kk][3] = qrB ? *reinterpret_cast<const uint32_t*>(qrB + col + 8) : 0u;
      }
    }
    float o[HD / 8][4];
#pragma unroll
    for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    const int key0 = warp * 16;
    for (int st = ks; st < ke; st += kDecKeys, ++it) {
      const int s = it % S;
      if (!mbar_wait(&full[s], (it / S) & 1) || *aborted) {
        record_error(status, kTimeoutTmaFull);
        *aborted = 1;
        return;
      }
      const uint32_t kt = smem_u32(smem + s * LY::kStageBytes);
      const uint32_t vt = kt + LY::kTileBytes;
      const int valid = ke - st;   // keys of this stage inside the context (may exceed 64)
      const bool ragged = key0 + 16 > valid;
      if (ragged) {
        // zero this warp's V rows past the context so 0 * (stale bytes) cannot produce NaN
        const int r_begin = max(key0, valid);
        constexpr int CH = HD / 8;
        for (int idx = lane; idx < (key0 + 16 - r_begin) * CH; idx += 32) {
          const int r = r_begin + idx / CH, c = idx % CH;
          asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(vt + tsw<HD>(r, c)), "r"(0) : "memory");
        }
        __syncwarp();
      }
      float s0[4], s1[4];
      qk16_t<HD>(s0, s1, qa, kt, key0);
      const int kb = st + key0 + (lane & 3) * 2;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kp = kb + (i & 1);
        const int lim = i < 2 ? limA : limB;
        s0[i] = kp < lim ? s0[i] * scale_log2 : -INFINITY;
        s1[i] = kp + 8 < lim ? s1[i] * scale_log2 : -INFINITY;
      }
      softmax_pv_t<HD>(s0, s1, m, l, o, vt, key0);
      __syncwarp();
      if (lane == 0) {
        if (ragged) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_local(&empty[s]);
      }
    }
    // ---- merge the four warps' partial softmax states ----
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
      l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
    }
    if (!group_sync(group, gphase, status)) return;   // previous item's merge reads are done
    if (g < R) {
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        so[(warp * R + g) * HD + n * 8 + c2] = o[n][0];
        so[(warp * R + g) * HD + n * 8 + c2 + 1] = o[n][1];
      }
    }
    if (g + 8 < R) {
#pragma unroll
      for (int n = 0; n < HD / 8; ++n) {
        so[(warp * R + g + 8) * HD + n * 8 + c2] = o[n][2];
        so[(warp * R + g + 8) * HD + n * 8 + c2 + 1] = o[n][3];
      }
    }
    if ((lane & 3) == 0) {
      sm[warp * 16 + g] = m[0];
      sm[warp * 16 + g + 8] = m[1];
      sl[warp * 16 + g] = l[0];
      sl[warp * 16 + g + 8] = l[1];
    }
    if (!group_sync(group, gphase, status)) return;
    for (int idx = threadIdx.x; idx < R * HD; idx += 128) {
      const int r = idx / HD, d = idx % HD;
      const int qi = nq == 1 ? 0 : r / G;
      const size_t qrow = (size_t)b * nq + qi;      // output row of query qi
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < 4; ++w) M = fmaxf(M, sm[w * 16 + r]);
      const float Mu = M == -INFINITY ? 0.f : M;
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(sm[w * 16 + r] - Mu);
        L += sl[w * 16 + r] * f;
        O += so[(w * R + r) * HD + d] * f;
      }
      const int h = kvh * G + r - qi * G;
      if (nchunks == 1) {
        out[(qrow * nh + h) * HD + d] = to_b(L > 0.f ? O / L : 0.f);
      } else {
        const size_t base = (qrow * nh + h) * max_splits + chunk;
        part_o[base * HD + d] = O;
        if (d == 0) {
          part_ml[base * 2] = M;
          part_ml[base * 2 + 1] = L;
        }
      }
    }
    if (nchunks == 1) continue;
    // publish this chunk; the CTA that completes the last chunk of (b, kv head) merges them all
    __threadfence();
    if (!group_sync(group, gphase, status)) return;
    if (threadIdx.x == 0) {
      int* cnt = counters + (size_t)b * nkv + kvh;
      const int prev = atomicAdd(cnt, 1);
      is_last = prev == nchunks - 1;
      if (is_last) *cnt = 0;
    }
    if (!group_sync(group, gphase, status)) return;
    if (!is_last) continue;
    __threadfence();
    for (int idx = threadIdx.x; idx < R * HD; idx += 128) {
      const int r = idx / HD, d = idx % HD;
      const int qi = nq == 1 ? 0 : r / G;
      const size_t qrow = (size_t)b * nq + qi;
      const int h = kvh * G + r - qi * G;
      const size_t base = (qrow * nh + h) * max_splits;
      float M = -INFINITY;
      for (int sp = 0; sp < nchunks; ++sp) M = fmaxf(M, __ldcg(&part_ml[(base + sp) * 2]));
      const float Mu = M == -INFINITY ? 0.f : M;
      float L = 0.f, O = 0.f;
      for (int sp = 0; sp < nchunks; ++sp) {
        const float f = exp2f(__ldcg(&part_ml[(base + sp) * 2]) - Mu);
        L += __ldcg(&part_ml[(base + sp) * 2 + 1]) * f;
        O += __ldcg(&part_o[(base + sp) * HD + d]) * f;
      }
      out[(qrow * nh + h) * HD + d] = to_b(L > 0.f ? O / L : 0.f);
    }
  }
}

// A cached map is valid only for the exact geometry it was encoded with: a later pool allocated at
// the same address (the caching allocator reuses freed blocks) may have the same row count but a
// different head dim, so the key holds every parameter of the encoding.
struct PoolKey {
  const void* p;
  int64_t rows, hd;
  int box;
  bool operator==(const PoolKey& o) const { return p == o.p && rows == o.rows && hd == o.hd && box == o.box; }
};
struct PoolKeyHash {
  size_t operator()(const PoolKey& k) const {
    return std::hash<const void*>()(k.p) ^ (std::hash<int64_t>()(k.rows) * 31) ^ (std::hash<int64_t>()(k.hd) * 131) ^
           (size_t)k.box;
  }
};

// Tensor map over one layer's K or V pool viewed as [blocks * kv_heads * block_size, head_dim].
const CUtensorMap& pool_map(const at::Tensor& pool, int box_rows) {
  static std::unordered_map<PoolKey, CUtensorMap, PoolKeyHash> cache;
  static std::mutex mu;
  const int64_t hd = pool.size(3), rows = pool.numel() / hd;
  PoolKey key{pool.data_ptr(), rows, hd, box_rows};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, pool.data_ptr(), dims, strides, box, estr,
                                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "llmserve_b200: cuTensorMapEncodeTiled failed for the KV pool (", (int)r, ")");
  return cache.emplace(key, m).first->second;
}

int sm_count() {
  static int n = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

}  // namespace

// Tensor map over one layer's K or V pool viewed as [blocks * kv_heads * block_size, head_dim] with a
// (box_rows x 64 dims) box, 128B swizzle; cached per (pool, box).  Shared with the prefill kernel.
const CUtensorMap& kv_pool_map(const at::Tensor& pool, int box_rows) { return pool_map(pool, box_rows); }

// Whether decode_attention_tma supports this pool (block size and head dim).
bool decode_tma_supported(int64_t block_size, int64_t head_dim) {
  return (head_dim == 64 || head_dim == 128) && block_size % 8 == 0 && (block_size % 64 == 0 || 64 % block_size == 0);
}

// q / out: bf16 [B * nq, nh, hd] -- nq consecutive query rows per sequence (nq = 1: decode; nq > 1:
// a packed verify chunk at the last nq positions of each context, causal among themselves), with
// nq * (nh / nkv) <= 16 so all of a (sequence, kv head)'s rows share one MMA tile.
void decode_attention_tma(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_tables,
                          at::Tensor context_lens, double scale, at::Tensor part_o, at::Tensor part_ml,
                          at::Tensor counters, int64_t max_splits, int64_t partition, int64_t nq,
                          at::Tensor status) {
  TORCH_CHECK(kc.dim() == 4 && vc.sizes() == kc.sizes() && kc.is_contiguous() && vc.is_contiguous() &&
                  kc.scalar_type() == at::kBFloat16 && vc.scalar_type() == at::kBFloat16,
              "llmserve_b200: KV pools must be contiguous bf16 [blocks, kv_heads, block_size, head_dim]");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "llmserve_b200: q must be bf16 [B, nh, hd]");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "llmserve_b200: block_tables int32");
  TORCH_CHECK(context_lens.scalar_type() == at::kInt && counters.scalar_type() == at::kInt, "llmserve_b200: int32 lens/counters");
  TORCH_CHECK(nq >= 1 && q.size(0) % nq == 0, "llmserve_b200: q rows must be a multiple of nq");
  const int B = q.size(0) / nq, nh = q.size(1), hd = q.size(2), nkv = kc.size(1), bs = kc.size(2);
  TORCH_CHECK(kc.size(3) == hd && nh % nkv == 0 && nq * (nh / nkv) <= 16,
              "llmserve_b200: head layout unsupported (queries x group size <= 16)");
  TORCH_CHECK(decode_tma_supported(bs, hd), "llmserve_b200: block size / head dim unsupported by the TMA decode kernel");
  TORCH_CHECK(partition % kDecKeys == 0 && partition > 0, "llmserve_b200: partition must be a multiple of 64");
  const int64_t cap = block_tables.size(1) * (int64_t)bs;
  const int max_chunks = (int)((cap + partition - 1) / partition);
  TORCH_CHECK(max_chunks <= max_splits, "llmserve_b200: workspace has too few splits");
  TORCH_CHECK(part_o.numel() >= (int64_t)B * nq * nh * max_splits * hd &&
                  part_ml.numel() >= (int64_t)B * nq * nh * max_splits * 2,
              "llmserve_b200: decode workspace too small");
  TORCH_CHECK(counters.numel() >= (int64_t)B * nkv, "llmserve_b200: decode counters too small");
  TORCH_CHECK((int64_t)kc.numel() / hd < (int64_t)INT32_MAX, "llmserve_b200: KV pool rows exceed int32");
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  const int box_rows = bs >= 64 ? 64 : bs;
  const CUtensorMap& mk = pool_map(kc, box_rows);
  const CUtensorMap& mv = pool_map(vc, box_rows);
  const int64_t n_items = (int64_t)max_chunks * B * nkv;
  const int G = nh / nkv;
  const float sl = (float)scale * kLog2e;
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status_ptr(status);
#define LSB_DEC_TMA(HD, ST)                                                                                         \
  do {                                                                                                              \
    const int smem = DecLayout<HD, ST>::smem_bytes(G * (int)nq);                                                  \
    ensure_dynamic_smem((const void*)decode_tma_kernel<HD, ST>, smem);                                            \
    int per_sm = 1;                                                                                                 \
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_tma_kernel<HD, ST>, kDecThreads, smem);           \
    const int grid = (int)std::min<int64_t>(n_items, (int64_t)sm_count() * std::max(per_sm, 1));                   \
    launch_pdl(decode_tma_kernel<HD, ST>, dim3(grid), dim3(kDecThreads), smem, stream, mk, mv,                      \
               (bf16*)out.data_ptr(), (const bf16*)q.data_ptr(), block_tables.data_ptr<int>(),                      \
               (int)block_tables.size(1), context_lens.data_ptr<int>(), sl, part_o.data_ptr<float>(),               \
               part_ml.data_ptr<float>(), counters.data_ptr<int>(), (int)max_splits, (int)partition, max_chunks, B, \
               nh, nkv, bs, box_rows, (int)kc.size(0), (int)nq, st);                                                \
  } while (0)
  const bool wide = G * nq > 8;   // verify chunks: a 4x merge buffer, one ring stage less
  if (hd == 128) {
    if (wide) LSB_DEC_TMA(128, 2);
    else LSB_DEC_TMA(128, 3);
  } else {
    if (wide) LSB_DEC_TMA(64, 5);
    else LSB_DEC_TMA(64, 6);
  }
#undef LSB_DEC_TMA
}

}  // namespace lsb
