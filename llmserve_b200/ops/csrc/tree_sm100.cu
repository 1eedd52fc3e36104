// Tree-verify attention (EAGLE3 tree speculation) on the 5th-generation tensor cores.
//
// The reference verifies a draft tree with one masked attention over [prefix keys | tree keys]
// (`llmserve/layers/attention.py:77-109`, SDPA with an ancestor mask).  Here the query rows of one
// KV head -- every (tree node, query head of the group) pair, node-major, row = node * G + head --
// share ONE 128-row UMMA tile, so each K/V byte is read once per KV head, not once per query head,
// and a tree of up to 128 / G nodes costs one tile.
//
// Keys: the committed prefix in the paged pool [blocks, kv_heads, block_size, head_dim] (visible to
// every node) followed by one tile of tree keys from the side buffers [n_tree, kv_heads, head_dim]
// under each node's ancestor bitmask.  The key tiles are split into chunks over the CTAs (grid =
// kv heads x chunks, so a long prefix still fills the SMs); each chunk stores its unnormalised O
// with its running max and sum, and tree_merge_kernel combines the chunks (log-sum-exp).  With a
// single chunk the CTA writes the output itself.
//
//   warp 4         : producer.  Prefix tiles: lane 0 issues 2-D tensor copies of K and V (128B
//                    swizzle, boxes of min(block_size, 64) keys, so pages need not be contiguous)
//                    into a 3-stage ring.  The tree tile: the warp copies the side-buffer rows into
//                    the same swizzled layout with plain loads and stores (rows past n_tree zeroed),
//                    fences the async proxy and arrives on the stage's barrier.
//   warp 5         : allocates 256 TMEM columns (O, two S buffers); lane 0 issues S = Q K^T two
//                    tiles ahead and O += P V (P K-major from shared memory, V MN-major from its
//                    tile), and frees a stage once its PV is done.
//   warps 0..3     : thread r owns tile row r.  It first writes its query row into the K-major
//                    Q tile, then runs the online softmax of the prefill kernel: tcgen05.ld of 64
//                    raw scores, mask (prefix end, bad blocks, ancestor bits; interior prefix
//                    tiles unmasked), one FFMA + ex2 per score, the running max moved only when it
//                    grows by more than 2^8 (O rescaled in TMEM then), P as bf16 into the swizzled
//                    P tile.  V rows of keys nobody may see are zeroed before the PV.
// Every wait is bounded; a timeout records an error code and raises a CTA-wide abort flag that
// every role polls, in-flight copies and MMAs are drained and TMEM is freed.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "umma.cuh"

namespace lsb {

const CUtensorMap& kv_pool_map(const at::Tensor& pool, int box_rows);
int* status_ptr(const at::Tensor& status);

namespace {

using namespace umma;

#define LSB_CHECK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

constexpr int kTRows = 128;      // tile rows (UMMA M): (node, head) pairs of one KV head
constexpr int kTKeys = 64;       // keys per K/V tile
constexpr int kTStages = 3;      // K/V ring depth
constexpr int kTThreads = 192;   // 4 softmax warps + producer warp + MMA warp
constexpr int kMaxTreeKeys = 32; // ancestor masks are 32-bit words
constexpr float kTRescaleLog2 = 8.f;
constexpr float kTLog2e = 1.4426950408889634f;

template <int HD>
struct TrLayout {
  static constexpr int kHalves = HD / 64;                // 128-byte column halves
  static constexpr int kQHalf = kTRows * 128;            // 16 KiB
  static constexpr int kQTile = kHalves * kQHalf;
  static constexpr int kKVHalf = kTKeys * 128;           // 8 KiB
  static constexpr int kTile = kHalves * kKVHalf;        // K (or V) of one stage
  static constexpr int kStage = 2 * kTile;
  static constexpr int kKVOff = kQTile;
  static constexpr int kPOff = kKVOff + kTStages * kStage;
  static constexpr int kPBytes = kTRows * kTKeys * 2;    // 16 KiB, one 128-byte row per tile row
  static constexpr int kBarOff = kPOff + kPBytes;
  static constexpr int kBytes = kBarOff + 256 + 1024;    // barriers + alignment slack
  static constexpr int kTmemCols = 256;                  // O at column 0, S buffers at 128 + 64 b
};

template <int HD>
__global__ void __launch_bounds__(kTThreads, 1) tree_tc_kernel(
    const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, bf16* __restrict__ out,
    float* __restrict__ part_o, float* __restrict__ part_ml, const bf16* __restrict__ q, const int* __restrict__ bt,
    int bt_len, int prefix_len, const bf16* __restrict__ tk, const bf16* __restrict__ tv, int n_tree,
    const int* __restrict__ mask_bits, int n_q, float scale_log2, int nh, int nkv, int bs, int box_keys, int nblk,
    int tiles_per_chunk, int* __restrict__ status) {
  using L = TrLayout<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;                   // 1 (one arrival per softmax warp)
  uint64_t* full = bars + 1;                 // kTStages
  uint64_t* empty = full + kTStages;         // kTStages
  uint64_t* s_full = empty + kTStages;       // 2 (S buffers)
  uint64_t* s_free = s_full + 2;             // 2
  uint64_t* p_full = s_free + 2;             // 1
  uint64_t* o_done = p_full + 1;             // 1 (one phase per PV)
  uint64_t* drain = o_done + 1;              // 1 -> 14 barriers, 112 bytes
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBarOff + 112);
  uint64_t* bad_keys = reinterpret_cast<uint64_t*>(smem + L::kBarOff + 128);   // kTStages masks
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;

  pdl_trigger();
  pdl_wait();
  const int kvh = blockIdx.x, chunk = blockIdx.y, nchunks = gridDim.y;
  const int G = nh / nkv, R = n_q * G;
  const int prefix = max(0, min(prefix_len, bt_len * bs));
  const int np = (prefix + kTKeys - 1) / kTKeys;          // prefix tiles; the tree tile is tile np
  const int total = np + (n_tree > 0 ? 1 : 0);
  const int j0 = chunk * tiles_per_chunk;
  const int nloc = max(0, min(total, j0 + tiles_per_chunk) - j0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(q_full, 4);
    for (int s = 0; s < kTStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------- producer ----------------
    int issued[kTStages] = {};
    for (int jl = 0; jl < nloc; ++jl) {
      const int j = j0 + jl, s = jl % kTStages, u = jl / kTStages;
      if (u >= 1 &&
          !__all_sync(0xffffffffu, wait_phase(&empty[s], (u - 1) & 1, abort_v, status, kTimeoutSmemEmpty)))
        break;
      uint8_t* kst = smem + L::kKVOff + s * L::kStage;
      uint8_t* vst = kst + L::kTile;
      if (j < np) {
        if (lane == 0) {
          const int k0 = j * kTKeys;
          const int segs = kTKeys / box_keys;
          uint64_t bad = 0;
          int rows[kTKeys / 8];
          for (int g = 0; g < segs; ++g) {
            const int kp = k0 + g * box_keys;
            int blk = 0;
            if (kp < prefix) {
              blk = bt[kp / bs];
              if (blk < 0 || blk >= nblk) {   // never dereferenced: block 0 is read and the keys masked
                record_error(status, kBadIndex);
                blk = 0;
                bad |= (box_keys == 64 ? ~0ull : (((1ull << box_keys) - 1) << (g * box_keys)));
              }
            }
            rows[g] = (blk * nkv + kvh) * bs + kp % bs;
          }
          bad_keys[s] = bad;   // published to the softmax warps by the arrival below
          mbar_expect_tx(&full[s], 2 * L::kTile);
          for (int g = 0; g < segs; ++g)
#pragma unroll
            for (int hf = 0; hf < L::kHalves; ++hf) {
              tma_2d(kst + hf * L::kKVHalf + g * box_keys * 128, &tm_k, &full[s], hf * 64, rows[g]);
              tma_2d(vst + hf * L::kKVHalf + g * box_keys * 128, &tm_v, &full[s], hf * 64, rows[g]);
            }
        }
      } else {
        // the tree tile: side-buffer rows into the swizzled layout, rows past n_tree zeroed
        constexpr int CH = L::kHalves * 8;   // 16-byte chunks per key row
        for (int idx = lane; idx < kTKeys * CH; idx += 32) {
          const int key = idx / CH, rem = idx % CH, hf = rem / 8, ch = rem % 8;
          uint4 kv = make_uint4(0, 0, 0, 0), vv = kv;
          if (key < n_tree) {
            const size_t off = ((size_t)key * nkv + kvh) * HD + hf * 64 + ch * 8;
            kv = *reinterpret_cast<const uint4*>(tk + off);
            vv = *reinterpret_cast<const uint4*>(tv + off);
          }
          const int so = hf * L::kKVHalf + key * 128 + ((ch ^ (key & 7)) << 4);
          *reinterpret_cast<uint4*>(kst + so) = kv;
          *reinterpret_cast<uint4*>(vst + so) = vv;
        }
        if (lane == 0) bad_keys[s] = 0ull;
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
      }
      issued[s] = u + 1;
    }
    // drain: every stage's most recent fill has landed before this CTA may exit
    if (lane == 0)
      for (int s = 0; s < kTStages; ++s)
        if (issued[s] > 0) mbar_wait(&full[s], (issued[s] - 1) & 1);
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && nloc > 0) {
      constexpr uint32_t id_s = idesc_f16(kTRows, kTKeys, false);
      constexpr uint32_t id_pv = idesc_f16(kTRows, HD, true);
      const uint32_t q_addr = smem_u32(smem);
      bool ok = wait_phase(q_full, 0, abort_v, status, kTimeoutTmaFull);
      auto issue_s = [&](int jl) -> bool {
        const int s = jl % kTStages, u = jl / kTStages, b = jl & 1, ub = jl >> 1;
        if (!wait_phase(&full[s], u & 1, abort_v, status, kTimeoutTmaFull)) return false;
        if (ub >= 1 && !wait_phase(&s_free[b], (ub - 1) & 1, abort_v, status, kTimeoutAccum)) return false;
        fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kKVOff + s * L::kStage);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int hf = kk / 4, c = kk % 4;
          mma(tmem + 128 + b * kTKeys, desc_kmajor(q_addr + hf * L::kQHalf + c * 32),
              desc_kmajor(k_addr + hf * L::kKVHalf + c * 32), id_s, kk != 0);
        }
        commit(&s_full[b]);
        return true;
      };
      auto issue_pv = [&](int jl) -> bool {
        const int s = jl % kTStages;
        if (!wait_phase(p_full, jl & 1, abort_v, status, kTimeoutAccum)) return false;
        fence_after();
        const uint32_t p_addr = smem_u32(smem + L::kPOff);
        const uint32_t v_addr = smem_u32(smem + L::kKVOff + s * L::kStage + L::kTile);
#pragma unroll
        for (int kk = 0; kk < kTKeys / 16; ++kk)
          mma(tmem, desc_kmajor(p_addr + kk * 32), desc_mnmajor(v_addr + kk * 16 * 128, L::kKVHalf), id_pv,
              (jl | kk) != 0);
        commit(o_done);
        commit(&empty[s]);   // K and V of this stage are no longer read
        return true;
      };
      for (int jl = 0; ok && jl < 2 && jl < nloc; ++jl) ok = issue_s(jl);
      for (int jl = 0; ok && jl < nloc; ++jl) {
        ok = issue_pv(jl);
        if (ok && jl + 2 < nloc) ok = issue_s(jl + 2);
      }
      // every MMA this thread issued has completed before the CTA tears down
      commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: thread r owns tile row r = (node r / G, head r % G) ----------------
    const int r = warp * 32 + lane;
    const bool row_ok = r < R;
    const int node = row_ok ? r / G : 0;
    const int head = kvh * G + (row_ok ? r - node * G : 0);
    {
      const bf16* qrow = q + ((size_t)node * nh + head) * HD;
#pragma unroll
      for (int hf = 0; hf < L::kHalves; ++hf)
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const uint4 v = row_ok ? *reinterpret_cast<const uint4*>(qrow + hf * 64 + ch * 8) : make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(smem + hf * L::kQHalf + r * 128 + ((ch ^ (r & 7)) << 4)) = v;
        }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }
    const uint32_t bits = row_ok ? (uint32_t)mask_bits[node] : 0u;
    const bool warp_rows_ok = warp * 32 + 31 < R;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t tmem_o = tmem + lane_base;
    const uint32_t tmem_s = tmem + 128 + lane_base;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // every wait is made warp-uniform (tcgen05.ld / st are warp-collective)
#define LSB_WAIT_ALL(bar, par, code)                                                   \
  if (!__all_sync(0xffffffffu, wait_phase(bar, par, abort_v, status, code))) {         \
    ok = false;                                                                        \
    break;                                                                             \
  }
    for (int jl = 0; jl < nloc; ++jl) {
      const int j = j0 + jl, s = jl % kTStages, u = jl / kTStages, b = jl & 1, ub = jl >> 1;
      LSB_WAIT_ALL(&s_full[b], ub & 1, kTimeoutAccum);
      fence_after();
      uint32_t raw[kTKeys];
#pragma unroll
      for (int c = 0; c < kTKeys; c += 16) tmem_ld16(tmem_s + b * kTKeys + c, raw + c);
      tmem_wait_ld();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);
      LSB_WAIT_ALL(&full[s], u & 1, kTimeoutTmaFull);   // publishes bad_keys[s]
      const uint64_t bad = bad_keys[s];
      const bool tree_tile = j >= np;
      const int k0 = j * kTKeys;
      const bool interior = !tree_tile && bad == 0ull && k0 + kTKeys <= prefix && warp_rows_ok;
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
      if (interior) {
#pragma unroll
        for (int c = 0; c < kTKeys; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(raw[c]));
      } else {
#pragma unroll
        for (int c = 0; c < kTKeys; ++c) {
          const bool valid = row_ok && (tree_tile ? (c < n_tree && ((bits >> (c & 31)) & 1u))
                                                  : (k0 + c < prefix && !((bad >> c) & 1ull)));
          if (!valid) raw[c] = __float_as_uint(-INFINITY);
          mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(raw[c]));
        }
      }
      const float mx_raw = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                 fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float mx = mx_raw * scale_log2;      // scale > 0: max commutes with the scaling
      float alpha = 1.f;
      if (mx > m_used + kTRescaleLog2) {
        alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
        m_used = mx;
        l *= alpha;
      }
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;   // a fully masked row: all P = 0
      uint32_t pw[kTKeys / 2];
      float sum8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) sum8[e] = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < kTKeys / 8; ++c8) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = ex2(fmaf(__uint_as_float(raw[c8 * 8 + e]), scale_log2, neg_m));   // ex2(-inf) = 0
          sum8[e] += p[e];
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) pw[c8 * 4 + e] = pack2_bf16(p[2 * e], p[2 * e + 1]);
      }
      l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      if (jl >= 1) {
        LSB_WAIT_ALL(o_done, (jl - 1) & 1, kTimeoutAccum);   // the previous PV read the P tile
      }
      uint8_t* prow = smem + L::kPOff + r * 128;
#pragma unroll
      for (int c8 = 0; c8 < kTKeys / 8; ++c8)
        *reinterpret_cast<uint4*>(prow + ((c8 ^ (r & 7)) << 4)) =
            make_uint4(pw[c8 * 4], pw[c8 * 4 + 1], pw[c8 * 4 + 2], pw[c8 * 4 + 3]);
      // zero the V rows of prefix keys nobody may see (past the prefix, or from a bad block)
      if (!tree_tile && (k0 + kTKeys > prefix || bad != 0ull)) {
        uint8_t* vt = smem + L::kKVOff + s * L::kStage + L::kTile;
        for (int idx = r; idx < kTKeys * L::kHalves * 8; idx += kTRows) {
          const int key = idx / (L::kHalves * 8), rem = idx % (L::kHalves * 8);
          const int hf = rem / 8, ch = rem % 8;
          if (k0 + key >= prefix || ((bad >> key) & 1ull))
            *reinterpret_cast<uint4*>(vt + hf * L::kKVHalf + key * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_async_smem();
      // rescale O in TMEM when some row of this warp moved its max (the previous PV is done)
      if (jl > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        fence_after();
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
          uint32_t o[16];
          tmem_ld16(tmem_o + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st16(tmem_o + c, o);
        }
        tmem_wait_st();
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
#undef LSB_WAIT_ALL
    bf16* orow = out + ((size_t)node * nh + head) * HD;
    const size_t prow_idx = ((size_t)chunk * nkv + kvh) * kTRows + r;
    if (ok && nloc > 0 &&
        __all_sync(0xffffffffu, wait_phase(o_done, (nloc - 1) & 1, abort_v, status, kTimeoutAccum))) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < HD; c += 16) {
        uint32_t o[16];
        tmem_ld16(tmem_o + c, o);
        tmem_wait_ld();
        if (!row_ok) continue;
        if (nchunks == 1) {
          uint4 w0, w1;
          w0.x = pack2_bf16(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv);
          w0.y = pack2_bf16(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv);
          w0.z = pack2_bf16(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv);
          w0.w = pack2_bf16(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv);
          w1.x = pack2_bf16(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv);
          w1.y = pack2_bf16(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv);
          w1.z = pack2_bf16(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv);
          w1.w = pack2_bf16(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv);
          *reinterpret_cast<uint4*>(orow + c) = w0;
          *reinterpret_cast<uint4*>(orow + c + 8) = w1;
        } else {
          float4* dst = reinterpret_cast<float4*>(part_o + prow_idx * HD + c);
#pragma unroll
          for (int e = 0; e < 4; ++e)
            dst[e] = make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                 __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
        }
      }
      if (row_ok && nchunks > 1) {
        part_ml[prow_idx * 2] = m_used;
        part_ml[prow_idx * 2 + 1] = l;
      }
    } else if (ok && nloc == 0 && row_ok) {
      // no keys in this chunk: an empty partial state (or zeros when it is the only chunk)
      if (nchunks == 1) {
        for (int c = 0; c < HD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
      } else {
        for (int c = 0; c < HD; c += 4) *reinterpret_cast<float4*>(part_o + prow_idx * HD + c) = make_float4(0, 0, 0, 0);
        part_ml[prow_idx * 2] = -INFINITY;
        part_ml[prow_idx * 2 + 1] = 0.f;
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 5) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kTmemCols));
  }
}

// Log-sum-exp merge of the chunks' partial states: one CTA per (kv head, tile row), a thread per
// head dimension.
template <int HD>
__global__ void tree_merge_kernel(bf16* __restrict__ out, const float* __restrict__ part_o,
                                  const float* __restrict__ part_ml, int nchunks, int nh, int nkv) {
  pdl_trigger();
  pdl_wait();
  const int kvh = blockIdx.x, r = blockIdx.y, G = nh / nkv;
  const int node = r / G, head = kvh * G + r - node * G;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int c = 0; c < nchunks; ++c) M = fmaxf(M, part_ml[(((size_t)c * nkv + kvh) * kTRows + r) * 2]);
  const float Mu = M == -INFINITY ? 0.f : M;
  float Lsum = 0.f, O = 0.f;
  for (int c = 0; c < nchunks; ++c) {
    const size_t i = ((size_t)c * nkv + kvh) * kTRows + r;
    const float f = exp2f(part_ml[i * 2] - Mu);
    Lsum += part_ml[i * 2 + 1] * f;
    O += part_o[i * HD + d] * f;
  }
  out[((size_t)node * nh + head) * HD + d] = to_b(Lsum > 0.f ? O / Lsum : 0.f);
}

int sm_count_tree() {
  static int n = [] {
    int dev = 0, v = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v;
  }();
  return n;
}

}  // namespace

// Whether the tensor-core tree kernel takes this shape: all (node, head) rows of a KV head in one
// 128-row tile, at most 32 tree keys (one ancestor word per node), a TMA-tileable block size.
bool tree_tc_supported(int64_t n_q, int64_t nh, int64_t nkv, int64_t n_tree, int64_t block_size, int64_t head_dim) {
  return (head_dim == 64 || head_dim == 128) && nkv > 0 && nh % nkv == 0 && n_q * (nh / nkv) <= kTRows &&
         n_tree <= kMaxTreeKeys && block_size % 8 == 0 && (block_size % 64 == 0 || 64 % block_size == 0);
}

// out / q: bf16 [n_q, nh, hd]; pools [blocks, kv_heads, block_size, hd]; bt int32 [table length]
// (one sequence); tk / tv bf16 [n_tree, kv_heads, hd]; mask_bits int32 [n_q]: bit t of node i set
// when node i may see tree key t.
void tree_attention_tc(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor bt, int64_t prefix_len,
                       at::Tensor tk, at::Tensor tv, at::Tensor mask_bits, double scale, at::Tensor status) {
  LSB_CHECK(q.dim() == 3 && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q must be contiguous bf16 [n, nh, hd]");
  LSB_CHECK(out.sizes() == q.sizes() && out.is_contiguous() && out.scalar_type() == at::kBFloat16, "bad output");
  LSB_CHECK(kc.dim() == 4 && vc.sizes() == kc.sizes() && kc.is_contiguous() && vc.is_contiguous() &&
                kc.scalar_type() == at::kBFloat16 && vc.scalar_type() == at::kBFloat16,
            "KV pools must be contiguous bf16 [blocks, kv_heads, block_size, head_dim]");
  const int n_q = q.size(0), nh = q.size(1), hd = q.size(2), nkv = kc.size(1), bs = kc.size(2);
  const int n_tree = tk.numel() ? tk.size(0) : 0;
  LSB_CHECK(kc.size(3) == hd, "head dim mismatch");
  LSB_CHECK(n_tree == 0 || (tk.dim() == 3 && tk.size(1) == nkv && tk.size(2) == hd && tk.is_contiguous() &&
                            tv.sizes() == tk.sizes() && tv.is_contiguous() && tk.scalar_type() == at::kBFloat16 &&
                            tv.scalar_type() == at::kBFloat16),
            "tree keys / values must be contiguous bf16 [n_tree, kv_heads, head_dim]");
  LSB_CHECK(mask_bits.scalar_type() == at::kInt && mask_bits.numel() == n_q, "mask_bits must be int32 [n]");
  LSB_CHECK(bt.scalar_type() == at::kInt && bt.is_contiguous(), "block table must be contiguous int32");
  LSB_CHECK(prefix_len >= 0, "negative prefix length");
  LSB_CHECK(tree_tc_supported(n_q, nh, nkv, n_tree, bs, hd), "shape unsupported by the tensor-core tree kernel");
  LSB_CHECK((int64_t)kc.numel() / hd < (int64_t)INT32_MAX, "KV pool rows exceed int32");
  if (n_q == 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  const int bt_len = bt.numel();
  const int64_t prefix = std::min<int64_t>(prefix_len, (int64_t)bt_len * bs);
  const int total = (int)((prefix + kTKeys - 1) / kTKeys) + (n_tree > 0 ? 1 : 0);
  if (total == 0) {
    out.zero_();
    return;
  }
  // chunks of the key tiles: at most one (kv head, chunk) CTA per SM, one wave
  int chunks = std::min(total, std::max(1, sm_count_tree() / nkv));
  const int per = (total + chunks - 1) / chunks;
  chunks = (total + per - 1) / per;
  at::Tensor part_o, part_ml;
  if (chunks > 1) {
    part_o = at::empty({(int64_t)chunks * nkv * kTRows * hd}, q.options().dtype(at::kFloat));
    part_ml = at::empty({(int64_t)chunks * nkv * kTRows * 2}, q.options().dtype(at::kFloat));
  }
  float* po = chunks > 1 ? part_o.data_ptr<float>() : nullptr;
  float* pml = chunks > 1 ? part_ml.data_ptr<float>() : nullptr;
  const int box_keys = bs >= 64 ? 64 : bs;
  const CUtensorMap& tm_k = kv_pool_map(kc, box_keys);
  const CUtensorMap& tm_v = kv_pool_map(vc, box_keys);
  const bf16* tkp = n_tree ? (const bf16*)tk.data_ptr() : nullptr;
  const bf16* tvp = n_tree ? (const bf16*)tv.data_ptr() : nullptr;
  const float sl = (float)scale * kTLog2e;
  const int R = n_q * (nh / nkv);
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status_ptr(status);
#define LSB_TREE_TC(HD)                                                                                           \
  do {                                                                                                            \
    const int smem = TrLayout<HD>::kBytes;                                                                        \
    ensure_dynamic_smem((const void*)tree_tc_kernel<HD>, smem);                                                  \
    launch_pdl(tree_tc_kernel<HD>, dim3(nkv, chunks), dim3(kTThreads), smem, stream, tm_k, tm_v,                   \
               (bf16*)out.data_ptr(), po, pml, (const bf16*)q.data_ptr(), bt.data_ptr<int>(), bt_len,             \
               (int)prefix, tkp, tvp, n_tree, mask_bits.data_ptr<int>(), n_q, sl, nh, nkv, bs, box_keys,           \
               (int)kc.size(0), per, st);                                                                         \
    if (chunks > 1)                                                                                               \
      launch_pdl(tree_merge_kernel<HD>, dim3(nkv, R), dim3(HD), 0, stream, (bf16*)out.data_ptr(),                  \
                 (const float*)po, (const float*)pml, chunks, nh, nkv);                                           \
  } while (0)
  if (hd == 128) LSB_TREE_TC(128);
  else LSB_TREE_TC(64);
#undef LSB_TREE_TC
  auto e = cudaGetLastError();
  LSB_CHECK(e == cudaSuccess, std::string("tree_tc launch failed: ") + cudaGetErrorString(e));
}

}  // namespace lsb
