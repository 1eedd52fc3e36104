// Varlen causal prefill attention on the 5th-generation tensor cores: S = Q K^T and O += P V are
// tcgen05.mma with fp32 accumulators in TMEM, Q / K / V tiles arrive by TMA straight from the
// packed query rows and the paged pool [blocks, kv_heads, block_size, head_dim].
//
// One CTA computes two 128-row query tiles ("A" and "B", UMMA M = 128 each) of one head against
// shared 64-key K/V tiles, so the tensor pipe always has one tile's MMAs to run while the other
// tile's softmax warps work:
//   warps 8 / 10, lane 0 : TMA producers.  Warp 8: Q of both tiles once (64-column halves, 128B
//                    swizzle), then K of each 64-key tile into a 4-stage ring freed as soon as the
//                    tile's S MMAs are done; warp 10: V into a 3-stage ring freed after the PV MMAs.
//                    A K/V tile is assembled from per-block boxes of min(block_size, 64) keys, so
//                    pages need not be contiguous; loads run three to four tiles ahead.
//   warp 9, lane 0 : MMA issuer.  S_t(j) = Q_t K_j^T into one of two TMEM S buffers per tile (both
//                    operands K-major); O_t += P_t(j) V_j (P K-major from shared memory, V read
//                    MN-major straight from its TMA tile).  Order: PV_A(j), PV_B(j), then S_A(j+2),
//                    S_B(j+2) -- the S of the next tile is always computed ahead, so each softmax
//                    warpgroup runs its tiles back to back.
//   warps 0..3 / 4..7 : softmax of tile A / B.  Thread r of a warpgroup owns query row r (TMEM lane
//                    r): tcgen05.ld of its 64 raw scores, causal / length mask (edge tiles only),
//                    online softmax in the log2 domain with one FFMA + ex2 per score, P as bf16 into
//                    the tile's swizzled shared-memory P buffer (reused once the tile's previous PV
//                    completed).  The running max only moves when it grows by more than 2^8 (P stays
//                    <= 256, exact in fp32 sums), so rescaling O in TMEM (tcgen05.ld / st after the
//                    previous PV completed) is rare.  At the end the same threads read O from TMEM,
//                    divide by the row sum and store bf16.
// Keys past the context (or from a block id outside the pool, recorded as kBadIndex) get P = 0,
// and their V rows are zeroed in shared memory by every warpgroup that uses the tile before its PV,
// so whatever the pool holds there never reaches O.  Every wait is bounded; a timeout records an
// error code, raises a CTA-wide abort flag that every role polls, drains the copies and MMAs in
// flight and frees TMEM.
//
// Short query chunks (EAGLE3 verify, decode-sized chunks) stay on the mma.sync kernel in
// attention.cu: a 128-row tile would be mostly empty there.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "umma.cuh"

namespace lsb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
const CUtensorMap& kv_pool_map(const at::Tensor& pool, int box_rows);
int* status_ptr(const at::Tensor& status);

namespace {

#define LSB_CHECK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

constexpr int kBQ = 128;        // query rows per tile (UMMA M)
constexpr int kQTiles = 2;      // query tiles per CTA, one softmax warpgroup each
constexpr int kBKV = 64;        // keys per K/V tile
constexpr int kStagesK = 4;     // K ring depth (a K tile is free once both S MMAs of its tile are done)
constexpr int kStagesV = 3;     // V ring depth (a V tile is free once both PV MMAs of its tile are done)
constexpr int kThreads = 352;   // 8 softmax warps + K producer warp + MMA warp + V producer warp
constexpr float kRescaleLog2 = 8.f;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD>
struct PfLayout {
  static constexpr int kHalves = HD / 64;                 // 128-byte column halves
  static constexpr int kQHalf = kBQ * 128;                // 16 KiB
  static constexpr int kQTile = kHalves * kQHalf;
  static constexpr int kKVHalf = kBKV * 128;              // 8 KiB
  static constexpr int kTileBytes = kHalves * kKVHalf;    // K (or V) of one tile
  static constexpr int kPBytes = kBQ * kBKV * 2;          // 16 KiB, one 128-byte row per query
  static constexpr int kKOff = kQTiles * kQTile;
  static constexpr int kVOff = kKOff + kStagesK * kTileBytes;
  static constexpr int kPOff = kVOff + kStagesV * kTileBytes;
  static constexpr int kBarOff = kPOff + kQTiles * kPBytes;
  static constexpr int kBytes = kBarOff + 256 + 1024;     // barriers + alignment slack
  // TMEM columns: O_t at 128 t; S_t buffers at 256 + 128 t + 64 b
  static constexpr int kTmemCols = 512;
};

using namespace umma;
// kind::f16 instruction descriptor of this kernel's MMAs: M = 128 query rows, N, B major-ness.
__host__ __device__ constexpr uint32_t idesc(int n, bool b_mn_major) { return idesc_f16(kBQ, n, b_mn_major); }
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) { return pack2_bf16(a, b); }

template <int HD>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, bf16* __restrict__ out, const int* __restrict__ cu_q,
    const int* __restrict__ seqlens_k, const int* __restrict__ block_tables, int bt_stride, float scale_log2, int nh,
    int nkv, int bs, int box_keys, int pairs_per_seq, int num_seqs, int nblk, int* __restrict__ status) {
  using L = PfLayout<HD>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;                         // 1
  uint64_t* k_full = bars + 1;                     // kStagesK
  uint64_t* k_empty = k_full + kStagesK;           // kStagesK
  uint64_t* v_full = k_empty + kStagesK;           // kStagesV
  uint64_t* v_empty = v_full + kStagesV;           // kStagesV
  uint64_t* s_full = v_empty + kStagesV;           // [tile][buffer]: 4
  uint64_t* s_free = s_full + 4;                   // 4
  uint64_t* p_full = s_free + 4;                   // [tile]: 2
  uint64_t* o_done = p_full + 2;                   // [tile]: 2 (one phase per PV of the tile)
  uint64_t* drain = o_done + 2;                    // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);   // byte 224 of the barrier block (28 barriers)
  uint64_t* bad_keys = reinterpret_cast<uint64_t*>(smem + L::kBarOff + 232);   // kStagesV masks, to byte 256
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;

  pdl_trigger();
  pdl_wait();
  // heaviest tile pairs first: blockIdx.y enumerates (pair from the last, sequence)
  const int qp = pairs_per_seq - 1 - (int)blockIdx.y / num_seqs;
  const int seq = (int)blockIdx.y % num_seqs;
  const int h = blockIdx.x, kvh = h / (nh / nkv);
  const int q0 = cu_q[seq], q_len = cu_q[seq + 1] - q0;
  if (qp * kQTiles * kBQ >= q_len) return;
  const int k_len = min(seqlens_k[seq], bt_stride * bs);
  const int shift = seqlens_k[seq] - q_len;                  // absolute position of query row 0
  // per query tile: key range (causal) and number of K/V tiles; tile B may be empty
  int kend_t[kQTiles], nt[kQTiles];
#pragma unroll
  for (int t = 0; t < kQTiles; ++t) {
    const int first = (qp * kQTiles + t) * kBQ;
    const int last = min(q_len, first + kBQ) - 1;
    kend_t[t] = first < q_len ? max(0, min(k_len, shift + last + 1)) : 0;
    nt[t] = (kend_t[t] + kBKV - 1) / kBKV;
  }
  const int kend = max(kend_t[0], kend_t[1]);
  const int ntiles = max(nt[0], nt[1]);
  const int* bt = block_tables + (size_t)seq * bt_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < kStagesK; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kStagesV; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    for (int t = 0; t < kQTiles; ++t) {
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8 || warp == 10) {
    // ---------------- TMA producers: warp 8 Q and K, warp 10 V ----------------
    const bool is_k = warp == 8;
    if (lane == 0 && ntiles > 0) {
      if (is_k) {
        mbar_expect_tx(q_full, kQTiles * L::kQTile);
#pragma unroll
        for (int t = 0; t < kQTiles; ++t)
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
            tma_2d(smem + t * L::kQTile + hf * L::kQHalf, &tm_q, q_full, h * HD + hf * 64,
                   q0 + (qp * kQTiles + t) * kBQ);
      }
      const int nst = is_k ? kStagesK : kStagesV;
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      const CUtensorMap* map = is_k ? &tm_k : &tm_v;
      int issued[kStagesK] = {};
      for (int j = 0; j < ntiles; ++j) {
        const int s = j % nst, u = j / nst;
        if (u >= 1 && !wait_phase(&empty[s], (u - 1) & 1, abort_v, status, kTimeoutSmemEmpty)) break;
        uint8_t* stage = smem + (is_k ? L::kKOff : L::kVOff) + s * L::kTileBytes;
        const int k0 = j * kBKV;
        uint64_t bad = 0;
        const int segs = kBKV / box_keys;
        int rows[kBKV / 8];
        for (int g = 0; g < segs; ++g) {
          const int kp = k0 + g * box_keys;
          int blk = 0;
          if (kp < kend) {
            blk = bt[kp / bs];
            if (blk < 0 || blk >= nblk) {
              if (!is_k) record_error(status, kBadIndex);
              blk = 0;
              bad |= (box_keys == 64 ? ~0ull : (((1ull << box_keys) - 1) << (g * box_keys)));
            }
          }
          rows[g] = (blk * nkv + kvh) * bs + kp % bs;
        }
        if (!is_k) bad_keys[s] = bad;   // published to the softmax warps by the v_full arrival below
        mbar_expect_tx(&full[s], L::kTileBytes);
        for (int g = 0; g < segs; ++g)
#pragma unroll
          for (int hf = 0; hf < L::kHalves; ++hf)
            tma_2d(stage + hf * L::kKVHalf + g * box_keys * 128, map, &full[s], hf * 64, rows[g]);
        issued[s] = u + 1;
      }
      // drain: every stage's most recent copies have landed before this CTA may exit
      if (is_k) mbar_wait(q_full, 0);
      for (int s = 0; s < nst; ++s)
        if (issued[s] > 0) mbar_wait(&full[s], (issued[s] - 1) & 1);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t id_s = idesc(kBKV, false);
      constexpr uint32_t id_pv = idesc(HD, true);
      const uint32_t q_addr = smem_u32(smem);
      bool ok = wait_phase(q_full, 0, abort_v, status, kTimeoutTmaFull);
      // S_t(j) into buffer j & 1 of tile t
      auto issue_s = [&](int t, int j) -> bool {
        const int s = j % kStagesK, u = j / kStagesK, b = j & 1, ub = j >> 1;
        if (!wait_phase(&k_full[s], u & 1, abort_v, status, kTimeoutTmaFull)) return false;
        if (ub >= 1 && !wait_phase(&s_free[t * 2 + b], (ub - 1) & 1, abort_v, status, kTimeoutAccum)) return false;
        fence_after();
        const uint32_t k_addr = smem_u32(smem + L::kKOff + s * L::kTileBytes);
        const uint32_t qa = q_addr + t * L::kQTile;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int hf = kk / 4, c = kk % 4;
          mma(tmem + 256 + t * 128 + b * kBKV, desc_kmajor(qa + hf * L::kQHalf + c * 32),
              desc_kmajor(k_addr + hf * L::kKVHalf + c * 32), id_s, kk != 0);
        }
        commit(&s_full[t * 2 + b]);
        // the K tile is free once the S MMAs of every query tile that uses it are done
        if (t == kQTiles - 1 || j >= nt[kQTiles - 1]) commit(&k_empty[s]);
        return true;
      };
      // O_t += P_t(j) V_j
      auto issue_pv = [&](int t, int j) -> bool {
        const int s = j % kStagesV, u = j / kStagesV;
        if (!wait_phase(&p_full[t], j & 1, abort_v, status, kTimeoutAccum)) return false;
        if (!wait_phase(&v_full[s], u & 1, abort_v, status, kTimeoutTmaFull)) return false;
        fence_after();
        const uint32_t p_addr = smem_u32(smem + L::kPOff + t * L::kPBytes);
        const uint32_t v_addr = smem_u32(smem + L::kVOff + s * L::kTileBytes);
#pragma unroll
        for (int kk = 0; kk < kBKV / 16; ++kk)
          mma(tmem + t * 128, desc_kmajor(p_addr + kk * 32), desc_mnmajor(v_addr + kk * 16 * 128, L::kKVHalf),
              id_pv, (j | kk) != 0);
        commit(&o_done[t]);
        return true;
      };
      for (int j = 0; ok && j < 2; ++j)
        for (int t = 0; ok && t < kQTiles; ++t)
          if (j < nt[t]) ok = issue_s(t, j);
      for (int j = 0; ok && j < ntiles; ++j) {
        for (int t = 0; ok && t < kQTiles; ++t)
          if (j < nt[t]) ok = issue_pv(t, j);
        if (!ok) break;
        commit(&v_empty[j % kStagesV]);          // every MMA reading V tile j was issued
        for (int t = 0; ok && t < kQTiles; ++t)
          if (j + 2 < nt[t]) ok = issue_s(t, j + 2);
      }
      // every MMA this thread issued has completed before the CTA tears down
      commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax: warpgroup t = tile t, query row r = 32 * (warp % 4) + lane ----------------
    const int t = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int qrow = (qp * kQTiles + t) * kBQ + r;
    const bool row_ok = qrow < q_len;
    const int qpos = shift + qrow;
    const int kend_me = kend_t[t], n_me = nt[t];
    // the warp's smallest query position (its lane 0) bounds which key tiles need the causal mask
    const int qpos_warp0 = shift + (qp * kQTiles + t) * kBQ + (warp & 3) * 32;
    const bool warp_rows_ok = (qrow - lane + 31) < q_len;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tmem_o = tmem + t * 128 + lane_base;
    const uint32_t tmem_s = tmem + 256 + t * 128 + lane_base;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // every wait is made warp-uniform (tcgen05.ld / st are warp-collective)
#define LSB_WAIT_ALL(bar, par, code)                                                     \
  if (!__all_sync(0xffffffffu, wait_phase(bar, par, abort_v, status, code))) { \
    ok = false;                                                                          \
    break;                                                                               \
  }
    for (int j = 0; j < n_me; ++j) {
      const int s = j % kStagesV, u = j / kStagesV, b = j & 1, ub = j >> 1;
      LSB_WAIT_ALL(&s_full[t * 2 + b], ub & 1, kTimeoutAccum);
      fence_after();
      uint32_t raw[kBKV];
#pragma unroll
      for (int c = 0; c < kBKV; c += 16) tmem_ld16(tmem_s + b * kBKV + c, raw + c);
      tmem_wait_ld();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[t * 2 + b]);
      const int k0 = j * kBKV;
      // the stage's bad-block mask is published by the producer's arrival on v_full (V has long
      // landed by now: it was issued right after K, which S needed)
      LSB_WAIT_ALL(&v_full[s], u & 1, kTimeoutTmaFull);
      const uint64_t bad = bad_keys[s];
      // interior tile for the whole warp: every key valid for every row -> no mask
      const bool interior = bad == 0ull && k0 + kBKV <= kend_me && k0 + kBKV - 1 <= qpos_warp0 && warp_rows_ok;
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
      if (interior) {
#pragma unroll
        for (int c = 0; c < kBKV; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(raw[c]));
      } else {
#pragma unroll
        for (int c = 0; c < kBKV; ++c) {
          const int kp = k0 + c;
          const bool valid = row_ok && kp <= qpos && kp < kend_me && !((bad >> c) & 1ull);
          if (!valid) raw[c] = __float_as_uint(-INFINITY);
          mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(raw[c]));
        }
      }
      const float mx_raw = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                 fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float mx = mx_raw * scale_log2;      // scale > 0: max commutes with the scaling
      float alpha = 1.f;
      if (mx > m_used + kRescaleLog2) {
        alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
        m_used = mx;
        l *= alpha;
      }
      const float neg_m = m_used == -INFINITY ? 0.f : -m_used;   // a fully masked row: all P = 0
      // P = exp2(s - m) packed to bf16 in registers first: the exponentials overlap this tile's
      // previous PV, which must finish before the P buffer is overwritten
      uint32_t pw[kBKV / 2];
      float sum8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) sum8[e] = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < kBKV / 8; ++c8) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          p[e] = ex2(fmaf(__uint_as_float(raw[c8 * 8 + e]), scale_log2, neg_m));   // ex2(-inf) = 0
          sum8[e] += p[e];
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) pw[c8 * 4 + e] = pack_bf16(p[2 * e], p[2 * e + 1]);
      }
      l += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      if (j >= 1) {
        LSB_WAIT_ALL(&o_done[t], (j - 1) & 1, kTimeoutAccum);
      }
      uint8_t* prow = smem + L::kPOff + t * L::kPBytes + r * 128;
#pragma unroll
      for (int c8 = 0; c8 < kBKV / 8; ++c8)
        *reinterpret_cast<uint4*>(prow + ((c8 ^ (r & 7)) << 4)) =
            make_uint4(pw[c8 * 4], pw[c8 * 4 + 1], pw[c8 * 4 + 2], pw[c8 * 4 + 3]);
      // zero the V rows of keys no query may see (past the context, or from a bad block)
      if (k0 + kBKV > kend || bad != 0ull) {
        uint8_t* vt = smem + L::kVOff + s * L::kTileBytes;
        for (int idx = r; idx < kBKV * L::kHalves * 8; idx += kBQ) {
          const int key = idx / (L::kHalves * 8), rem = idx % (L::kHalves * 8);
          const int hf = rem / 8, ch = rem % 8;
          if (k0 + key >= kend || ((bad >> key) & 1ull))
            *reinterpret_cast<uint4*>(vt + hf * L::kKVHalf + key * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_async_smem();
      // rescale O in TMEM when some row of this warp moved its max (the previous PV is done)
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
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
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
#undef LSB_WAIT_ALL
    // epilogue: O / l -> bf16
    if (ok && n_me > 0 &&
        __all_sync(0xffffffffu, wait_phase(&o_done[t], (n_me - 1) & 1, abort_v, status, kTimeoutAccum))) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = out + ((size_t)(q0 + (row_ok ? qrow : 0)) * nh + h) * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 16) {
        uint32_t o[16];
        tmem_ld16(tmem_o + c, o);
        tmem_wait_ld();
        if (row_ok) {
          uint4 w0, w1;
          w0.x = pack_bf16(__uint_as_float(o[0]) * inv, __uint_as_float(o[1]) * inv);
          w0.y = pack_bf16(__uint_as_float(o[2]) * inv, __uint_as_float(o[3]) * inv);
          w0.z = pack_bf16(__uint_as_float(o[4]) * inv, __uint_as_float(o[5]) * inv);
          w0.w = pack_bf16(__uint_as_float(o[6]) * inv, __uint_as_float(o[7]) * inv);
          w1.x = pack_bf16(__uint_as_float(o[8]) * inv, __uint_as_float(o[9]) * inv);
          w1.y = pack_bf16(__uint_as_float(o[10]) * inv, __uint_as_float(o[11]) * inv);
          w1.z = pack_bf16(__uint_as_float(o[12]) * inv, __uint_as_float(o[13]) * inv);
          w1.w = pack_bf16(__uint_as_float(o[14]) * inv, __uint_as_float(o[15]) * inv);
          *reinterpret_cast<uint4*>(orow + c) = w0;
          *reinterpret_cast<uint4*>(orow + c + 8) = w1;
        }
      }
    } else if (row_ok && n_me == 0) {
      bf16* orow = out + ((size_t)(q0 + qrow) * nh + h) * HD;
      for (int c = 0; c < HD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 9) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::kTmemCols));
  }
}

}  // namespace

// Whether the tensor-core prefill kernel takes this shape (head dim and a TMA-tileable block size).
bool prefill_tc_supported(int64_t block_size, int64_t head_dim) {
  return (head_dim == 64 || head_dim == 128) && block_size % 8 == 0 && (block_size % 64 == 0 || 64 % block_size == 0);
}

// out / q: bf16 [T, nh, hd]; pools [blocks, kv_heads, block_size, hd]; cu_q int32 [B + 1];
// seqlens_k int32 [B]; block_tables int32 [B, stride].
void prefill_attention_tc(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor cu_q,
                          at::Tensor seqlens_k, at::Tensor block_tables, double scale, int64_t max_q,
                          at::Tensor status) {
  LSB_CHECK(q.dim() == 3 && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q must be contiguous bf16 [T, nh, hd]");
  LSB_CHECK(out.sizes() == q.sizes() && out.is_contiguous() && out.scalar_type() == at::kBFloat16, "bad output");
  LSB_CHECK(kc.dim() == 4 && vc.sizes() == kc.sizes() && kc.is_contiguous() && vc.is_contiguous() &&
                kc.scalar_type() == at::kBFloat16 && vc.scalar_type() == at::kBFloat16,
            "KV pools must be contiguous bf16 [blocks, kv_heads, block_size, head_dim]");
  LSB_CHECK(cu_q.scalar_type() == at::kInt && seqlens_k.scalar_type() == at::kInt &&
                block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(),
            "cu_seqlens_q / seqlens_k / block_tables must be int32");
  const int T = q.size(0), nh = q.size(1), hd = q.size(2), nkv = kc.size(1), bs = kc.size(2);
  const int B = seqlens_k.numel();
  LSB_CHECK(kc.size(3) == hd && nh % nkv == 0, "head layout mismatch");
  LSB_CHECK(prefill_tc_supported(bs, hd), "block size / head dim unsupported by the tensor-core prefill kernel");
  LSB_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0, "q must be 16-byte aligned");
  LSB_CHECK((int64_t)kc.numel() / hd < (int64_t)INT32_MAX && (int64_t)T * nh * hd < (int64_t)INT32_MAX,
            "sizes exceed int32 tensor-map coordinates");
  if (T == 0 || B == 0 || max_q <= 0) return;
  const at::cuda::CUDAGuard guard(q.device());
  CUtensorMap tm_q;
  {
    cuuint64_t dims[2] = {(cuuint64_t)nh * hd, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)nh * hd * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)kBQ};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = tensor_map_encoder()(&tm_q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q.data_ptr(), dims, strides, box,
                                      estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    LSB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed for q (" + std::to_string((int)r) + ")");
  }
  const int box_keys = bs >= 64 ? 64 : bs;
  const CUtensorMap& tm_k = kv_pool_map(kc, box_keys);
  const CUtensorMap& tm_v = kv_pool_map(vc, box_keys);
  const int pairs = (int)((max_q + kQTiles * kBQ - 1) / (kQTiles * kBQ));
  LSB_CHECK((int64_t)pairs * B < 65536, "too many query tiles for one launch");
  const float sl = (float)scale * kLog2e;
  auto stream = at::cuda::getCurrentCUDAStream();
  int* st = status_ptr(status);
#define LSB_PF_TC(HD)                                                                                              \
  do {                                                                                                             \
    const int smem = PfLayout<HD>::kBytes;                                                                         \
    ensure_dynamic_smem((const void*)prefill_tc_kernel<HD>, smem);                                               \
    launch_pdl(prefill_tc_kernel<HD>, dim3(nh, pairs * B), dim3(kThreads), smem, stream, tm_q, tm_k, tm_v,        \
               (bf16*)out.data_ptr(), cu_q.data_ptr<int>(), seqlens_k.data_ptr<int>(), block_tables.data_ptr<int>(), \
               (int)block_tables.size(1), sl, nh, nkv, bs, box_keys, pairs, B, (int)kc.size(0), st);               \
  } while (0)
  if (hd == 128) LSB_PF_TC(128);
  else LSB_PF_TC(64);
#undef LSB_PF_TC
  auto e = cudaGetLastError();
  LSB_CHECK(e == cudaSuccess, std::string("prefill_tc launch failed: ") + cudaGetErrorString(e));
}

}  // namespace lsb
