// Paged attention kernels over the pool layout [num_blocks, kv_heads, block_size, head_dim].
//
// decode:  split-KV ("flash-decoding") with the G query heads that share a KV head packed as
//          the rows of one 16-row tensor-core tile, so every K/V byte is read once per KV head.
//          Split partials (unnormalised O, running max, sum) go to a caller-provided workspace
//          and the CTA finishing a (sequence, KV head)'s last split merges them; a context of
//          one split is written directly.  (Kernel in attention_tiles.cuh.)
// prefill: varlen causal FlashAttention-2 style tiles (64 query rows x 64 keys per step) over
//          paged keys, covering plain / chunked / prefix-cached prefill and packed verify.
// tree:    EAGLE3 tree verify -- paged prefix keys plus a side buffer of tree-node keys under
//          an ancestor bitmask per query row.
//
// The QK^T and PV products of decode and prefill use mma.sync m16n8k16 (bf16 -> fp32); decode is
// bound by HBM bandwidth, not by the tensor pipe.  K/V tiles are staged in shared memory with
// cp.async, XOR-swizzled by row so the ldmatrix reads are conflict-free.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "attention_tiles.cuh"
#include "common.cuh"

namespace lsb {
namespace {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }
#define LSB_CHECK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

// ------------------------------------------------------------------------------------------
// Prefill (varlen, causal, paged keys)
// ------------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(NTHREADS) prefill_kernel(
    bf16* __restrict__ out, const bf16* __restrict__ q, const bf16* __restrict__ kc, const bf16* __restrict__ vc,
    const int* __restrict__ cu_q, const int* __restrict__ seqlens_k, const int* __restrict__ block_tables,
    int bt_stride, float scale_log2, int nh, int nkv, int bs, int tiles_per_seq, int nblk, int* __restrict__ status) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) char smem[];
  bf16* sq = reinterpret_cast<bf16*>(smem);
  bf16* sk[2] = {reinterpret_cast<bf16*>(smem + KT * HD * 2), reinterpret_cast<bf16*>(smem + 3 * KT * HD * 2)};
  bf16* sv[2] = {reinterpret_cast<bf16*>(smem + 2 * KT * HD * 2), reinterpret_cast<bf16*>(smem + 4 * KT * HD * 2)};
  const int seq = blockIdx.x / tiles_per_seq, qt = blockIdx.x % tiles_per_seq;
  const int h = blockIdx.y, kvh = h / (nh / nkv);
  const int q0 = cu_q[seq], q_len = cu_q[seq + 1] - q0;
  if (qt * 64 >= q_len) return;
  const int k_len = seqlens_k[seq];
  const int shift = k_len - q_len;                 // absolute position of query row 0
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int* bt = block_tables + (size_t)seq * bt_stride;
  constexpr int CH = HD / 8;
  // stage the 64-row query tile
  for (int i = threadIdx.x; i < 64 * CH; i += NTHREADS) {
    const int r = i / CH, c = i % CH;
    const int row = qt * 64 + r;
    const bool ok = row < q_len;
    const bf16* src = q + ((size_t)(q0 + (ok ? row : 0)) * nh + h) * HD + c * 8;
    cp_async16(reinterpret_cast<char*>(sq) + swz<HD>(r, c), src, ok);
  }
  cp_async_commit();
  const int last_row = min(q_len, (qt + 1) * 64) - 1;
  const int kend = min(k_len, shift + last_row + 1);
  const int ntiles = (kend + KT - 1) / KT;
  if (ntiles > 0) {
    load_kv_tile<HD>(sk[0], sv[0], kc, vc, bt, 0, kend, kvh, nkv, bs, nblk, status);
    cp_async_commit();
    cp_async_wait<1>();
  } else {
    cp_async_wait<0>();
  }
  __syncthreads();
  uint32_t qa[HD / 16][4];
  {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk)
      ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], smem_u32(sq) + swz<HD>(r, kk * 2 + (lane >> 4)));
  }
  float o[HD / 8][4];
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int row_a = qt * 64 + warp * 16 + (lane >> 2);   // rows of c0/c1 and c2/c3 (+8)
  const int qpos[2] = {shift + row_a, shift + row_a + 8};
  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) {
      load_kv_tile<HD>(sk[(t + 1) & 1], sv[(t + 1) & 1], kc, vc, bt, (t + 1) * KT, kend, kvh, nkv, bs, nblk, status);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < KT / 16; ++ks) {
      float s0[4], s1[4];
      qk16<HD>(s0, s1, qa, smem_u32(sk[t & 1]), ks * 16);
      const int kb = t * KT + ks * 16 + (lane & 3) * 2;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kp = kb + (i & 1);
        const int qp = qpos[i >> 1];
        s0[i] = (kp <= qp && kp < kend) ? s0[i] * scale_log2 : -INFINITY;
        s1[i] = (kp + 8 <= qp && kp + 8 < kend) ? s1[i] * scale_log2 : -INFINITY;
      }
      softmax_pv<HD>(s0, s1, m, l, o, smem_u32(sv[t & 1]), ks * 16);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  const int c2 = (lane & 3) * 2;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = row_a + half * 8;
    if (row >= q_len) continue;
    const float inv = l[half] > 0.f ? 1.f / l[half] : 0.f;
    bf16* dst = out + ((size_t)(q0 + row) * nh + h) * HD;
#pragma unroll
    for (int n = 0; n < HD / 8; ++n)
      *reinterpret_cast<uint32_t*>(dst + n * 8 + c2) = pack_bf16(o[n][half * 2] * inv, o[n][half * 2 + 1] * inv);
  }
}

// ------------------------------------------------------------------------------------------
// Tree verify (one CTA per (query node, head)); CUDA-core dot products, online softmax per warp.
// ------------------------------------------------------------------------------------------
template <int HD>
__global__ void tree_kernel(bf16* __restrict__ out, const bf16* __restrict__ q, const bf16* __restrict__ kc,
                            const bf16* __restrict__ vc, const int* __restrict__ bt, int prefix_len,
                            const bf16* __restrict__ tk, const bf16* __restrict__ tv, int n_tree,
                            const int* __restrict__ mask_bits, float scale_log2, int nh, int nkv, int bs, int nblk,
                            int* __restrict__ status) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = HD / 32;
  __shared__ float sm[4], sl[4], so[4][HD];
  const int qi = blockIdx.x, h = blockIdx.y, kvh = h / (nh / nkv);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float qv[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) qv[j] = to_f(q[((size_t)qi * nh + h) * HD + lane * PER + j]);
  const int bits = mask_bits[qi];
  float m = -INFINITY, l = 0.f, acc[PER] = {};
  const int total = prefix_len + n_tree;
  for (int key = warp; key < total; key += 4) {
    const bf16 *kp, *vp;
    if (key < prefix_len) {
      const int blk = bt[key / bs];
      if ((unsigned)blk >= (unsigned)nblk) {   // never dereferenced: the key is skipped
        if (lane == 0) record_error(status, kBadIndex);
        continue;
      }
      const size_t off = (((size_t)blk * nkv + kvh) * bs + key % bs) * HD;
      kp = kc + off;
      vp = vc + off;
    } else {
      const int node = key - prefix_len;
      if (!((bits >> node) & 1)) continue;
      kp = tk + ((size_t)node * nkv + kvh) * HD;
      vp = tv + ((size_t)node * nkv + kvh) * HD;
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) s += qv[j] * to_f(kp[lane * PER + j]);
    s = warp_sum(s) * scale_log2;
    const float mn = fmaxf(m, s);
    const float corr = exp2f(m - mn), p = exp2f(s - mn);
    l = l * corr + p;
#pragma unroll
    for (int j = 0; j < PER; ++j) acc[j] = acc[j] * corr + p * to_f(vp[lane * PER + j]);
    m = mn;
  }
  if (lane == 0) {
    sm[warp] = m;
    sl[warp] = l;
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) so[warp][lane * PER + j] = acc[j];
  __syncthreads();
  if (warp == 0) {
    float M = fmaxf(fmaxf(sm[0], sm[1]), fmaxf(sm[2], sm[3]));
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    for (int w = 0; w < 4; ++w) L += sl[w] * exp2f(sm[w] - Mu);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      float O = 0.f;
      for (int w = 0; w < 4; ++w) O += so[w][lane * PER + j] * exp2f(sm[w] - Mu);
      out[((size_t)qi * nh + h) * HD + lane * PER + j] = to_b(L > 0.f ? O / L : 0.f);
    }
  }
}

void check_pool(const at::Tensor& kc, const at::Tensor& vc) {
  LSB_CHECK(kc.is_cuda() && kc.scalar_type() == at::kBFloat16 && kc.is_contiguous() && kc.dim() == 4,
            "k_cache must be contiguous bf16 [blocks, kv_heads, block_size, head_dim]");
  LSB_CHECK(vc.sizes() == kc.sizes() && vc.scalar_type() == at::kBFloat16 && vc.is_contiguous(),
            "v_cache must match k_cache");
}

}  // namespace

int* status_ptr(const at::Tensor& status);

void decode_attention(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor block_tables,
                      at::Tensor context_lens, double scale, at::Tensor part_o, at::Tensor part_ml, at::Tensor counters,
                      int64_t max_splits, int64_t partition, int64_t grid_z, at::Tensor status) {
  check_pool(kc, vc);
  LSB_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "q must be bf16 [B, nh, hd]");
  LSB_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "block_tables must be int32");
  LSB_CHECK(context_lens.scalar_type() == at::kInt, "context_lens must be int32");
  LSB_CHECK(counters.scalar_type() == at::kInt, "counters must be int32");
  const int B = q.size(0), nh = q.size(1), hd = q.size(2), nkv = kc.size(1), bs = kc.size(2);
  LSB_CHECK(kc.size(3) == hd && nh % nkv == 0 && nh / nkv <= 16, "head layout unsupported (group size <= 16)");
  LSB_CHECK(partition % KT == 0, "partition must be a multiple of 64");
  LSB_CHECK(block_tables.size(1) * (int64_t)bs <= max_splits * partition, "workspace has too few splits");
  LSB_CHECK(part_o.numel() >= (int64_t)B * nh * max_splits * hd && part_ml.numel() >= (int64_t)B * nh * max_splits * 2,
            "decode workspace too small");
  LSB_CHECK(counters.numel() >= (int64_t)B * nkv, "decode counters too small");
  if (B == 0) return;
  const at::cuda::CUDAGuard g(q.device());
  // CTAs per (sequence, kv head): one when the batch alone gives >= 2 waves, else enough to fill the SMs
  const int z = grid_z > 0 ? (int)std::min<int64_t>(grid_z, max_splits)
                           : (int)std::max<int64_t>(1, std::min<int64_t>(max_splits, (148 * 3 + B * nkv - 1) / (B * nkv)));
  dim3 grid(B, nkv, z);
  const float sl = (float)scale * kLog2e;
#define LSB_DEC(HD)                                                                                                \
  do {                                                                                                             \
    const int smem = decode_smem(HD);                                                                              \
    cudaFuncSetAttribute(decode_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                    \
    launch_pdl(decode_kernel<HD>, grid, NTHREADS, smem, stream(), (bf16*)out.data_ptr(), (const bf16*)q.data_ptr(), \
               (const bf16*)kc.data_ptr(), (const bf16*)vc.data_ptr(), block_tables.data_ptr<int>(),               \
               (int)block_tables.size(1), context_lens.data_ptr<int>(), sl, part_o.data_ptr<float>(),             \
               part_ml.data_ptr<float>(), counters.data_ptr<int>(), (int)max_splits, (int)partition, nh, nkv, bs,   \
               (int)kc.size(0), status_ptr(status));                                                               \
  } while (0)
  if (hd == 128) LSB_DEC(128);
  else if (hd == 64) LSB_DEC(64);
  else LSB_CHECK(false, "head_dim must be 64 or 128");
#undef LSB_DEC
}

void prefill_attention(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor cu_q,
                       at::Tensor seqlens_k, at::Tensor block_tables, double scale, int64_t max_seqlen_q,
                       at::Tensor status) {
  check_pool(kc, vc);
  LSB_CHECK(q.scalar_type() == at::kBFloat16 && q.is_contiguous() && q.dim() == 3, "q must be bf16 [T, nh, hd]");
  LSB_CHECK(cu_q.scalar_type() == at::kInt && seqlens_k.scalar_type() == at::kInt, "cu_seqlens / seqlens_k int32");
  LSB_CHECK(block_tables.scalar_type() == at::kInt && block_tables.is_contiguous(), "block_tables must be int32");
  const int nseq = seqlens_k.numel(), nh = q.size(1), hd = q.size(2), nkv = kc.size(1), bs = kc.size(2);
  if (nseq == 0 || q.size(0) == 0) return;
  const int tiles = (int)((max_seqlen_q + 63) / 64);
  const at::cuda::CUDAGuard g(q.device());
  dim3 grid(nseq * tiles, nh);
  const float sl = (float)scale * kLog2e;
#define LSB_PRE(HD)                                                                                               \
  do {                                                                                                            \
    const int smem = 5 * KT * HD * 2;                                                                             \
    cudaFuncSetAttribute(prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                  \
    launch_pdl(prefill_kernel<HD>, grid, NTHREADS, smem, stream(),                                                        \
        (bf16*)out.data_ptr(), (const bf16*)q.data_ptr(), (const bf16*)kc.data_ptr(), (const bf16*)vc.data_ptr(),  \
        cu_q.data_ptr<int>(), seqlens_k.data_ptr<int>(), block_tables.data_ptr<int>(), block_tables.size(1), sl,   \
        nh, nkv, bs, tiles, (int)kc.size(0), status_ptr(status));                                                  \
  } while (0)
  if (hd == 128) LSB_PRE(128);
  else if (hd == 64) LSB_PRE(64);
  else LSB_CHECK(false, "head_dim must be 64 or 128");
#undef LSB_PRE
}

void tree_attention(at::Tensor out, at::Tensor q, at::Tensor kc, at::Tensor vc, at::Tensor bt, int64_t prefix_len,
                    at::Tensor tk, at::Tensor tv, at::Tensor mask_bits, double scale, at::Tensor status) {
  check_pool(kc, vc);
  const int n = q.size(0), nh = q.size(1), hd = q.size(2), nkv = kc.size(1), bs = kc.size(2);
  LSB_CHECK(tk.size(0) <= 32, "at most 32 tree nodes");
  LSB_CHECK(mask_bits.scalar_type() == at::kInt && mask_bits.numel() == n, "mask_bits must be int32 [n]");
  if (n == 0) return;
  const at::cuda::CUDAGuard g(q.device());
  const float sl = (float)scale * kLog2e;
  if (hd == 128)
    launch_pdl(tree_kernel<128>, dim3(n, nh), 128, 0, stream(), 
        (bf16*)out.data_ptr(), (const bf16*)q.data_ptr(), (const bf16*)kc.data_ptr(), (const bf16*)vc.data_ptr(),
        bt.data_ptr<int>(), prefix_len, (const bf16*)tk.data_ptr(), (const bf16*)tv.data_ptr(), tk.size(0),
        mask_bits.data_ptr<int>(), sl, nh, nkv, bs, (int)kc.size(0), status_ptr(status));
  else if (hd == 64)
    launch_pdl(tree_kernel<64>, dim3(n, nh), 128, 0, stream(), 
        (bf16*)out.data_ptr(), (const bf16*)q.data_ptr(), (const bf16*)kc.data_ptr(), (const bf16*)vc.data_ptr(),
        bt.data_ptr<int>(), prefix_len, (const bf16*)tk.data_ptr(), (const bf16*)tv.data_ptr(), tk.size(0),
        mask_bits.data_ptr<int>(), sl, nh, nkv, bs, (int)kc.size(0), status_ptr(status));
  else
    LSB_CHECK(false, "head_dim must be 64 or 128");
}

}  // namespace lsb
