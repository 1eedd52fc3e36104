// Memory-bound kernels of the serving path: RMSNorm (+ residual add), SiLU-mul, embedding
// gather, fused QK-norm + RoPE + paged K/V store, K/V scatter, tree-KV commit, split-K
// reductions with their epilogues, and row argmax / sampling.
//
// All of them are single-pass over their bytes with 16-byte vector accesses where the row
// length allows; statistics are accumulated in fp32.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cooperative_groups.h>
#include <cstdlib>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

#include "common.cuh"

namespace lsb {

namespace {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

#define LSB_CHECK(cond, msg) TORCH_CHECK(cond, "llmserve_b200: ", msg)

inline void check_bf16(const at::Tensor& t, const char* name) {
  LSB_CHECK(t.is_cuda(), std::string(name) + " must be a CUDA tensor");
  LSB_CHECK(t.scalar_type() == at::kBFloat16, std::string(name) + " must be bfloat16");
  LSB_CHECK(t.is_contiguous(), std::string(name) + " must be contiguous");
}

struct alignas(16) Vec8 {
  bf16 v[8];
};

// ------------------------------------------------------------------------------------------
// RMSNorm: out = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w)
// ------------------------------------------------------------------------------------------
template <bool kAddResidual>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(bf16* __restrict__ out, bf16* __restrict__ res_out, const bf16* __restrict__ x,
                               const bf16* __restrict__ residual, const bf16* __restrict__ w, int H, float eps) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float srow[];            // H floats: the (summed) row in fp32
  __shared__ float scratch[32];
  const int row = blockIdx.x;
  const bf16* xr = x + (size_t)row * H;
  const bf16* rr = kAddResidual ? residual + (size_t)row * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    Vec8 a = *reinterpret_cast<const Vec8*>(xr + i);
    Vec8 r;
    if (kAddResidual) r = *reinterpret_cast<const Vec8*>(rr + i);
    Vec8 ro;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = to_f(a.v[j]);
      if (kAddResidual) {
        v += to_f(r.v[j]);
        ro.v[j] = to_b(v);
      }
      srow[i + j] = v;
      ss += v * v;
    }
    if (kAddResidual) *reinterpret_cast<Vec8*>(res_out + (size_t)row * H + i) = ro;
  }
  const float inv = rsqrtf(block_sum(ss, scratch) / H + eps);
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    Vec8 wv = *reinterpret_cast<const Vec8*>(w + i);
    Vec8 o;
#pragma unroll
    for (int j = 0; j < 8; ++j) o.v[j] = to_b(to_f(to_b(srow[i + j] * inv)) * to_f(wv.v[j]));
    *reinterpret_cast<Vec8*>(out + (size_t)row * H + i) = o;
  }
}

int norm_threads(int H) {
  int t = H / 8;
  t = ((t + 31) / 32) * 32;
  return std::max(32, std::min(1024, t));
}

// ------------------------------------------------------------------------------------------
// SiLU-mul: out[t, i] = bf16(silu(x[t, i]) * x[t, I + i])
// ------------------------------------------------------------------------------------------
// INTERLEAVED: the input row holds gate/up in alternating 64-column chunks (g0..g63, u0..u63, ...)
// instead of [gate (I) | up (I)].
template <bool INTERLEAVED>
__global__ void silu_mul_kernel(bf16* __restrict__ out, const bf16* __restrict__ x, int I, int64_t total_vec) {
  pdl_trigger();
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int vec_per_row = I / 8;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total_vec; v += stride) {
    const int64_t row = v / vec_per_row;
    const int col = (int)(v % vec_per_row) * 8;
    const int64_t gcol = INTERLEAVED ? (col / 64) * 128 + col % 64 : col;
    const int64_t ucol = INTERLEAVED ? gcol + 64 : I + col;
    Vec8 g = *reinterpret_cast<const Vec8*>(x + row * 2 * I + gcol);
    Vec8 u = *reinterpret_cast<const Vec8*>(x + row * 2 * I + ucol);
    Vec8 o;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gv = to_f(g.v[j]);
      o.v[j] = to_b(gv / (1.f + expf(-gv)) * to_f(u.v[j]));
    }
    *reinterpret_cast<Vec8*>(out + row * I + col) = o;
  }
}

// ------------------------------------------------------------------------------------------
// Embedding gather (replicated table)
// ------------------------------------------------------------------------------------------
__global__ void embedding_kernel(bf16* __restrict__ out, const int64_t* __restrict__ ids, const bf16* __restrict__ table,
                                 int H, int64_t V, int* status) {
  pdl_trigger();
  pdl_wait();
  const int64_t id = ids[blockIdx.x];
  bf16* o = out + (size_t)blockIdx.x * H;
  if (id < 0 || id >= V) {
    record_error(status, kBadIndex);
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) *reinterpret_cast<Vec8*>(o + i) = Vec8{};
    return;
  }
  const bf16* src = table + id * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8)
    *reinterpret_cast<Vec8*>(o + i) = *reinterpret_cast<const Vec8*>(src + i);
}

// ------------------------------------------------------------------------------------------
// Fused per-head RMSNorm (q/k) + neox RoPE + paged store of k and v.
// One warp per (token, head); heads [0, nh) are queries, [nh, nh+nkv) keys, then values.
// Lane l owns dims [l*P, l*P+P) of the first half and the same offsets in the second half
// (P = hd/64), which are exactly the pairs the rotation mixes.
// ------------------------------------------------------------------------------------------
template <int P, bool kStore, int S>
__global__ void qkv_rope_kernel(bf16* __restrict__ q_out, bf16* __restrict__ k_out, const bf16* __restrict__ qkv,
                                const float* __restrict__ part,
                                const int64_t* __restrict__ positions, const float* __restrict__ cos_sin,
                                const bf16* __restrict__ q_w, const bf16* __restrict__ k_w, float eps,
                                bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                const int* __restrict__ slot_mapping, int T, int nh, int nkv, int block_size,
                                int64_t num_slots, int* status) {
  pdl_trigger();
  pdl_wait();
  constexpr int HD = 64 * P;
  constexpr int HALF = HD / 2;
  const int warps_per_block = blockDim.x >> 5;
  const int head = blockIdx.y * warps_per_block + (threadIdx.x >> 5);
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int nheads = nh + 2 * nkv;
  if (head >= nheads) return;
  const size_t row_off = (size_t)t * nheads * HD + (size_t)head * HD;
  const int d0 = lane * P;
  float a[P], b[P];
  if constexpr (S == 0) {
    const bf16* src = qkv + row_off;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      a[j] = to_f(src[d0 + j]);
      b[j] = to_f(src[HALF + d0 + j]);
    }
  } else {
    // fused split-K reduction of the QKV projection (rounded to bf16 like a bf16 GEMM output)
    const size_t plane = (size_t)T * nheads * HD;
    float pa[S][P], pb[S][P];
#pragma unroll
    for (int s = 0; s < S; ++s)
#pragma unroll
      for (int j = 0; j < P; ++j) {
        pa[s][j] = __ldcg(part + s * plane + row_off + d0 + j);
        pb[s][j] = __ldcg(part + s * plane + row_off + HALF + d0 + j);
      }
#pragma unroll
    for (int j = 0; j < P; ++j) {
      float x = 0.f, y = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) {
        x += pa[s][j];
        y += pb[s][j];
      }
      a[j] = to_f(to_b(x));
      b[j] = to_f(to_b(y));
    }
  }
  const bool is_q = head < nh, is_k = !is_q && head < nh + nkv;
  if (is_q || is_k) {
    const bf16* w = is_q ? q_w : k_w;
    if (w != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < P; ++j) ss += a[j] * a[j] + b[j] * b[j];
      const float inv = rsqrtf(warp_sum(ss) / HD + eps);
#pragma unroll
      for (int j = 0; j < P; ++j) {
        a[j] = to_f(to_b(to_f(to_b(a[j] * inv)) * to_f(w[d0 + j])));
        b[j] = to_f(to_b(to_f(to_b(b[j] * inv)) * to_f(w[HALF + d0 + j])));
      }
    }
    const float* cs = cos_sin + positions[t] * HD;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const float c = cs[d0 + j], s = cs[HALF + d0 + j];
      const float x1 = a[j], x2 = b[j];
      a[j] = x1 * c - x2 * s;
      b[j] = x2 * c + x1 * s;
    }
  }
  if (is_q) {
    bf16* dst = q_out + (size_t)t * nh * HD + (size_t)head * HD;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      dst[d0 + j] = to_b(a[j]);
      dst[HALF + d0 + j] = to_b(b[j]);
    }
    return;
  }
  const int kvh = is_k ? head - nh : head - nh - nkv;
  if constexpr (kStore) {
    const int slot = slot_mapping[t];
    if (slot < 0) return;
    if (slot >= num_slots) {
      record_error(status, kBadIndex);
      return;
    }
    const int blk = slot / block_size, off = slot % block_size;
    bf16* dst = (is_k ? k_cache : v_cache) + (((size_t)blk * nkv + kvh) * block_size + off) * HD;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      dst[d0 + j] = to_b(a[j]);
      dst[HALF + d0 + j] = to_b(b[j]);
    }
  } else {
    if (!is_k) return;
    bf16* dst = k_out + (size_t)t * nkv * HD + (size_t)kvh * HD;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      dst[d0 + j] = to_b(a[j]);
      dst[HALF + d0 + j] = to_b(b[j]);
    }
  }
}

// ------------------------------------------------------------------------------------------
// K/V scatter and tree commit
// ------------------------------------------------------------------------------------------
__global__ void store_kv_kernel(const bf16* __restrict__ k, const bf16* __restrict__ v, bf16* __restrict__ k_cache,
                                bf16* __restrict__ v_cache, const int* __restrict__ slots, int nkv, int hd,
                                int block_size, int64_t num_slots, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y;
  const int slot = slots[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0) record_error(status, kBadIndex);
    return;
  }
  const int blk = slot / block_size, off = slot % block_size;
  const size_t src = ((size_t)t * nkv + h) * hd;
  const size_t dst = (((size_t)blk * nkv + h) * block_size + off) * hd;
  for (int i = threadIdx.x * 8; i < hd; i += blockDim.x * 8) {
    *reinterpret_cast<Vec8*>(k_cache + dst + i) = *reinterpret_cast<const Vec8*>(k + src + i);
    *reinterpret_cast<Vec8*>(v_cache + dst + i) = *reinterpret_cast<const Vec8*>(v + src + i);
  }
}

// grid (layers, committed nodes, kv heads)
__global__ void commit_tree_kv_kernel(const bf16* __restrict__ tk, const bf16* __restrict__ tv, bf16* __restrict__ kc,
                                      bf16* __restrict__ vc, const int* __restrict__ nodes, const int* __restrict__ slots,
                                      int n_nodes, int nkv, int hd, int block_size, int64_t blocks_per_layer,
                                      int* status) {
  pdl_trigger();
  pdl_wait();
  const int layer = blockIdx.x, j = blockIdx.y, h = blockIdx.z;
  const int node = nodes[j], slot = slots[j];
  if (node < 0 || node >= n_nodes || slot < 0 || slot >= blocks_per_layer * block_size) {
    if (threadIdx.x == 0) record_error(status, kBadIndex);
    return;
  }
  const int blk = slot / block_size, off = slot % block_size;
  const size_t src = (((size_t)layer * n_nodes + node) * nkv + h) * hd;
  const size_t dst = ((((size_t)layer * blocks_per_layer + blk) * nkv + h) * block_size + off) * hd;
  for (int i = threadIdx.x * 8; i < hd; i += blockDim.x * 8) {
    *reinterpret_cast<Vec8*>(kc + dst + i) = *reinterpret_cast<const Vec8*>(tk + src + i);
    *reinterpret_cast<Vec8*>(vc + dst + i) = *reinterpret_cast<const Vec8*>(tv + src + i);
  }
}

// ------------------------------------------------------------------------------------------
// split-K reductions (partials fp32 [S, T, N])
// ------------------------------------------------------------------------------------------
__global__ void splitk_reduce_kernel(bf16* __restrict__ out, const float* __restrict__ part, int S, int64_t TN) {
  pdl_trigger();
  pdl_wait();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 4;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < TN; i += stride) {
    float4 acc = *reinterpret_cast<const float4*>(part + i);
    for (int s = 1; s < S; ++s) {
      const float4 p = *reinterpret_cast<const float4*>(part + (int64_t)s * TN + i);
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    *reinterpret_cast<__nv_bfloat162*>(out + i) = lo;
    *reinterpret_cast<__nv_bfloat162*>(out + i + 2) = hi;
  }
}

// One block per row: y = bf16(sum_s part); s = y + residual; res_out = bf16(s);
// out = rmsnorm(s) * w.  Rounding y to bf16 first keeps the value stream of a bf16 GEMM
// followed by a separate add+RMSNorm.  All split loads of a thread are issued before any use
// (compile-time split count), so the row costs one memory latency, not one per split.
template <int S>
__global__ void __launch_bounds__(512) splitk_add_rmsnorm_kernel(bf16* __restrict__ out, bf16* __restrict__ res_out,
                                                                 const float* __restrict__ part,
                                                                 const bf16* __restrict__ residual,
                                                                 const bf16* __restrict__ w, int S_rt, int T, int N,
                                                                 float eps) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float srow[];
  __shared__ float scratch[32];
  const int row = blockIdx.x;
  const int64_t TN = (int64_t)T * N;
  const int nsplit = S > 0 ? S : S_rt;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < N; i += blockDim.x * 4) {
    const int64_t off = (int64_t)row * N + i;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (S > 0) {
      float4 p[S];
#pragma unroll
      for (int s = 0; s < S; ++s) p[s] = __ldcg(reinterpret_cast<const float4*>(part + s * TN + off));
#pragma unroll
      for (int s = 0; s < S; ++s) {
        acc.x += p[s].x; acc.y += p[s].y; acc.z += p[s].z; acc.w += p[s].w;
      }
    } else {
      for (int s = 0; s < nsplit; ++s) {
        const float4 p = __ldcg(reinterpret_cast<const float4*>(part + s * TN + off));
        acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
      }
    }
    const uint2 rraw = *reinterpret_cast<const uint2*>(residual + off);
    const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rraw.x);
    const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rraw.y);
    float v[4] = {to_f(to_b(acc.x)) + __low2float(r01), to_f(to_b(acc.y)) + __high2float(r01),
                  to_f(to_b(acc.z)) + __low2float(r23), to_f(to_b(acc.w)) + __high2float(r23)};
    __nv_bfloat162 o01 = __floats2bfloat162_rn(v[0], v[1]), o23 = __floats2bfloat162_rn(v[2], v[3]);
    uint2 oraw;
    oraw.x = *reinterpret_cast<uint32_t*>(&o01);
    oraw.y = *reinterpret_cast<uint32_t*>(&o23);
    *reinterpret_cast<uint2*>(res_out + off) = oraw;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      srow[i + j] = v[j];
      ss += v[j] * v[j];
    }
  }
  const float inv = rsqrtf(block_sum(ss, scratch) / N + eps);
  for (int i = threadIdx.x * 4; i < N; i += blockDim.x * 4) {
    const uint2 wraw = *reinterpret_cast<const uint2*>(w + i);
    const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wraw.x);
    const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wraw.y);
    const float wv[4] = {__low2float(w01), __high2float(w01), __low2float(w23), __high2float(w23)};
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = to_f(to_b(to_f(to_b(srow[i + j] * inv)) * wv[j]));
    __nv_bfloat162 o01 = __floats2bfloat162_rn(o[0], o[1]), o23 = __floats2bfloat162_rn(o[2], o[3]);
    uint2 oraw;
    oraw.x = *reinterpret_cast<uint32_t*>(&o01);
    oraw.y = *reinterpret_cast<uint32_t*>(&o23);
    *reinterpret_cast<uint2*>(out + (int64_t)row * N + i) = oraw;
  }
}

// Same operation with a row spread over a cluster of CL CTAs (each owns N / CL columns): a decode
// step has few rows (T = 64 at C = 64), so one CTA per row leaves most SMs idle and serialises
// every row's partial reads in one SM.  Each CTA issues all S partial loads of its columns at
// once, and the CTAs of a row add their sums of squares through distributed shared memory.
template <int S, int CL, int kPer>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(256)
    splitk_add_rmsnorm_cluster_kernel(bf16* __restrict__ out, bf16* __restrict__ res_out,
                                      const float* __restrict__ part, const bf16* __restrict__ residual,
                                      const bf16* __restrict__ w, int T, int N, float eps) {
  namespace cg = cooperative_groups;
  // kPer float4 chunks per thread: N = CL * 256 * 4 * kPer
  pdl_trigger();
  pdl_wait();
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float red[8];
  __shared__ float cta_ss;
  const int row = blockIdx.y;
  const int cols = N / CL;
  const int c0 = (int)cluster.block_rank() * cols;
  const int64_t TN = (int64_t)T * N;
  float4 v[kPer];
  float ss = 0.f;
  float4 p[kPer][S];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int col = c0 + (threadIdx.x + k * 256) * 4;
    if (col < c0 + cols) {
      const int64_t off = (int64_t)row * N + col;
#pragma unroll
      for (int s2 = 0; s2 < S; ++s2) p[k][s2] = __ldcg(reinterpret_cast<const float4*>(part + s2 * TN + off));
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int col = c0 + (threadIdx.x + k * 256) * 4;
    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (col >= c0 + cols) continue;
    const int64_t off = (int64_t)row * N + col;
    float4 acc = p[k][0];
#pragma unroll
    for (int s2 = 1; s2 < S; ++s2) {
      acc.x += p[k][s2].x; acc.y += p[k][s2].y; acc.z += p[k][s2].z; acc.w += p[k][s2].w;
    }
    const uint2 rr = *reinterpret_cast<const uint2*>(residual + off);
    const __nv_bfloat162 r01 = *reinterpret_cast<const __nv_bfloat162*>(&rr.x);
    const __nv_bfloat162 r23 = *reinterpret_cast<const __nv_bfloat162*>(&rr.y);
    v[k].x = to_f(to_b(acc.x)) + __low2float(r01);
    v[k].y = to_f(to_b(acc.y)) + __high2float(r01);
    v[k].z = to_f(to_b(acc.z)) + __low2float(r23);
    v[k].w = to_f(to_b(acc.w)) + __high2float(r23);
    const __nv_bfloat162 o01 = __floats2bfloat162_rn(v[k].x, v[k].y), o23 = __floats2bfloat162_rn(v[k].z, v[k].w);
    uint2 oraw;
    oraw.x = *reinterpret_cast<const uint32_t*>(&o01);
    oraw.y = *reinterpret_cast<const uint32_t*>(&o23);
    *reinterpret_cast<uint2*>(res_out + off) = oraw;
    ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    cta_ss = t;
  }
  cluster.sync();
  float total = 0.f;
#pragma unroll
  for (int c = 0; c < CL; ++c) total += *cluster.map_shared_rank(&cta_ss, c);
  cluster.sync();                                  // keep cta_ss alive until every CTA has read it
  const float inv = rsqrtf(total / N + eps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int col = c0 + (threadIdx.x + k * 256) * 4;
    if (col >= c0 + cols) continue;
    const uint2 wraw = *reinterpret_cast<const uint2*>(w + col);
    const __nv_bfloat162 w01 = *reinterpret_cast<const __nv_bfloat162*>(&wraw.x);
    const __nv_bfloat162 w23 = *reinterpret_cast<const __nv_bfloat162*>(&wraw.y);
    const float o0 = to_f(to_b(to_f(to_b(v[k].x * inv)) * __low2float(w01)));
    const float o1 = to_f(to_b(to_f(to_b(v[k].y * inv)) * __high2float(w01)));
    const float o2 = to_f(to_b(to_f(to_b(v[k].z * inv)) * __low2float(w23)));
    const float o3 = to_f(to_b(to_f(to_b(v[k].w * inv)) * __high2float(w23)));
    const __nv_bfloat162 q01 = __floats2bfloat162_rn(o0, o1), q23 = __floats2bfloat162_rn(o2, o3);
    uint2 oraw;
    oraw.x = *reinterpret_cast<const uint32_t*>(&q01);
    oraw.y = *reinterpret_cast<const uint32_t*>(&q23);
    *reinterpret_cast<uint2*>(out + (int64_t)row * N + col) = oraw;
  }
}

// split-K reduction of a gate/up projection + SiLU-mul -> bf16 [T, N/2].  INTERLEAVED: rows
// interleaved per 64 (g0..g63, u0..u63, g64, ...); otherwise [gate (N/2) | up (N/2)].
template <bool INTERLEAVED>
__global__ void splitk_silu_kernel(bf16* __restrict__ out, const float* __restrict__ part, int S, int T, int N) {
  pdl_trigger();
  pdl_wait();
  const int half = N / 2;
  const int64_t total = (int64_t)T * half;
  const int64_t TN = (int64_t)T * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / half;
    const int j = (int)(i % half);
    const int64_t gidx = INTERLEAVED ? t * N + (j / 64) * 128 + (j % 64) : t * N + j;
    const int64_t uoff = INTERLEAVED ? 64 : half;
    float g = 0.f, u = 0.f;
    for (int s = 0; s < S; ++s) {
      g += __ldcg(part + s * TN + gidx);
      u += __ldcg(part + s * TN + gidx + uoff);
    }
    g = to_f(to_b(g));
    u = to_f(to_b(u));
    out[i] = to_b(g / (1.f + expf(-g)) * u);
  }
}

// Decode-step input ids for the overlapped (one step ahead) decode loop: row i takes the token
// the previous step sampled for its row feed[i] (still on the device), or the host-supplied id
// when feed[i] < 0.  Replaces the int32 -> int64 widening of the ids at the head of the step.
__global__ void feed_ids_kernel(int64_t* __restrict__ out, const int* __restrict__ ids,
                                const int* __restrict__ feed, const int64_t* __restrict__ prev, int n, int n_prev,
                                int* status) {
  pdl_trigger();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int f = feed[i];
    int64_t v = ids[i];
    if (f >= 0) {
      if (f < n_prev) v = prev[f];
      else if (status != nullptr) record_error(status, kBadIndex);
    }
    out[i] = v;
  }
}

// Greedy speculative acceptance for a batch, packed for one host copy: row b of `out` is
// [accepted count a, final token (target id at row a: the correction, or the bonus when a == g),
//  start token, the g draft tokens].  Draft j is accepted while it equals the target's argmax at
// verify row j, for every j before it.
__global__ void greedy_accept_kernel(int64_t* __restrict__ out, const int64_t* __restrict__ target,
                                     const int64_t* __restrict__ draft, const int64_t* __restrict__ start, int B,
                                     int g) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t* t = target + (int64_t)b * (g + 1);
  const int64_t* d = draft + (int64_t)b * g;
  int64_t* o = out + (int64_t)b * (g + 3);
  int a = 0;
  while (a < g && d[a] == t[a]) ++a;
  o[0] = a;
  o[1] = t[a];
  o[2] = start[b];
  for (int j = 0; j < g; ++j) o[3 + j] = d[j];
}

// ------------------------------------------------------------------------------------------
// Row argmax (lowest index on ties) and exponential-race sampling
// ------------------------------------------------------------------------------------------
struct ArgBest {
  float v;
  int64_t i;
};

__device__ __forceinline__ ArgBest better(ArgBest a, ArgBest b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ __forceinline__ ArgBest block_argmax(ArgBest cur) {
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest other{__shfl_xor_sync(0xffffffffu, cur.v, o), __shfl_xor_sync(0xffffffffu, cur.i, o)};
    cur = better(cur, other);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    sv[warp] = cur.v;
    si[warp] = cur.i;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    cur = lane < nw ? ArgBest{sv[lane], si[lane]} : ArgBest{-INFINITY, INT64_MAX};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgBest other{__shfl_xor_sync(0xffffffffu, cur.v, o), __shfl_xor_sync(0xffffffffu, cur.i, o)};
      cur = better(cur, other);
    }
  }
  return cur;
}

template <typename T>
__device__ __forceinline__ float load_f(const T* p, int64_t i);
template <>
__device__ __forceinline__ float load_f<bf16>(const bf16* p, int64_t i) { return to_f(p[i]); }
template <>
__device__ __forceinline__ float load_f<float>(const float* p, int64_t i) { return p[i]; }

template <typename T>
__global__ void argmax_kernel(int64_t* __restrict__ out_idx, float* __restrict__ out_val, const T* __restrict__ logits,
                              int64_t V) {
  pdl_trigger();
  pdl_wait();
  const T* row = logits + (int64_t)blockIdx.x * V;
  ArgBest best{-INFINITY, INT64_MAX};
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = load_f(row, i);
    if (v > best.v) best = ArgBest{v, i};   // strided scan: first hit per thread is its lowest index
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) {
    out_idx[blockIdx.x] = best.i == INT64_MAX ? 0 : best.i;
    out_val[blockIdx.x] = best.v;
  }
}

// SplitMix64 finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number generators",
// OOPSLA 2014) applied to a (seed, index) counter.
__device__ __forceinline__ float counter_uniform(uint64_t seed, uint64_t idx) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ull + idx * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

template <typename T>
__global__ void sample_kernel(int64_t* __restrict__ out, const T* __restrict__ logits, const float* __restrict__ temps,
                              int64_t V, uint64_t seed) {
  pdl_trigger();
  pdl_wait();
  const int64_t r = blockIdx.x;
  const T* row = logits + r * V;
  const float inv_t = 1.f / temps[r];
  ArgBest best{-INFINITY, INT64_MAX};
  for (int64_t i = threadIdx.x; i < V; i += blockDim.x) {
    const float u = counter_uniform(seed, (uint64_t)(r * V + i));
    const float score = load_f(row, i) * inv_t - logf(-logf(u));
    if (score > best.v) best = ArgBest{score, i};
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) out[r] = best.i == INT64_MAX ? 0 : best.i;
}

int grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16));
}

}  // namespace

void ensure_dynamic_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{func, dev}];
  if (bytes > have) {
    cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    have = bytes;
  }
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("LLMSERVE_PDL");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

int* status_ptr(const at::Tensor& status) { return status.defined() && status.numel() ? status.data_ptr<int>() : nullptr; }

// ---- host launchers ---------------------------------------------------------------------------
void rms_norm(at::Tensor out, at::Tensor x, at::Tensor w, double eps) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  check_bf16(w, "weight");
  const int H = x.size(-1);
  LSB_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  const int64_t rows = x.numel() / H;
  if (rows == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  launch_pdl(rmsnorm_kernel<false>, rows, norm_threads(H), H * sizeof(float), stream(), 
      (bf16*)out.data_ptr(), nullptr, (const bf16*)x.data_ptr(), nullptr, (const bf16*)w.data_ptr(), H, (float)eps);
}

void add_rms_norm(at::Tensor out, at::Tensor res_out, at::Tensor x, at::Tensor residual, at::Tensor w, double eps) {
  check_bf16(x, "x");
  check_bf16(residual, "residual");
  check_bf16(out, "out");
  check_bf16(res_out, "residual_out");
  const int H = x.size(-1);
  LSB_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  const int64_t rows = x.numel() / H;
  if (rows == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  launch_pdl(rmsnorm_kernel<true>, rows, norm_threads(H), H * sizeof(float), stream(), 
      (bf16*)out.data_ptr(), (bf16*)res_out.data_ptr(), (const bf16*)x.data_ptr(), (const bf16*)residual.data_ptr(),
      (const bf16*)w.data_ptr(), H, (float)eps);
}

void silu_and_mul(at::Tensor out, at::Tensor x) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  const int I = out.size(-1);
  LSB_CHECK(x.size(-1) == 2 * I && I % 8 == 0, "silu_and_mul expects [T, 2I] -> [T, I], I % 8 == 0");
  const int64_t vec = out.numel() / 8;
  if (vec == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  launch_pdl(silu_mul_kernel<false>, grid_for(vec, 256), 256, 0, stream(), (bf16*)out.data_ptr(),
             (const bf16*)x.data_ptr(), I, vec);
}

void silu_and_mul_interleaved(at::Tensor out, at::Tensor x) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  const int I = out.size(-1);
  LSB_CHECK(x.size(-1) == 2 * I && I % 64 == 0, "interleaved silu_and_mul expects [T, 2I] -> [T, I], I % 64 == 0");
  const int64_t vec = out.numel() / 8;
  if (vec == 0) return;
  const at::cuda::CUDAGuard g(x.device());
  launch_pdl(silu_mul_kernel<true>, grid_for(vec, 256), 256, 0, stream(), (bf16*)out.data_ptr(),
             (const bf16*)x.data_ptr(), I, vec);
}

void greedy_accept(at::Tensor out, at::Tensor target, at::Tensor draft, at::Tensor start) {
  LSB_CHECK(out.scalar_type() == at::kLong && target.scalar_type() == at::kLong && draft.scalar_type() == at::kLong &&
                start.scalar_type() == at::kLong, "greedy_accept: int64 tensors");
  LSB_CHECK(out.is_contiguous() && target.is_contiguous() && draft.is_contiguous() && start.is_contiguous(),
            "greedy_accept: contiguous tensors");
  const int B = draft.size(0), g = draft.size(1);
  LSB_CHECK(target.size(0) == B && target.size(1) == g + 1 && start.numel() == B && out.size(0) == B &&
                out.size(1) == g + 3, "greedy_accept: shapes [B, g+1], [B, g], [B] -> [B, g+3]");
  if (B == 0) return;
  const at::cuda::CUDAGuard guard(out.device());
  launch_pdl(greedy_accept_kernel, (B + 127) / 128, 128, 0, stream(), out.data_ptr<int64_t>(),
             target.data_ptr<int64_t>(), draft.data_ptr<int64_t>(), start.data_ptr<int64_t>(), B, g);
}

void feed_ids(at::Tensor out, at::Tensor ids, at::Tensor feed, at::Tensor prev, at::Tensor status) {
  LSB_CHECK(out.scalar_type() == at::kLong && ids.scalar_type() == at::kInt && feed.scalar_type() == at::kInt &&
                prev.scalar_type() == at::kLong, "feed_ids: out int64, ids/feed int32, prev int64");
  LSB_CHECK(out.is_contiguous() && ids.is_contiguous() && feed.is_contiguous() && prev.is_contiguous(),
            "feed_ids: contiguous tensors");
  const int n = out.numel();
  LSB_CHECK(ids.numel() == n && feed.numel() == n, "feed_ids: length mismatch");
  if (n == 0) return;
  const at::cuda::CUDAGuard g(out.device());
  launch_pdl(feed_ids_kernel, 1, 256, 0, stream(), out.data_ptr<int64_t>(), ids.data_ptr<int>(), feed.data_ptr<int>(),
             prev.data_ptr<int64_t>(), n, (int)prev.numel(), status_ptr(status));
}

void embedding(at::Tensor out, at::Tensor ids, at::Tensor table, at::Tensor status) {
  check_bf16(table, "table");
  check_bf16(out, "out");
  LSB_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be contiguous int64");
  const int H = table.size(1);
  LSB_CHECK(H % 8 == 0, "embedding width must be a multiple of 8");
  if (ids.numel() == 0) return;
  const at::cuda::CUDAGuard g(table.device());
  launch_pdl(embedding_kernel, ids.numel(), 128, 0, stream(), (bf16*)out.data_ptr(), ids.data_ptr<int64_t>(),
                                                      (const bf16*)table.data_ptr(), H, table.size(0),
                                                      status_ptr(status));
}

void qkv_rope(at::Tensor q_out, at::Tensor k_out, at::Tensor qkv, at::Tensor positions, at::Tensor cos_sin,
              at::Tensor q_w, at::Tensor k_w, double eps, at::Tensor k_cache, at::Tensor v_cache,
              at::Tensor slot_mapping, int64_t nh, int64_t nkv, int64_t hd, bool store, at::Tensor status) {
  // qkv: bf16 [T, W], or fp32 split-K partials [S, T, W] (S in 1, 2, 4, 8)
  const bool from_partials = qkv.scalar_type() == at::kFloat;
  int S = 0;
  if (from_partials) {
    LSB_CHECK(qkv.dim() == 3 && qkv.is_contiguous(), "qkv partials must be contiguous [S, T, W]");
    S = qkv.size(0);
    LSB_CHECK(S >= 1 && S <= 8, "qkv partial count must be 1..8");
    LSB_CHECK(store, "partials input needs the paged-store variant");
    qkv = qkv.view({S * qkv.size(1), qkv.size(2)});
  } else {
    check_bf16(qkv, "qkv");
  }
  check_bf16(q_out, "q_out");
  LSB_CHECK(positions.scalar_type() == at::kLong, "positions must be int64");
  LSB_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous(), "cos_sin cache must be fp32");
  LSB_CHECK(cos_sin.size(1) == hd, "cos_sin width must equal head_dim");
  LSB_CHECK(hd == 64 || hd == 128, "head_dim must be 64 or 128");
  LSB_CHECK(qkv.size(1) == (nh + 2 * nkv) * hd, "qkv width mismatch");
  const int T = from_partials ? qkv.size(0) / S : qkv.size(0);
  if (T == 0) return;
  const bf16* qw = q_w.numel() ? (const bf16*)q_w.data_ptr() : nullptr;
  const bf16* kw = k_w.numel() ? (const bf16*)k_w.data_ptr() : nullptr;
  int block_size = 1;
  int64_t num_slots = 0;
  if (store) {
    check_bf16(k_cache, "k_cache");
    check_bf16(v_cache, "v_cache");
    LSB_CHECK(slot_mapping.scalar_type() == at::kInt && slot_mapping.numel() == T, "slot_mapping must be int32 [T]");
    LSB_CHECK(k_cache.dim() == 4 && k_cache.size(1) == nkv && k_cache.size(3) == hd, "cache must be [blocks, nkv, bs, hd]");
    block_size = k_cache.size(2);
    num_slots = k_cache.size(0) * (int64_t)block_size;
  } else {
    check_bf16(k_out, "k_out");
  }
  const int heads = nh + 2 * nkv;
  const int warps = 4;
  dim3 grid(T, (heads + warps - 1) / warps);
  const at::cuda::CUDAGuard g(qkv.device());
#define LSB_ROPE(P, ST, SP)                                                                                     \
  launch_pdl(qkv_rope_kernel<P, ST, SP>, grid, warps * 32, 0, stream(), (bf16*)q_out.data_ptr(),              \
             ST ? nullptr : (bf16*)k_out.data_ptr(), SP ? nullptr : (const bf16*)qkv.data_ptr(),                  \
             SP ? qkv.data_ptr<float>() : nullptr, positions.data_ptr<int64_t>(), cos_sin.data_ptr<float>(), qw, \
             kw, (float)eps, ST ? (bf16*)k_cache.data_ptr() : nullptr, ST ? (bf16*)v_cache.data_ptr() : nullptr,  \
             ST ? slot_mapping.data_ptr<int>() : nullptr, T, (int)nh, (int)nkv, block_size, num_slots,            \
             status_ptr(status))
#define LSB_ROPE_S(P)                       \
  switch (S) {                              \
    case 0: LSB_ROPE(P, true, 0); break;    \
    case 1: LSB_ROPE(P, true, 1); break;    \
    case 2: LSB_ROPE(P, true, 2); break;    \
    case 3: LSB_ROPE(P, true, 3); break;    \
    case 4: LSB_ROPE(P, true, 4); break;    \
    case 5: LSB_ROPE(P, true, 5); break;    \
    case 6: LSB_ROPE(P, true, 6); break;    \
    case 7: LSB_ROPE(P, true, 7); break;    \
    default: LSB_ROPE(P, true, 8); break;   \
  }
  if (hd == 128) {
    if (store) { LSB_ROPE_S(2) } else LSB_ROPE(2, false, 0);
  } else {
    if (store) { LSB_ROPE_S(1) } else LSB_ROPE(1, false, 0);
  }
#undef LSB_ROPE_S
#undef LSB_ROPE
}

void store_kvcache(at::Tensor k, at::Tensor v, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slots,
                   at::Tensor status) {
  check_bf16(k, "k");
  check_bf16(v, "v");
  check_bf16(k_cache, "k_cache");
  check_bf16(v_cache, "v_cache");
  LSB_CHECK(slots.scalar_type() == at::kInt && slots.numel() == k.size(0), "slot_mapping must be int32 [T]");
  const int T = k.size(0), nkv = k.size(1), hd = k.size(2);
  LSB_CHECK(hd % 8 == 0 && k_cache.size(1) == nkv && k_cache.size(3) == hd, "cache shape mismatch");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(k.device());
  launch_pdl(store_kv_kernel, dim3(T, nkv), 32, 0, stream(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(),
                                                      (bf16*)k_cache.data_ptr(), (bf16*)v_cache.data_ptr(),
                                                      slots.data_ptr<int>(), nkv, hd, k_cache.size(2),
                                                      k_cache.size(0) * k_cache.size(2), status_ptr(status));
}

void commit_tree_kv(at::Tensor tk, at::Tensor tv, at::Tensor kc, at::Tensor vc, at::Tensor nodes, at::Tensor slots,
                    at::Tensor status) {
  check_bf16(tk, "tree_k");
  check_bf16(tv, "tree_v");
  check_bf16(kc, "k_cache");
  check_bf16(vc, "v_cache");
  const int L = tk.size(0), n = tk.size(1), nkv = tk.size(2), hd = tk.size(3);
  const int m = nodes.numel();
  if (m == 0) return;
  const at::cuda::CUDAGuard g(tk.device());
  launch_pdl(commit_tree_kv_kernel, dim3(L, m, nkv), 32, 0, stream(), 
      (const bf16*)tk.data_ptr(), (const bf16*)tv.data_ptr(), (bf16*)kc.data_ptr(), (bf16*)vc.data_ptr(),
      nodes.data_ptr<int>(), slots.data_ptr<int>(), n, nkv, hd, kc.size(3), kc.size(1), status_ptr(status));
}

void splitk_reduce(at::Tensor out, at::Tensor partials) {
  check_bf16(out, "out");
  LSB_CHECK(partials.scalar_type() == at::kFloat && partials.is_contiguous(), "partials must be fp32");
  const int S = partials.size(0);
  const int64_t TN = out.numel();
  LSB_CHECK(partials.numel() == S * TN && TN % 4 == 0, "partials shape mismatch");
  if (TN == 0) return;
  const at::cuda::CUDAGuard g(out.device());
  launch_pdl(splitk_reduce_kernel, grid_for(TN / 4, 256), 256, 0, stream(), (bf16*)out.data_ptr(), partials.data_ptr<float>(),
                                                                     S, TN);
}

void splitk_reduce_add_rmsnorm(at::Tensor out, at::Tensor res_out, at::Tensor partials, at::Tensor residual,
                               at::Tensor w, double eps) {
  check_bf16(out, "out");
  check_bf16(res_out, "residual_out");
  check_bf16(residual, "residual");
  LSB_CHECK(partials.scalar_type() == at::kFloat && partials.is_contiguous(), "partials must be fp32");
  const int S = partials.size(0), T = partials.size(1), N = partials.size(2);
  LSB_CHECK(N % 4 == 0 && residual.numel() == (int64_t)T * N, "shape mismatch");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(out.device());
  int threads = std::min(512, std::max(32, ((N / 4 + 31) / 32) * 32));
  auto args = std::make_tuple((bf16*)out.data_ptr(), (bf16*)res_out.data_ptr(), partials.data_ptr<float>(),
                              (const bf16*)residual.data_ptr(), (const bf16*)w.data_ptr(), S, T, N, (float)eps);
  if ((N == 4096 || N == 8192) && S >= 1 && S <= 8 && std::getenv("LLMSERVE_NORM_ROW_CTA") == nullptr) {
    // a cluster of 4 CTAs per row: one (N = 4096) or two float4 per thread and split
    auto cargs = std::make_tuple((bf16*)out.data_ptr(), (bf16*)res_out.data_ptr(), partials.data_ptr<float>(),
                                 (const bf16*)residual.data_ptr(), (const bf16*)w.data_ptr(), T, N, (float)eps);
    auto cgo = [&](auto kern) {
      std::apply([&](auto... a) { launch_pdl(kern, dim3(4, T), 256, 0, stream(), a...); }, cargs);
    };
#define LSB_NORM_CL(KP)                                                   \
    switch (S) {                                                          \
      case 1: cgo(splitk_add_rmsnorm_cluster_kernel<1, 4, KP>); break;    \
      case 2: cgo(splitk_add_rmsnorm_cluster_kernel<2, 4, KP>); break;    \
      case 3: cgo(splitk_add_rmsnorm_cluster_kernel<3, 4, KP>); break;    \
      case 4: cgo(splitk_add_rmsnorm_cluster_kernel<4, 4, KP>); break;    \
      case 5: cgo(splitk_add_rmsnorm_cluster_kernel<5, 4, KP>); break;    \
      case 6: cgo(splitk_add_rmsnorm_cluster_kernel<6, 4, KP>); break;    \
      case 7: cgo(splitk_add_rmsnorm_cluster_kernel<7, 4, KP>); break;    \
      default: cgo(splitk_add_rmsnorm_cluster_kernel<8, 4, KP>); break;   \
    }
    if (N == 4096) { LSB_NORM_CL(1) } else { LSB_NORM_CL(2) }
#undef LSB_NORM_CL
    return;
  }
  auto go = [&](auto kern) {
    std::apply([&](auto... a) { launch_pdl(kern, T, threads, N * sizeof(float), stream(), a...); }, args);
  };
  switch (S) {
    case 1: go(splitk_add_rmsnorm_kernel<1>); break;
    case 2: go(splitk_add_rmsnorm_kernel<2>); break;
    case 3: go(splitk_add_rmsnorm_kernel<3>); break;
    case 4: go(splitk_add_rmsnorm_kernel<4>); break;
    case 5: go(splitk_add_rmsnorm_kernel<5>); break;
    case 6: go(splitk_add_rmsnorm_kernel<6>); break;
    case 7: go(splitk_add_rmsnorm_kernel<7>); break;
    case 8: go(splitk_add_rmsnorm_kernel<8>); break;
    default: go(splitk_add_rmsnorm_kernel<0>); break;
  }
}

void splitk_silu(at::Tensor out, at::Tensor partials) {
  check_bf16(out, "out");
  LSB_CHECK(partials.scalar_type() == at::kFloat && partials.is_contiguous() && partials.dim() == 3, "bad partials");
  const int S = partials.size(0), T = partials.size(1), N = partials.size(2);
  LSB_CHECK(N % 128 == 0 && out.numel() == (int64_t)T * (N / 2), "interleaved gate/up shape mismatch");
  if (T == 0) return;
  const at::cuda::CUDAGuard g(out.device());
  launch_pdl(splitk_silu_kernel<true>, grid_for((int64_t)T * N / 2, 256), 256, 0, stream(), (bf16*)out.data_ptr(),
             partials.data_ptr<float>(), S, T, N);
}

// Same for a [gate | up] projection (the layout the checkpoint loader writes).
void argmax_rows(at::Tensor out_idx, at::Tensor out_val, at::Tensor logits) {
  LSB_CHECK(logits.is_cuda() && logits.is_contiguous() && logits.dim() == 2, "logits must be a contiguous CUDA matrix");
  const int64_t B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard g(logits.device());
  if (logits.scalar_type() == at::kBFloat16)
    launch_pdl(argmax_kernel<bf16>, B, 1024, 0, stream(), out_idx.data_ptr<int64_t>(), out_val.data_ptr<float>(),
                                                  (const bf16*)logits.data_ptr(), V);
  else if (logits.scalar_type() == at::kFloat)
    launch_pdl(argmax_kernel<float>, B, 1024, 0, stream(), out_idx.data_ptr<int64_t>(), out_val.data_ptr<float>(),
                                                   logits.data_ptr<float>(), V);
  else
    LSB_CHECK(false, "argmax supports bf16 and fp32 logits");
}

void sample_rows(at::Tensor out, at::Tensor logits, at::Tensor temps, int64_t seed) {
  LSB_CHECK(logits.is_cuda() && logits.is_contiguous() && logits.dim() == 2, "logits must be a contiguous CUDA matrix");
  const int64_t B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const at::cuda::CUDAGuard g(logits.device());
  if (logits.scalar_type() == at::kBFloat16)
    launch_pdl(sample_kernel<bf16>, B, 1024, 0, stream(), out.data_ptr<int64_t>(), (const bf16*)logits.data_ptr(),
                                                  temps.data_ptr<float>(), V, (uint64_t)seed);
  else
    launch_pdl(sample_kernel<float>, B, 1024, 0, stream(), out.data_ptr<int64_t>(), logits.data_ptr<float>(),
                                                   temps.data_ptr<float>(), V, (uint64_t)seed);
}

}  // namespace lsb
