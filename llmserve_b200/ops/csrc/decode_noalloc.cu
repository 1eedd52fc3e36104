// Split-KV paged decode attention with its scratch in a static device array (no allocation).
// See decode_noalloc.h for the contract; the kernel is the one behind decode_attention.
#include <stdint.h>
#include <stdio.h>

#include <mutex>

#include "attention_tiles.cuh"
#include "decode_noalloc.h"

namespace {

// Layout: [split counters: LSB_NOALLOC_MAX_PAIRS int32][max/sum: 2 floats per slot][O: head_dim floats per slot]
static __device__ __align__(256) unsigned char g_decode_scratch[LSB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_setup_mutex;
thread_local char g_error[256] = "";

int fail(int code, const char* msg) {
  snprintf(g_error, sizeof(g_error), "%s", msg);
  return code;
}

int partition_for(int pairs) { return pairs < 148 ? 128 : pairs < 296 ? 256 : 512; }

// Per-device set-up, run by the first call on that device (with it current).
int setup(int dev, void** addr) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      snprintf(g_error, sizeof(g_error), "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return -3;
    }
    const int s64 = lsb::decode_smem(64), s128 = lsb::decode_smem(128);
    if (cudaFuncSetAttribute(lsb::decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, s64) != cudaSuccess ||
        cudaFuncSetAttribute(lsb::decode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, s128) != cudaSuccess) {
      snprintf(g_error, sizeof(g_error), "cudaFuncSetAttribute failed: %s", cudaGetErrorString(cudaGetLastError()));
      return -3;
    }
    g_scratch_addr[dev] = p;
  }
  *addr = g_scratch_addr[dev];
  return 0;
}

}  // namespace

extern "C" int lsb_decode_attention_noalloc(void* out, const void* q, const void* k_cache, const void* v_cache,
                                            const int* block_tables, int block_table_stride,
                                            const int* context_lens, int batch, int num_heads, int num_kv_heads,
                                            int head_dim, int num_blocks, int block_size, float scale,
                                            cudaStream_t stream) {
  if (!out || !q || !k_cache || !v_cache || !block_tables || !context_lens)
    return fail(-1, "null pointer argument");
  if (batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_blocks <= 0 || block_size <= 0 ||
      block_table_stride <= 0)
    return fail(-1, "sizes must be positive");
  if (head_dim != 64 && head_dim != 128) return fail(-1, "head_dim must be 64 or 128");
  if (num_heads % num_kv_heads != 0 || num_heads / num_kv_heads > 16)
    return fail(-1, "num_heads must be a multiple of num_kv_heads with at most 16 per KV head");
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) % 4 != 0)
    return fail(-1, "k_cache / v_cache must be 16-byte aligned and q / out 4-byte aligned");
  const int64_t pairs = (int64_t)batch * num_kv_heads;
  if (pairs > LSB_NOALLOC_MAX_PAIRS) return fail(-2, "batch * num_kv_heads exceeds LSB_NOALLOC_MAX_PAIRS");
  const int partition = partition_for((int)pairs);
  const int64_t max_keys = (int64_t)block_table_stride * block_size;
  const int64_t max_splits = (max_keys + partition - 1) / partition;
  const int64_t slots = (int64_t)batch * num_heads * max_splits;
  const int64_t need = (int64_t)LSB_NOALLOC_MAX_PAIRS * 4 + slots * (2 + head_dim) * 4;
  if (need > (int64_t)LSB_NOALLOC_SCRATCH_BYTES)
    return fail(-2, "split partials exceed LSB_NOALLOC_SCRATCH_BYTES (too many sequences x heads x context)");

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return fail(-3, "cudaGetDevice failed");
  void* base = nullptr;
  if (int rc = setup(dev, &base)) return rc;
  int* counters = static_cast<int*>(base);
  float* part_ml = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + (size_t)LSB_NOALLOC_MAX_PAIRS * 4);
  float* part_o = part_ml + slots * 2;   // 8-byte multiple offset keeps float alignment

  // counters must start at zero for this call's (sequence, kv head) pairs
  cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)pairs * sizeof(int), stream);
  if (e != cudaSuccess) {
    snprintf(g_error, sizeof(g_error), "cudaMemsetAsync failed: %s", cudaGetErrorString(e));
    return -3;
  }
  const int z = (int)std::max<int64_t>(1, std::min<int64_t>(max_splits, (148 * 3 + pairs - 1) / pairs));
  dim3 grid(batch, num_kv_heads, z);
  const float sl = scale * lsb::kLog2e;
  if (head_dim == 128)
    lsb::launch_pdl(lsb::decode_kernel<128>, grid, dim3(lsb::NTHREADS), (size_t)lsb::decode_smem(128), stream,
                    (lsb::bf16*)out, (const lsb::bf16*)q, (const lsb::bf16*)k_cache, (const lsb::bf16*)v_cache,
                    block_tables, block_table_stride, context_lens, sl, part_o, part_ml, counters, (int)max_splits,
                    partition, num_heads, num_kv_heads, block_size, num_blocks, (int*)nullptr);
  else
    lsb::launch_pdl(lsb::decode_kernel<64>, grid, dim3(lsb::NTHREADS), (size_t)lsb::decode_smem(64), stream,
                    (lsb::bf16*)out, (const lsb::bf16*)q, (const lsb::bf16*)k_cache, (const lsb::bf16*)v_cache,
                    block_tables, block_table_stride, context_lens, sl, part_o, part_ml, counters, (int)max_splits,
                    partition, num_heads, num_kv_heads, block_size, num_blocks, (int*)nullptr);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(g_error, sizeof(g_error), "kernel launch failed: %s", cudaGetErrorString(e));
    return -3;
  }
  g_error[0] = '\0';
  return 0;
}

extern "C" const char* lsb_noalloc_last_error(void) { return g_error; }

extern "C" size_t lsb_noalloc_scratch_bytes(void) { return LSB_NOALLOC_SCRATCH_BYTES; }
