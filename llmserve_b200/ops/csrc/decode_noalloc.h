// C entry point for split-KV paged decode attention that allocates no device memory.
//
// This entry point has no counterpart in the reference implementation; it exists for callers
// of this library that cannot allocate GPU memory themselves, e.g. code running inside a host
// framework that owns every device allocation through its own pool (or forbids allocation on
// the serving path), or a plugin that is handed pointers and a stream and nothing else.  Those
// callers cannot provide the workspace that llmserve_b200._C.decode_attention takes, so this
// variant keeps its scratch in a fixed-size static device array inside the library instead.
//
// Tensors (all device pointers, row-major, contiguous):
//   out, q        bf16 [batch, num_heads, head_dim]
//   k_cache,
//   v_cache       bf16 [num_blocks, num_kv_heads, block_size, head_dim]   (16-byte aligned)
//   block_tables  int32 [batch, block_table_stride]
//   context_lens  int32 [batch]
//
// Inputs the host cannot check without a synchronisation are made safe on the device: a context
// longer than block_table_stride * block_size is clamped to it (so block-table reads and split
// slots stay inside what was sized here), and a block id outside [0, num_blocks) is never
// dereferenced -- its keys and values read as zeros.  Both give a defined result for garbage in,
// not an error code.  A context of 0 writes zeros.
//
// Limits: head_dim 64 or 128; num_heads a multiple of num_kv_heads with at most 16 query heads
// per KV head; batch * num_kv_heads <= LSB_NOALLOC_MAX_PAIRS; and the split partials
//   batch * num_heads * ceil(block_table_stride * block_size / partition) * (head_dim + 2) * 4 B
// must fit in LSB_NOALLOC_SCRATCH_BYTES - LSB_NOALLOC_MAX_PAIRS * 4 (partition = 128, 256 or
// 512 keys, chosen from batch * num_kv_heads).  Larger requests are rejected, nothing is launched.
//
// The scratch array is shared by every call in the process on a given GPU and keeps the last
// call's contents; the split counters are cleared by every call.  Calls whose executions overlap
// on the GPU (different streams without ordering) race on the scratch and give wrong results:
// order them on one stream or serialise them.  Every GPU that loads the library holds the array
// (LSB_NOALLOC_SCRATCH_BYTES) until the process exits.
//
// The first call on a device looks up the array's device address (cudaGetSymbolAddress) and
// sets the kernel's shared-memory attribute with that device current; make that first call
// before capturing any stream into a CUDA graph.
//
// Returns 0 on success, or a negative code with a message from lsb_noalloc_last_error():
//   -1 invalid argument, -2 request exceeds the scratch limits, -3 CUDA error.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#define LSB_NOALLOC_SCRATCH_BYTES (16u << 20)
#define LSB_NOALLOC_MAX_PAIRS 16384

#ifdef __cplusplus
extern "C" {
#endif

int lsb_decode_attention_noalloc(void* out, const void* q, const void* k_cache, const void* v_cache,
                                 const int* block_tables, int block_table_stride, const int* context_lens,
                                 int batch, int num_heads, int num_kv_heads, int head_dim, int num_blocks,
                                 int block_size, float scale, cudaStream_t stream);

const char* lsb_noalloc_last_error(void);

size_t lsb_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif
