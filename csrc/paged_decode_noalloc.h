// C interface of the allocation-free paged decode attention entry point
// (paged_decode_noalloc.cu).  This interface has no counterpart in the
// reference project.
//
// It is for callers that cannot allocate device memory while they launch
// work: a serving loop that gave the whole device pool to its KV cache, code
// that runs inside an allocator or memory-accounting hook (a cudaMalloc there
// would re-enter the allocator), or a C/C++ program without PyTorch.  The
// entry point keeps its split-K scratch in a fixed module-global array and
// allocates nothing; the caller passes every input and the output.
//
// Plain C, no PyTorch types: include it from C or C++ and link against the
// extension library (kvserve_b200/_C*.so), or bind the symbols with ctypes.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Status codes returned by kvs_paged_decode_attention_noalloc.
enum KvsNoallocStatus {
  KVS_NOALLOC_OK = 0,
  // A null pointer, an unsupported shape (head_dim 64 or 128; 1, 2, 4 or 8
  // query heads per KV head), a pointer not aligned to 16 bytes or an element
  // stride that is not a multiple of 8.  Nothing was launched.
  KVS_NOALLOC_BAD_ARGUMENT = 1,
  // batch x query_heads x splits exceeds the scratch capacity
  // (kvs_paged_decode_noalloc_capacity()).  Nothing was launched.
  KVS_NOALLOC_TOO_LARGE = 2,
  // A CUDA call of this function failed; kvs_noalloc_last_cuda_error() gives
  // the cudaError_t value.
  KVS_NOALLOC_CUDA_ERROR = 3,
  // The calling thread already had an unread CUDA error when the call began.
  // Nothing was launched and that error was left in place for its owner.
  KVS_NOALLOC_PENDING_ERROR = 4,
};

// Text for a status code (static storage, never freed).
const char* kvs_noalloc_error_string(int code);

// Largest number of split-K partial records (batch x query_heads x splits)
// one call may need.
int64_t kvs_paged_decode_noalloc_capacity(void);

// cudaError_t of the last failing CUDA call made by this entry point on the
// calling thread (0 when none failed).
int kvs_noalloc_last_cuda_error(void);

// Single-token GQA attention over a paged bf16 KV cache, without allocating.
//   q            [batch, num_q_heads, head_dim], q_batch_stride elements between rows
//   k/v_cache    [num_blocks, block_size, num_kv_heads, head_dim] with element strides
//                block_stride, token_stride, head_stride (head_dim contiguous)
//   block_tables int32 [batch, block_table_stride]
//   context_lens int32 [batch], each <= max_context
//   out          [batch, num_q_heads, head_dim], out_batch_stride elements between rows
//   stream       a cudaStream_t (NULL: the legacy default stream)
// Pointers must be device memory of the current device, 16-byte aligned, and
// every element stride a multiple of 8.  The call is stream-ordered and
// returns before the work finishes.  Calls share one scratch array: calls that
// may overlap on the GPU race on it, so order them on one stream.  The first
// call on a device looks up the array's device address; make that call before
// any stream capture.
int kvs_paged_decode_attention_noalloc(const void* q, int64_t q_batch_stride, const void* k_cache,
                                       const void* v_cache, int64_t block_stride, int64_t token_stride,
                                       int64_t head_stride, const int32_t* block_tables,
                                       int64_t block_table_stride, const int32_t* context_lens, int batch,
                                       int num_q_heads, int num_kv_heads, int head_dim, int block_size,
                                       int max_context, float scale, void* out, int64_t out_batch_stride,
                                       void* stream);

#ifdef __cplusplus
}
#endif
