// Allocation-free C entry point for split-K paged decode attention.
//
// This entry point has no counterpart in the reference project.
//
// Who it is for: callers that cannot allocate device memory at the moment
// they launch work — for example a serving loop that has handed the whole GPU
// memory pool to its KV cache up front, code running inside a custom
// allocator or a memory-accounting hook (where calling cudaMalloc would
// re-enter the allocator), or a C/C++ host program without PyTorch and its
// caching allocator.  The regular entry point (paged_decode_attention in
// attention_decode.cu) needs a temporary buffer for the per-split partial
// results; here that buffer is a fixed array in the module's own global
// memory instead, so a call allocates nothing: no cudaMalloc, no cudaFree,
// no allocating library routine.  The caller still provides every input and
// the output.
//
// Limits and rules:
//   * The scratch array holds kMaxRecords partial records of up to 128 floats
//     (batch x query_heads x splits <= 2048, head_dim <= 128; about 1.1 MB).
//     Every GPU that loads this library keeps that array until the process
//     exits.  A call whose split schedule would need more records is rejected
//     with KVS_NOALLOC_TOO_LARGE before anything is launched.
//   * All calls share the one array.  Calls whose work may overlap on the GPU
//     (different streams without ordering, or different host threads) race on
//     it and produce wrong results; order them on one stream.
//   * Nothing in the array has to start at zero: every partial record that a
//     call reads is written earlier by the same call, so contents left over
//     from a previous call are never used.
//   * The first call on a device looks up the device address of the array
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before capturing a stream into a CUDA graph.
//   * The device that is current when calling must own every pointer passed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "attention_decode_kernels.cuh"
#include "common.cuh"
#include "ops.h"
#include "paged_decode_noalloc.h"

namespace {

constexpr int64_t kMaxRecords = 2048;  // batch * query_heads * splits
constexpr int64_t kMaxHeadDim = 128;
constexpr int64_t kScratchFloats = kMaxRecords * kMaxHeadDim + kMaxRecords * 2;
constexpr int kMaxDevices = 64;

// The scratch lives in the module's global memory; in host code the name is
// only a host-side handle, never a device address.
static __device__ __align__(256) float g_decode_scratch[kScratchFloats];

std::mutex g_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// cudaError_t of the last failing CUDA call, per calling thread.
thread_local int t_last_cuda_error = 0;

int cuda_failed(cudaError_t e) {
  t_last_cuda_error = int(e);
  return KVS_NOALLOC_CUDA_ERROR;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Device address of the scratch array for the current device (looked up once).
int scratch_for_current_device(float** out) {
  int dev = -1;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return cuda_failed(de);
  if (dev < 0 || dev >= kMaxDevices) return cuda_failed(cudaErrorInvalidDevice);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return cuda_failed(e);
    if (p == nullptr) return cuda_failed(cudaErrorInvalidSymbol);
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return KVS_NOALLOC_OK;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* kvs_noalloc_error_string(int code) {
  switch (code) {
    case KVS_NOALLOC_OK: return "ok";
    case KVS_NOALLOC_BAD_ARGUMENT:
      return "invalid argument (null pointer, head_dim not 64/128, not 1/2/4/8 query heads per KV head, "
             "pointer not 16-byte aligned or element stride not a multiple of 8); nothing was launched";
    case KVS_NOALLOC_TOO_LARGE:
      return "batch x query_heads x splits exceeds the fixed scratch capacity of 2048 records; nothing was launched";
    case KVS_NOALLOC_CUDA_ERROR: return "a CUDA call failed (its code: kvs_noalloc_last_cuda_error())";
    case KVS_NOALLOC_PENDING_ERROR:
      return "the calling thread had an unread CUDA error before the call; nothing was launched";
    default: return "unknown status";
  }
}

__attribute__((visibility("default"))) int64_t kvs_paged_decode_noalloc_capacity(void) { return kMaxRecords; }

__attribute__((visibility("default"))) int kvs_noalloc_last_cuda_error(void) { return t_last_cuda_error; }

// Single-token GQA attention over a paged KV cache, like the regular entry
// point, without allocating (declared in paged_decode_noalloc.h).  Layouts
// (bf16, innermost dimension contiguous):
//   q       [batch, num_q_heads, head_dim]          (q_batch_stride elements between rows)
//   k/v     [num_blocks, block_size, num_kv_heads, head_dim] with the given strides
//   out     [batch, num_q_heads, head_dim]          (out_batch_stride elements between rows)
//   block_tables int32 [batch, block_table_stride], context_lens int32 [batch]
// Returns 0 on success or a KvsNoallocStatus code (kvs_noalloc_error_string).
__attribute__((visibility("default"))) int kvs_paged_decode_attention_noalloc(
    const void* q, int64_t q_batch_stride, const void* k_cache, const void* v_cache, int64_t block_stride,
    int64_t token_stride, int64_t head_stride, const int32_t* block_tables, int64_t block_table_stride,
    const int32_t* context_lens, int batch, int num_q_heads, int num_kv_heads, int head_dim, int block_size,
    int max_context, float scale, void* out, int64_t out_batch_stride, void* stream) {
  using namespace kvs;
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || block_tables == nullptr ||
      context_lens == nullptr || out == nullptr || batch < 1 || num_q_heads < 1 || num_kv_heads < 1 ||
      num_q_heads % num_kv_heads != 0 || block_size < 1 || max_context < 1)
    return KVS_NOALLOC_BAD_ARGUMENT;
  if (head_dim != 64 && head_dim != 128) return KVS_NOALLOC_BAD_ARGUMENT;
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return KVS_NOALLOC_BAD_ARGUMENT;
  // the kernels move 16-byte vectors of q, K, V and out: every base pointer
  // and every element stride (bf16, 8 per vector) must keep that alignment
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out)) return KVS_NOALLOC_BAD_ARGUMENT;
  if (q_batch_stride % 8 || block_stride % 8 || token_stride % 8 || head_stride % 8 || out_batch_stride % 8)
    return KVS_NOALLOC_BAD_ARGUMENT;
  // q/out rows hold num_q_heads contiguous heads; K/V heads must not overlap
  // (token and block strides are free: NHD and HND caches both work)
  if (q_batch_stride < int64_t(num_q_heads) * head_dim || out_batch_stride < int64_t(num_q_heads) * head_dim ||
      head_stride < head_dim || token_stride < 1 || block_stride < 1 || block_table_stride < 1)
    return KVS_NOALLOC_BAD_ARGUMENT;
  // an error left unread by earlier work is the caller's; do not clear it and
  // do not report it as this call's failure
  if (cudaPeekAtLastError() != cudaSuccess) return KVS_NOALLOC_PENDING_ERROR;
  t_last_cuda_error = 0;
  int64_t splits = paged_decode_splits(batch, num_kv_heads, max_context);
  const int chunk = int(std::max<int64_t>(16, ((max_context + splits - 1) / splits + 15) / 16 * 16));
  splits = (max_context + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  if (splits > 1 && int64_t(batch) * num_q_heads * splits > kMaxRecords) return KVS_NOALLOC_TOO_LARGE;
  float* scratch = nullptr;
  const int st_code = scratch_for_current_device(&scratch);
  if (st_code != KVS_NOALLOC_OK) return st_code;
  const int64_t records = int64_t(batch) * num_q_heads * splits;
  float* part_o = splits > 1 ? scratch : nullptr;
  float* part_ml = splits > 1 ? scratch + records * head_dim : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid(int(splits), num_kv_heads, batch);
  const float sl2 = scale * 1.4426950408889634f;
  auto qp = static_cast<const bf16*>(q);
  auto kp = static_cast<const bf16*>(k_cache);
  auto vp = static_cast<const bf16*>(v_cache);
  auto op = static_cast<bf16*>(out);
  if (head_dim == 128)
    launch_decode<128>(G, grid, st, qp, q_batch_stride, kp, vp, block_stride, token_stride, head_stride, block_tables,
                       block_table_stride, context_lens, block_size, num_q_heads, int(splits), chunk, sl2, part_o,
                       part_ml, op, out_batch_stride);
  else
    launch_decode<64>(G, grid, st, qp, q_batch_stride, kp, vp, block_stride, token_stride, head_stride, block_tables,
                      block_table_stride, context_lens, block_size, num_q_heads, int(splits), chunk, sl2, part_o,
                      part_ml, op, out_batch_stride);
  // no error was pending at entry, so an error now belongs to this launch
  const cudaError_t e1 = cudaGetLastError();
  if (e1 != cudaSuccess) return cuda_failed(e1);
  if (splits > 1) {
    dim3 g2(num_q_heads, batch);
    if (head_dim == 128)
      merge_splits_kernel<128><<<g2, 128, 0, st>>>(part_o, part_ml, num_q_heads, int(splits), op, out_batch_stride);
    else
      merge_splits_kernel<64><<<g2, 64, 0, st>>>(part_o, part_ml, num_q_heads, int(splits), op, out_batch_stride);
    const cudaError_t e2 = cudaGetLastError();
    if (e2 != cudaSuccess) return cuda_failed(e2);
  }
  return KVS_NOALLOC_OK;
}

}  // extern "C"
