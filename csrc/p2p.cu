// Peer-memory plumbing for the NVLink KV hand-off.
//
// The decode GPU allocates its receive slots and flag words with plain
// cudaMalloc (outside the PyTorch caching allocator, so that the block can be
// exported), exports them with CUDA IPC, and the prefill GPU maps them with
// cudaIpcOpenMemHandle(..., cudaIpcMemLazyEnablePeerAccess).  Kernels then
// store straight into the mapped address over NVLink 5 / NVSwitch.  This
// replaces the reference's NCCL send/recv of KV bundles
// (kvserve_v1/transport/nccl_transport.py:435-445, 649-656).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "ops.h"

namespace kvs {
namespace {
__global__ void fill_u32_kernel(uint32_t* p, uint32_t v, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    p[i] = v;
}
__global__ void read_u32_kernel(const uint32_t* p, uint32_t* out, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    out[i] = ld_acquire_sys_u32(p + i);
}
__global__ void store_release_kernel(uint32_t* p, uint32_t v) {
  __threadfence_system();
  st_release_sys_u32(p, v);
}
// Bounded device-side wait used by tests of the timeout path: polls a flag
// for at most timeout_ns and records kStatusTimeout instead of hanging.
__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns,
                                 uint32_t* status) {
  if (!wait_flag_geq(flag, target, timeout_ns)) atomicCAS(status, 0u, uint32_t(kStatusTimeout));
}
// First-token hand-off: the prefill rank publishes the sampled token next to
// the layer flags of the decode rank's receive slot (value, then the request
// sequence number with release semantics); the decode rank acquire-waits
// (bounded) and copies the token into its decode state.
__global__ void publish_token_kernel(const int32_t* tok, uint32_t* dst, uint32_t seq) {
  dst[0] = uint32_t(tok[0]);
  __threadfence_system();
  st_release_sys_u32(dst + 1, seq);
}
__global__ void take_token_kernel(const uint32_t* src, uint32_t seq, uint64_t timeout_ns, int32_t* out,
                                  int32_t* out2, uint32_t* status) {
  if (!wait_flag_geq(src + 1, seq, timeout_ns)) {
    atomicCAS(status, 0u, uint32_t(kStatusTimeout));
    return;
  }
  const int32_t t = int32_t(ld_acquire_sys_u32(src));
  out[0] = t;
  if (out2) out2[0] = t;
}
}  // namespace

void publish_token(torch::Tensor tok, int64_t dst_ptr, int64_t seq) {
  KVS_CHECK_ARG(tok.scalar_type() == at::kInt && tok.is_cuda() && tok.numel() >= 1, "publish_token: int32 token");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  publish_token_kernel<<<1, 1, 0, st>>>(tok.data_ptr<int32_t>(), reinterpret_cast<uint32_t*>(dst_ptr),
                                        uint32_t(seq));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void take_token(int64_t src_ptr, int64_t seq, int64_t timeout_ns, torch::Tensor out,
                c10::optional<torch::Tensor> out2, torch::Tensor status) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  take_token_kernel<<<1, 1, 0, st>>>(reinterpret_cast<const uint32_t*>(src_ptr), uint32_t(seq),
                                     uint64_t(timeout_ns), out.data_ptr<int32_t>(),
                                     out2.has_value() ? out2->data_ptr<int32_t>() : nullptr,
                                     reinterpret_cast<uint32_t*>(status.data_ptr<int32_t>()));
  KVS_CUDA_CHECK(cudaGetLastError());
}

int64_t dev_alloc(int64_t bytes) {
  void* p = nullptr;
  KVS_CUDA_CHECK(cudaMalloc(&p, size_t(std::max<int64_t>(bytes, 256))));
  KVS_CUDA_CHECK(cudaMemset(p, 0, size_t(std::max<int64_t>(bytes, 256))));
  return reinterpret_cast<int64_t>(p);
}

void dev_free(int64_t ptr) {
  if (ptr) KVS_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

std::string ipc_get_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  KVS_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open_handle(const std::string& handle) {
  KVS_CHECK_ARG(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  KVS_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) {
  if (ptr) KVS_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

bool can_access_peer(int64_t dev, int64_t peer) {
  int ok = 0;
  KVS_CUDA_CHECK(cudaDeviceCanAccessPeer(&ok, int(dev), int(peer)));
  return ok != 0;
}

torch::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, int64_t dtype_code, int64_t device) {
  const auto dtype = static_cast<c10::ScalarType>(dtype_code);
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, int(device));
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {}, opts);
}

void fill_u32(int64_t ptr, int64_t value, int64_t count) {
  if (count <= 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int grid = int(std::min<int64_t>(ceil_div(count, 256), 1024));
  fill_u32_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<uint32_t*>(ptr), uint32_t(value), count);
  KVS_CUDA_CHECK(cudaGetLastError());
}

void read_u32(int64_t ptr, torch::Tensor out) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t n = out.numel();
  read_u32_kernel<<<int(std::min<int64_t>(ceil_div(n, 256), 1024)), 256, 0, st>>>(
      reinterpret_cast<const uint32_t*>(ptr), reinterpret_cast<uint32_t*>(out.data_ptr<int32_t>()), n);
  KVS_CUDA_CHECK(cudaGetLastError());
}

void store_release_u32(int64_t ptr, int64_t value) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  store_release_kernel<<<1, 1, 0, st>>>(reinterpret_cast<uint32_t*>(ptr), uint32_t(value));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void wait_flag(int64_t flag_ptr, int64_t target, int64_t timeout_ns, torch::Tensor status) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  wait_flag_kernel<<<1, 32, 0, st>>>(reinterpret_cast<const uint32_t*>(flag_ptr), uint32_t(target),
                                     uint64_t(timeout_ns),
                                     reinterpret_cast<uint32_t*>(status.data_ptr<int32_t>()));
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
