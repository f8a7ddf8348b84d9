// Decode-step (small M) bf16 GEMM: y[M, N] = x[M, K] * W[N, K]^T, M <= 8.
// Weight streaming is the whole cost, so each warp owns ROWS output rows and
// keeps ROWS x UNROLL independent 16-byte weight loads in flight; x lives in
// shared memory (bf16, 16-byte loads).  Used for every projection of a decode step and for
// the LM head (where the tcgen05 tile kernel would leave SMs idle).  A PDL launch: the
// first weight loads are in flight before the kernel waits for its predecessor.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "gemv_core.cuh"
#include "ops.h"

namespace kvs {
namespace {

constexpr int kThreads = kGemvThreads;

// THREADS: 256, or 512 when x is so large that only one CTA fits per SM
// (that CTA must then keep twice the weight loads in flight).
template <int M, int THREADS>
__global__ void __launch_bounds__(THREADS) gemv_kernel(const bf16* __restrict__ x, int64_t ldx,
                                                        const bf16* __restrict__ w, int64_t ldw,
                                                        bf16* __restrict__ y, int64_t ldy, int N, int K,
                                                        const bf16* __restrict__ bias) {
  extern __shared__ uint4 xs_raw[];  // [M][K] bf16
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kRows = THREADS / 32 * kGemvRows;   // rows per block
  const int nblk = (N + kRows - 1) / kRows;
  pdl_trigger();
  GemvWarp<M> g;
  g.prefetch(w, ldw, (blockIdx.x * (THREADS / 32) + warp) * kGemvRows, N, K, lane);
  pdl_wait();   // x is the previous kernel's output
  gemv_stage_x<M>(x, ldx, xs_raw, K);
  __syncthreads();
  // a CTA takes row blocks blockIdx.x, blockIdx.x + gridDim.x, ... so x is
  // staged once per CTA (with several tokens the grid is one wave)
  for (int blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const int row0 = (blk * (THREADS / 32) + warp) * kGemvRows;
    if (row0 < N) {
      float acc[kGemvRows][M];
      g.run(w, ldw, reinterpret_cast<const bf16*>(xs_raw), row0, N, K, lane, acc);
      if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
          if (row0 + r >= N) break;
#pragma unroll
          for (int m = 0; m < M; ++m)
            y[int64_t(m) * ldy + row0 + r] = rn(acc[r][m] + (bias ? to_f32(bias[row0 + r]) : 0.f));
        }
      }
    }
    g.have = false;
  }
}

// CTAs of a GEMV kernel resident at once with `smem` bytes of x (cached).
template <typename Kern>
int gemv_wave(Kern kern, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kern), smem);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  int per_sm = 0, dev = 0, sms = 0;
  KVS_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem));
  KVS_CUDA_CHECK(cudaGetDevice(&dev));
  KVS_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return cache[key] = std::max(1, per_sm) * sms;
}

// Resident CTAs of gemv_kernel<M, THR> over the GPU (sets its shared-memory limit first).
template <int M, int THR>
int gemv_capacity(size_t smem) {
  static bool set = false;
  if (!set) {
    KVS_CUDA_CHECK(cudaFuncSetAttribute(gemv_kernel<M, THR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
    set = true;
  }
  return gemv_wave(gemv_kernel<M, THR>, THR, smem);
}

// Few tokens: one row block per CTA.  4+ tokens: one wave, so each CTA stages
// x (read from L2 again by every CTA) once for all its row blocks.
template <int M, int THR>
void launch_gemv(size_t smem, cudaStream_t st, const bf16* xp, int64_t ldx, const bf16* wp, int64_t ldw, bf16* yp,
                 int64_t ldy, int N, int K, const bf16* bp) {
  const int cap = gemv_capacity<M, THR>(smem);
  const int nblk = (N + THR / 32 * kGemvRows - 1) / (THR / 32 * kGemvRows);
  const int grid = M >= 4 ? std::min(nblk, cap) : nblk;
  launch_pdl(gemv_kernel<M, THR>, dim3(grid), dim3(THR), smem, st, xp, ldx, wp, ldw, yp, ldy, N, K, bp);
}

// 4+ tokens: 512-thread CTAs when they keep at least as many warps resident
// as 256-thread ones (x is then staged half as often); measured at M = 8:
// 2.4-2.5 TB/s against 1.9-2.1 with 256 threads.
template <int M>
bool gemv_wide(size_t smem) {
  if (M < 4) return false;
  return gemv_capacity<M, 512>(smem) * 16 >= gemv_capacity<M, kThreads>(smem) * (kThreads / 32);
}

}  // namespace

void gemv_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor y, c10::optional<torch::Tensor> bias) {
  KVS_CHECK_ARG(x.is_cuda() && w.is_cuda() && y.is_cuda() && x.scalar_type() == at::kBFloat16 &&
                    w.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16,
                "gemv: CUDA bf16");
  KVS_CHECK_ARG(x.dim() == 2 && w.dim() == 2 && y.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1 &&
                    y.stride(1) == 1,
                "gemv: row-major 2-D operands");
  const int M = int(x.size(0)), K = int(x.size(1)), N = int(w.size(0));
  KVS_CHECK_ARG(w.size(1) == K && y.size(0) == M && y.size(1) == N, "gemv: shape mismatch");
  KVS_CHECK_ARG(M >= 1 && M <= 8, "gemv: 1 <= M <= 8");
  KVS_CHECK_ARG(K % 8 == 0 && w.stride(0) % 8 == 0, "gemv: K must be a multiple of 8");
  KVS_CHECK_ARG(x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0, "gemv: leading dims must be multiples of 8");
  KVS_CHECK_ARG(size_t(K) * 2 <= 200 * 1024, "gemv: K too large");
  // Rows of x are staged in shared memory; split M when they do not fit.
  const int max_rows = int(std::min<size_t>(8, (200 * 1024) / (size_t(K) * 2)));
  if (M > max_rows) {
    for (int m0 = 0; m0 < M; m0 += max_rows) {
      const int mm = std::min(max_rows, M - m0);
      gemv_bf16(x.narrow(0, m0, mm), w, y.narrow(0, m0, mm), bias);
    }
    return;
  }
  const bf16* bp = nullptr;
  if (bias.has_value()) {
    KVS_CHECK_ARG(bias->numel() == N && bias->is_contiguous() && bias->scalar_type() == at::kBFloat16,
                  "gemv: bias must be contiguous bf16 [N]");
    bp = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  const size_t smem = size_t(M) * K * 2;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto yp = reinterpret_cast<bf16*>(y.data_ptr());
#define KVS_GEMV_CASE(MM)                                                                                  \
  case MM:                                                                                                 \
    if (gemv_wide<MM>(smem))                                                                               \
      launch_gemv<MM, 512>(smem, st, xp, x.stride(0), wp, w.stride(0), yp, y.stride(0), N, K, bp);        \
    else                                                                                                   \
      launch_gemv<MM, kThreads>(smem, st, xp, x.stride(0), wp, w.stride(0), yp, y.stride(0), N, K, bp);   \
    break;
  switch (M) {
    KVS_GEMV_CASE(1)
    KVS_GEMV_CASE(2)
    KVS_GEMV_CASE(3)
    KVS_GEMV_CASE(4)
    KVS_GEMV_CASE(5)
    KVS_GEMV_CASE(6)
    KVS_GEMV_CASE(7)
    KVS_GEMV_CASE(8)
  }
#undef KVS_GEMV_CASE
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
