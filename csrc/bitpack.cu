// Standalone sm_100a kernels of the modular compression pipeline:
//
//   * BitPack codec — lossless fixed-width packing of uint8 symbols with the
//     16-byte header (magic 0x0150424B LE, bits, 3 zero bytes, count u64 LE)
//     and LSB-first symbol order of the reference
//     (kvserve_v1/compression/codec/bitpack_codec.py:20-69).  Instead of a
//     device assert (which would invalidate the CUDA context), an
//     out-of-range symbol or a header mismatch sets a status word that the
//     host reads back and raises on.
//   * FWHT — normalised Walsh-Hadamard transform of power-of-two row chunks
//     with optional Rademacher signs, fp32 math, one bf16 rounding
//     (the behaviour of kvserve_v1/compression/transformer/hadamard_func.py:75-231).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "kv_frame.h"
#include "ops.h"

namespace kvs {
namespace {

// One thread produces 8 output bytes = 64/bits symbols... instead, one thread
// packs a group of 8 symbols into `bits` bytes (byte aligned for any width).
__global__ void bitpack_pack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ out,
                                    int64_t n, int bits, uint32_t* status) {
  const int64_t groups = (n + 7) / 8;
  const uint32_t limit = 1u << bits;
  for (int64_t gi = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += int64_t(gridDim.x) * blockDim.x) {
    const int64_t first = gi * 8;
    uint64_t acc = 0;
    if (first + 8 <= n) {
      const uint2 raw = *reinterpret_cast<const uint2*>(src + first);
      const uint64_t w = uint64_t(raw.x) | (uint64_t(raw.y) << 32);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t q = uint32_t(w >> (8 * e)) & 0xffu;
        if (q >= limit) atomicCAS(status, 0u, uint32_t(kStatusBadSymbol));
        acc |= uint64_t(q & (limit - 1)) << (e * bits);
      }
    } else {
      for (int e = 0; first + e < n; ++e) {
        const uint32_t q = src[first + e];
        if (q >= limit) atomicCAS(status, 0u, uint32_t(kStatusBadSymbol));
        acc |= uint64_t(q & (limit - 1)) << (e * bits);
      }
    }
    // Bytes of this group: [gi*bits, gi*bits + bits) clipped to the stream size.
    const int64_t size = (n * bits + 7) / 8;
    uint8_t* dst = out + 16 + gi * bits;
    for (int i = 0; i < bits; ++i)
      if (gi * bits + i < size) dst[i] = uint8_t(acc >> (8 * i));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    uint32_t w[4] = {kBitpackMagic, uint32_t(bits), uint32_t(uint64_t(n)), uint32_t(uint64_t(n) >> 32)};
    *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void bitpack_unpack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ out,
                                      int64_t n, int bits, uint32_t* status) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const uint4 h = *reinterpret_cast<const uint4*>(src);
    if (h.x != kBitpackMagic || h.y != uint32_t(bits) || h.z != uint32_t(uint64_t(n)) ||
        h.w != uint32_t(uint64_t(n) >> 32))
      atomicCAS(status, 0u, uint32_t(kStatusBadHeader));
  }
  const int64_t groups = (n + 7) / 8;
  const int64_t size = (n * bits + 7) / 8;
  const uint64_t mask = (1ull << bits) - 1ull;
  for (int64_t gi = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; gi < groups;
       gi += int64_t(gridDim.x) * blockDim.x) {
    const uint8_t* s = src + 16 + gi * bits;
    uint64_t acc = 0;
    for (int i = 0; i < bits; ++i)
      if (gi * bits + i < size) acc |= uint64_t(s[i]) << (8 * i);
    const int64_t first = gi * 8;
    if (first + 8 <= n) {
      uint64_t w = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) w |= ((acc >> (e * bits)) & mask) << (8 * e);
      *reinterpret_cast<uint2*>(out + first) = make_uint2(uint32_t(w), uint32_t(w >> 32));
    } else {
      for (int e = 0; first + e < n; ++e) out[first + e] = uint8_t((acc >> (e * bits)) & mask);
    }
  }
}

// Row-chunk FWHT in shared memory: one CTA per row, chunks of descending
// powers of two (e.g. 96 -> 64 + 32), each normalised by 1/sqrt(chunk).
// mode 0: y = H(sign * x); mode 1 (inverse): y = sign * H(x).
__global__ void fwht_rows_kernel(const bf16* __restrict__ x, bf16* __restrict__ y, int64_t rows,
                                 int n, const float* __restrict__ signs, int64_t sign_period_rows,
                                 int inverse) {
  extern __shared__ float buf[];
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const bf16* xr = x + row * n;
    const float* sr = signs ? signs + (row % sign_period_rows) * n : nullptr;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v = to_f32(xr[i]);
      if (sr && !inverse) v *= sr[i];
      buf[i] = v;
    }
    __syncthreads();
    int start = 0, remaining = n;
    while (remaining > 0) {
      int chunk = 1;
      while (chunk * 2 <= remaining) chunk *= 2;
      for (int h = 1; h < chunk; h <<= 1) {
        for (int i = threadIdx.x; i < chunk / 2; i += blockDim.x) {
          const int lo = start + (i / h) * (2 * h) + (i % h);
          const float a = buf[lo], b = buf[lo + h];
          buf[lo] = a + b;
          buf[lo + h] = a - b;
        }
        __syncthreads();
      }
      const float sc = rsqrtf(float(chunk));
      for (int i = threadIdx.x; i < chunk; i += blockDim.x) buf[start + i] *= sc;
      __syncthreads();
      start += chunk;
      remaining -= chunk;
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      float v = buf[i];
      if (sr && inverse) v *= sr[i];
      y[row * n + i] = rn(v);
    }
    __syncthreads();
  }
}

int grid_for(int64_t work, int threads) {
  return int(std::max<int64_t>(1, std::min<int64_t>(ceil_div(work, threads), 148 * 16)));
}

}  // namespace

void bitpack_encode(torch::Tensor src, torch::Tensor out, int64_t bits, torch::Tensor status) {
  KVS_CHECK_ARG(src.is_cuda() && src.scalar_type() == at::kByte && src.is_contiguous(),
                "bitpack source must be contiguous CUDA uint8");
  KVS_CHECK_ARG(bits >= 1 && bits <= 8, "bitpack_bits must be in [1, 8]");
  const int64_t n = src.numel();
  KVS_CHECK_ARG(out.numel() == 16 + (n * bits + 7) / 8 && out.scalar_type() == at::kByte,
                "bitpack output size mismatch");
  KVS_CHECK_ARG((reinterpret_cast<uintptr_t>(src.data_ptr()) & 7) == 0 &&
                    (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
                "bitpack buffers must be aligned");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  bitpack_pack_kernel<<<grid_for((n + 7) / 8, 256), 256, 0, st>>>(
      src.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), n, int(bits),
      reinterpret_cast<uint32_t*>(status.data_ptr<int32_t>()));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void bitpack_decode(torch::Tensor src, torch::Tensor out, int64_t bits, torch::Tensor status) {
  KVS_CHECK_ARG(src.is_cuda() && src.scalar_type() == at::kByte && src.is_contiguous(),
                "bitpack payload must be contiguous CUDA uint8");
  KVS_CHECK_ARG(bits >= 1 && bits <= 8, "bitpack_bits must be in [1, 8]");
  const int64_t n = out.numel();
  KVS_CHECK_ARG(src.numel() == 16 + (n * bits + 7) / 8, "bitpack payload length does not match shape and bit width");
  KVS_CHECK_ARG((reinterpret_cast<uintptr_t>(src.data_ptr()) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(out.data_ptr()) & 7) == 0,
                "bitpack buffers must be aligned");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  bitpack_unpack_kernel<<<grid_for((n + 7) / 8, 256), 256, 0, st>>>(
      src.data_ptr<uint8_t>(), out.data_ptr<uint8_t>(), n, int(bits),
      reinterpret_cast<uint32_t*>(status.data_ptr<int32_t>()));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void fwht_rows(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> signs, bool inverse) {
  KVS_CHECK_ARG(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() &&
                    y.is_contiguous() && y.sizes() == x.sizes(),
                "fwht: contiguous CUDA bf16 in/out of equal shape");
  const int n = int(x.size(-1));
  KVS_CHECK_ARG(n >= 1 && n <= 8192, "fwht: last dim must be in [1, 8192]");
  const int64_t rows = x.numel() / n;
  const float* sp = nullptr;
  int64_t period = 1;
  if (signs.has_value()) {
    KVS_CHECK_ARG(signs->scalar_type() == at::kFloat && signs->is_contiguous() && signs->size(-1) == n,
                  "fwht: signs must be contiguous fp32 [..., n]");
    sp = signs->data_ptr<float>();
    period = signs->numel() / n;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int threads = std::min(512, std::max(32, n / 2));
  fwht_rows_kernel<<<grid_for(rows, 1), threads, size_t(n) * 4, st>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<bf16*>(y.data_ptr()), rows, n, sp,
      period, inverse ? 1 : 0);
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
