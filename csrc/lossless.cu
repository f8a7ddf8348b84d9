// Lossless byte codec on sm_100a: per chunk, tuple shuffle (8-byte tuples
// -> 8 byte planes), bit shuffle (8 bit planes, LSB-first) and zero-word
// elimination over 16-bit words (bitmap + non-zero words) — the
// "TUPL8_1 BIT_8 RZE_2" chain in LC-framework notation (Burtscher et al.),
// implemented from the published method; container "kvs-rze-v1":
//   [0,24)  "KVLZ", u32 version=1, u64 total bytes, u32 chunk bytes, u32 chunks
//   u32 size per chunk (bit 31 = stored raw), then the chunks, 4-byte aligned.
//
// Encode = three launches, no host round trip until the caller asks for the
// size: (1) one CTA per chunk codes into a fixed per-chunk scratch slot and
// records its size, (2) one CTA scans the sizes into offsets and writes the
// header/size table and the total, (3) one CTA per chunk compacts its slot
// into the output.  Decode = (1) scan, (2) one CTA per chunk restores.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "ops.h"

namespace kvs {
namespace {

constexpr int kChunk = 16384;
constexpr int kThreads = 512;
constexpr uint32_t kRawFlag = 1u << 31;
constexpr int kHeader = 24;

__host__ __device__ inline int pad16(int n) { return (n + 15) / 16 * 16; }
__host__ __device__ inline int64_t slot_bytes(int chunk) { return int64_t(chunk) / 16 + chunk + 16; }

// 8x8 bit-matrix transpose: byte k of x, bit b  ->  byte b of result, bit k.
__device__ __forceinline__ uint64_t transpose8(uint64_t x) {
  uint64_t t;
  t = (x ^ (x >> 7)) & 0x00AA00AA00AA00AAull; x = x ^ t ^ (t << 7);
  t = (x ^ (x >> 14)) & 0x0000CCCC0000CCCCull; x = x ^ t ^ (t << 14);
  t = (x ^ (x >> 28)) & 0x00000000F0F0F0F0ull; x = x ^ t ^ (t << 28);
  return x;
}

// Exclusive block-wide prefix sum of one int per thread; returns the total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < (blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < (blockDim.x >> 5)) warp_sums[lane] = s;
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  total = warp_sums[(blockDim.x >> 5) - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kThreads) rze_encode_chunks(const uint8_t* __restrict__ src, int64_t total,
                                                              int chunk, uint8_t* __restrict__ scratch,
                                                              uint32_t* __restrict__ sizes) {
  extern __shared__ uint8_t sm[];
  uint8_t* in_s = sm;              // [chunk]
  uint8_t* planes = sm + chunk;    // [chunk]
  __shared__ int warp_sums[32];
  const int c = blockIdx.x;
  const int64_t base = int64_t(c) * chunk;
  const int clen = int(total - base < int64_t(chunk) ? total - base : int64_t(chunk));
  const int n = pad16(clen);
  uint8_t* slot = scratch + int64_t(c) * slot_bytes(chunk);
  for (int i = threadIdx.x; i < n; i += blockDim.x) in_s[i] = i < clen ? src[base + i] : 0;
  __syncthreads();
  const int n8 = n / 8;
  // tuple + bit shuffle: thread q builds plane byte q of all 8 planes
  for (int q = threadIdx.x; q < n8; q += blockDim.x) {
    uint64_t x = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int p = 8 * q + k;          // position in the tuple-shuffled array
      const int j = p / n8, i = p % n8;  // tup[j*n8 + i] = in[8i + j]
      x |= uint64_t(in_s[8 * i + j]) << (8 * k);
    }
    const uint64_t t = transpose8(x);
#pragma unroll
    for (int b = 0; b < 8; ++b) planes[b * n8 + q] = uint8_t(t >> (8 * b));
  }
  __syncthreads();
  // zero-word elimination over n/2 16-bit words; each thread owns 16 words
  const int words = n / 2;
  const uint16_t* w16 = reinterpret_cast<const uint16_t*>(planes);
  const int per = 16;
  const int w0 = threadIdx.x * per;
  int cnt = 0;
  uint32_t mask = 0;
  for (int k = 0; k < per; ++k) {
    const int w = w0 + k;
    if (w < words && w16[w] != 0) {
      mask |= 1u << k;
      ++cnt;
    }
  }
  int nnz = 0;
  // blockDim.x * per must cover the chunk: 512 * 16 = 8192 words = 16 KB
  const int before = block_exclusive_scan(cnt, warp_sums, nnz);
  const int bm_bytes = (words + 7) / 8;
  const int coded = bm_bytes + 2 * nnz;
  const bool raw = coded >= clen;
  if (!raw) {
    if (w0 < words) {
      slot[w0 / 8] = uint8_t(mask & 0xffu);
      if (w0 / 8 + 1 < bm_bytes) slot[w0 / 8 + 1] = uint8_t(mask >> 8);
    }
    int pos = before;
    for (int k = 0; k < per; ++k) {
      if (mask & (1u << k)) {
        const uint16_t v = w16[w0 + k];
        slot[bm_bytes + 2 * pos] = uint8_t(v);
        slot[bm_bytes + 2 * pos + 1] = uint8_t(v >> 8);
        ++pos;
      }
    }
  } else {
    for (int i = threadIdx.x; i < clen; i += blockDim.x) slot[i] = in_s[i];
  }
  if (threadIdx.x == 0) sizes[c] = raw ? (uint32_t(clen) | kRawFlag) : uint32_t(coded);
}

__device__ __forceinline__ int64_t payload_len(uint32_t s) { return int64_t(s & ~kRawFlag); }

// Single CTA: offsets[c] = header + 4*chunks + sum of 4-aligned lengths; also
// writes the header + size table into `out` (if non-null) and the total size.
__global__ void __launch_bounds__(1024) rze_scan(const uint32_t* __restrict__ sizes, int nchunks, int64_t total,
                                                 int chunk, int64_t* __restrict__ offsets, uint8_t* __restrict__ out,
                                                 int64_t* __restrict__ out_total) {
  __shared__ int64_t carry;
  __shared__ int warp_sums[32];
  if (threadIdx.x == 0) carry = kHeader + 4 * int64_t(nchunks);
  __syncthreads();
  for (int b = 0; b < nchunks; b += blockDim.x) {
    const int c = b + threadIdx.x;
    const int len = c < nchunks ? int((payload_len(sizes[c]) + 3) / 4 * 4) : 0;
    int tot = 0;
    // chunk lengths <= 16 KB and <= 1024 chunks per pass keep this within int
    const int ex = block_exclusive_scan(len, warp_sums, tot);
    if (c < nchunks) offsets[c] = carry + ex;
    __syncthreads();
    if (threadIdx.x == 0) carry += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (out_total) *out_total = carry;
    if (out) {
      uint32_t* h = reinterpret_cast<uint32_t*>(out);
      h[0] = 0x5A4C564Bu;  // "KVLZ"
      h[1] = 1u;
      h[2] = uint32_t(uint64_t(total));
      h[3] = uint32_t(uint64_t(total) >> 32);
      h[4] = uint32_t(chunk);
      h[5] = uint32_t(nchunks);
    }
  }
  if (out)
    for (int c = threadIdx.x; c < nchunks; c += blockDim.x)
      reinterpret_cast<uint32_t*>(out + kHeader)[c] = sizes[c];
}

__global__ void __launch_bounds__(256) rze_compact(const uint8_t* __restrict__ scratch, int chunk,
                                                   const uint32_t* __restrict__ sizes,
                                                   const int64_t* __restrict__ offsets, uint8_t* __restrict__ out) {
  const int c = blockIdx.x;
  const uint8_t* slot = scratch + int64_t(c) * slot_bytes(chunk);
  const int64_t len = payload_len(sizes[c]);
  uint8_t* dst = out + offsets[c];
  const int64_t padded = (len + 3) / 4 * 4;
  for (int64_t i = threadIdx.x; i < padded; i += blockDim.x) dst[i] = i < len ? slot[i] : 0;
}

__global__ void __launch_bounds__(kThreads) rze_decode_chunks(const uint8_t* __restrict__ src, int64_t total,
                                                              int chunk, const uint32_t* __restrict__ sizes,
                                                              const int64_t* __restrict__ offsets,
                                                              uint8_t* __restrict__ dst) {
  extern __shared__ uint8_t sm[];
  uint8_t* planes = sm;           // [chunk]
  uint8_t* out_s = sm + chunk;    // [chunk]
  __shared__ int warp_sums[32];
  const int c = blockIdx.x;
  const int64_t base = int64_t(c) * chunk;
  const int clen = int(total - base < int64_t(chunk) ? total - base : int64_t(chunk));
  const int n = pad16(clen);
  const uint8_t* in = src + offsets[c];
  const uint32_t sz = sizes[c];
  if (sz & kRawFlag) {
    for (int i = threadIdx.x; i < clen; i += blockDim.x) dst[base + i] = in[i];
    return;
  }
  const int words = n / 2;
  const int bm_bytes = (words + 7) / 8;
  const int per = 16;
  const int w0 = threadIdx.x * per;
  uint32_t mask = 0;
  if (w0 < words) {
    mask = in[w0 / 8];
    if (w0 / 8 + 1 < bm_bytes) mask |= uint32_t(in[w0 / 8 + 1]) << 8;
    const int valid = min(per, words - w0);
    if (valid < 32) mask &= (1u << valid) - 1u;
  }
  int nnz = 0;
  const int before = block_exclusive_scan(__popc(mask), warp_sums, nnz);
  uint16_t* w16 = reinterpret_cast<uint16_t*>(planes);
  int pos = before;
  for (int k = 0; k < per; ++k) {
    const int w = w0 + k;
    if (w >= words) break;
    if (mask & (1u << k)) {
      w16[w] = uint16_t(in[bm_bytes + 2 * pos]) | uint16_t(uint16_t(in[bm_bytes + 2 * pos + 1]) << 8);
      ++pos;
    } else {
      w16[w] = 0;
    }
  }
  __syncthreads();
  const int n8 = n / 8;
  for (int q = threadIdx.x; q < n8; q += blockDim.x) {
    uint64_t x = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) x |= uint64_t(planes[b * n8 + q]) << (8 * b);
    const uint64_t t = transpose8(x);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int p = 8 * q + k;
      const int j = p / n8, i = p % n8;
      out_s[8 * i + j] = uint8_t(t >> (8 * k));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < clen; i += blockDim.x) dst[base + i] = out_s[i];
}

}  // namespace

int64_t rze_max_encoded_bytes(int64_t n, int64_t chunk) {
  const int64_t nchunks = (n + chunk - 1) / chunk;
  return kHeader + 4 * nchunks + nchunks * (slot_bytes(int(chunk)) + 4);
}

int64_t rze_scratch_bytes(int64_t n, int64_t chunk) {
  const int64_t nchunks = (n + chunk - 1) / chunk;
  return nchunks * (slot_bytes(int(chunk)) + 4 + 8) + 16;
}

// Encodes `src` (uint8, contiguous) into `out` (capacity >= rze_max_encoded_bytes)
// using `scratch` (>= rze_scratch_bytes) and writes the encoded size to out_total[0].
void rze_encode(torch::Tensor src, torch::Tensor out, torch::Tensor scratch, torch::Tensor out_total,
                int64_t chunk) {
  KVS_CHECK_ARG(src.is_cuda() && src.is_contiguous() && src.scalar_type() == at::kByte, "rze: uint8 CUDA source");
  KVS_CHECK_ARG(chunk == kChunk, "rze: chunk must be 16384 bytes");
  const int64_t n = src.numel();
  const int64_t nchunks = (n + chunk - 1) / chunk;
  KVS_CHECK_ARG(out.numel() >= rze_max_encoded_bytes(n, chunk) && scratch.numel() >= rze_scratch_bytes(n, chunk),
                "rze: output or scratch too small");
  KVS_CHECK_ARG(out_total.scalar_type() == at::kLong, "rze: out_total int64");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  uint8_t* scr = scratch.data_ptr<uint8_t>();
  uint8_t* slots = scr;
  uint32_t* sizes = reinterpret_cast<uint32_t*>(scr + nchunks * slot_bytes(int(chunk)));
  int64_t* offsets = reinterpret_cast<int64_t*>(
      (reinterpret_cast<uintptr_t>(sizes + nchunks) + 15) & ~uintptr_t(15));
  static bool attr = false;
  if (!attr) {
    KVS_CUDA_CHECK(cudaFuncSetAttribute(rze_encode_chunks, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kChunk));
    KVS_CUDA_CHECK(cudaFuncSetAttribute(rze_decode_chunks, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kChunk));
    attr = true;
  }
  if (nchunks > 0)
    rze_encode_chunks<<<int(nchunks), kThreads, 2 * kChunk, st>>>(src.data_ptr<uint8_t>(), n, int(chunk), slots,
                                                                  sizes);
  rze_scan<<<1, 1024, 0, st>>>(sizes, int(nchunks), n, int(chunk), offsets, out.data_ptr<uint8_t>(),
                               out_total.data_ptr<int64_t>());
  if (nchunks > 0)
    rze_compact<<<int(nchunks), 256, 0, st>>>(slots, int(chunk), sizes, offsets, out.data_ptr<uint8_t>());
  KVS_CUDA_CHECK(cudaGetLastError());
}

void rze_decode(torch::Tensor src, torch::Tensor out, torch::Tensor scratch, int64_t chunk) {
  KVS_CHECK_ARG(src.is_cuda() && src.scalar_type() == at::kByte && out.is_cuda() && out.is_contiguous(),
                "rze: CUDA tensors");
  KVS_CHECK_ARG(chunk == kChunk, "rze: chunk must be 16384 bytes");
  const int64_t n = out.numel() * out.element_size();
  const int64_t nchunks = (n + chunk - 1) / chunk;
  KVS_CHECK_ARG(src.numel() >= kHeader + 4 * nchunks, "rze: payload shorter than its size table");
  KVS_CHECK_ARG(scratch.numel() >= 8 * nchunks + 16, "rze: scratch too small");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const uint32_t* sizes = reinterpret_cast<const uint32_t*>(src.data_ptr<uint8_t>() + kHeader);
  int64_t* offsets = reinterpret_cast<int64_t*>(
      (reinterpret_cast<uintptr_t>(scratch.data_ptr<uint8_t>()) + 15) & ~uintptr_t(15));
  static bool attr = false;
  if (!attr) {
    KVS_CUDA_CHECK(cudaFuncSetAttribute(rze_decode_chunks, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * kChunk));
    attr = true;
  }
  rze_scan<<<1, 1024, 0, st>>>(sizes, int(nchunks), n, int(chunk), offsets, nullptr, nullptr);
  if (nchunks > 0)
    rze_decode_chunks<<<int(nchunks), kThreads, 2 * kChunk, st>>>(src.data_ptr<uint8_t>(), n, int(chunk), sizes,
                                                                  offsets, reinterpret_cast<uint8_t*>(out.data_ptr()));
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
