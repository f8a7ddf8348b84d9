// Weight-streaming core shared by the decode-step GEMV kernels
// (y[M, N] = x[M, K] * W[N, K]^T, M <= 8): each warp owns kGemvRows output
// rows and keeps kGemvRows x U independent 16-byte weight loads in flight;
// x is staged in shared memory (bf16, 16-byte loads).  The kernels that use
// it differ only in their epilogue (plain store, tensor-parallel all-reduce,
// greedy argmax).
#pragma once

#include "common.cuh"

namespace kvs {

constexpr int kGemvThreads = 256;
constexpr int kGemvRows = 2;                                         // output rows per warp
constexpr int kGemvRowsPerCta = (kGemvThreads / 32) * kGemvRows;     // 16

__device__ __forceinline__ void gemv_load_x8(const bf16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(h[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ void gemv_unpack8(const uint4& w, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(h[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ float gemv_dot8(const uint4& w, const float (&x)[8], float acc) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = __bfloat1622float2(h[e]);
    acc = fmaf(t.x, x[2 * e], acc);
    acc = fmaf(t.y, x[2 * e + 1], acc);
  }
  return acc;
}

// Computes the warp's kGemvRows rows starting at row0 (row0 < N) for all M
// tokens; on return every lane holds the full dot products in acc.  xs is the
// [M][K] shared-memory copy of x, staged by the caller between the first
// weight loads (issued here through `prefetch`) and this call.
template <int M>
struct GemvWarp {
  static constexpr int U = M <= 2 ? 8 : 4;  // 16-byte loads in flight per row per lane
  uint4 wv[kGemvRows][U];
  bool have = false;

  // First batch of weight loads, issued before x is staged so the weight
  // stream starts at kernel entry instead of after the barrier.
  __device__ __forceinline__ void prefetch(const bf16* __restrict__ w, int64_t ldw, int row0, int N, int K,
                                           int lane) {
    const int kvec = K / 8;
    have = row0 < N && lane + 32 * (U - 1) < kvec;
    if (have) {
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
        for (int u = 0; u < U; ++u)
          wv[r][u] = __ldcs(reinterpret_cast<const uint4*>(w + int64_t(min(row0 + r, N - 1)) * ldw) + lane + 32 * u);
    }
  }

  __device__ __forceinline__ void run(const bf16* __restrict__ w, int64_t ldw, const bf16* xs, int row0, int N,
                                      int K, int lane, float (&acc)[kGemvRows][M]) {
    const int kvec = K / 8;
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
    int kv = lane;
    for (bool h = have; kv + 32 * (U - 1) < kvec; kv += 32 * U, h = false) {
      if (!h) {
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int row = min(row0 + r, N - 1);
            wv[r][u] = __ldcs(reinterpret_cast<const uint4*>(w + int64_t(row) * ldw) + kv + 32 * u);
          }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = (kv + 32 * u) * 8;
        // each weight vector is converted once and reused for every token
        float wf[kGemvRows][8];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) gemv_unpack8(wv[r][u], wf[r]);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float xf[8];
          gemv_load_x8(xs + m * K + k, xf);
#pragma unroll
          for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[r][m] = fmaf(wf[r][e], xf[e], acc[r][m]);
        }
      }
    }
    for (; kv < kvec; kv += 32) {
      const int k = kv * 8;
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r) {
        const int row = min(row0 + r, N - 1);
        const uint4 wq = __ldcs(reinterpret_cast<const uint4*>(w + int64_t(row) * ldw) + kv);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float xf[8];
          gemv_load_x8(xs + m * K + k, xf);
          acc[r][m] = gemv_dot8(wq, xf, acc[r][m]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v = acc[r][m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        acc[r][m] = v;
      }
  }
};

// Stage x [M, K] (row stride ldx) into shared memory with 16-byte copies.
template <int M>
__device__ __forceinline__ void gemv_stage_x(const bf16* __restrict__ x, int64_t ldx, uint4* xs_raw, int K) {
  for (int i = threadIdx.x; i < M * K / 8; i += blockDim.x) {
    const int m = i / (K / 8), k8 = i % (K / 8);
    xs_raw[i] = *reinterpret_cast<const uint4*>(x + int64_t(m) * ldx + k8 * 8);
  }
}

}  // namespace kvs
