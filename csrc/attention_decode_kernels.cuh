// Kernels of the split-K paged decode attention, shared by the regular
// entry point (attention_decode.cu) and the allocation-free C entry point
// (paged_decode_noalloc.cu).  See attention_decode.cu for the design.
#pragma once
#include "common.cuh"

namespace kvs {
namespace {

constexpr int kThreads = 128;
constexpr int kMaxGroup = 8;  // query heads per KV head

template <int D, int G>
__global__ void __launch_bounds__(kThreads) paged_decode_kernel(
    const bf16* __restrict__ q, int64_t q_tok_stride, const bf16* __restrict__ kc, const bf16* __restrict__ vc,
    int64_t blk_stride, int64_t tok_stride, int64_t head_stride, const int32_t* __restrict__ block_tables,
    int64_t bt_stride, const int32_t* __restrict__ ctx_lens, int block_size, int Hq, int splits, int chunk,
    float scale_log2, float* __restrict__ part_o, float* __restrict__ part_ml, bf16* __restrict__ out,
    int64_t out_tok_stride) {
  constexpr int LANES = D / 8;          // lanes per token row
  constexpr int TPW = 32 / LANES;       // tokens per warp step
  constexpr int kGroups = (kThreads / 32) * TPW;
  __shared__ float s_m[kGroups][G], s_l[kGroups][G];
  __shared__ float s_o[kGroups][G][D];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int ctx = ctx_lens[b];
  const int t_begin = split * chunk;
  const int t_end = min(ctx, t_begin + chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lir = lane % LANES, sub = lane / LANES;
  const int grp = warp * TPW + sub;
  float qf[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const bf16* qp = q + int64_t(b) * q_tok_stride + int64_t(kvh * G + g) * D + lir * 8;
    const uint4 raw = *reinterpret_cast<const uint4*>(qp);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      qf[g][2 * e] = f.x * scale_log2;
      qf[g][2 * e + 1] = f.y * scale_log2;
    }
  }
  float m[G], l[G], o[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[g][e] = 0.f;
  }
  const int32_t* bt = block_tables + int64_t(b) * bt_stride;
  for (int t0 = t_begin; t0 < t_end; t0 += (kThreads / 32) * TPW) {
    const int t = t0 + warp * TPW + sub;
    const bool valid = t < t_end;
    float kf[8], vf[8];
    if (valid) {
      const int blk = bt[t / block_size];
      const int64_t off = int64_t(blk) * blk_stride + int64_t(t % block_size) * tok_stride +
                          int64_t(kvh) * head_stride + lir * 8;
      const uint4 kr = *reinterpret_cast<const uint4*>(kc + off);
      const uint4 vr = *reinterpret_cast<const uint4*>(vc + off);
      const __nv_bfloat162* kh = reinterpret_cast<const __nv_bfloat162*>(&kr);
      const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vr);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __bfloat1622float2(kh[e]);
        const float2 c = __bfloat1622float2(vh[e]);
        kf[2 * e] = a.x;
        kf[2 * e + 1] = a.y;
        vf[2 * e] = c.x;
        vf[2 * e + 1] = c.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) kf[e] = vf[e] = 0.f;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(qf[g][e], kf[e], s);
#pragma unroll
      for (int mm = 1; mm < LANES; mm <<= 1) s += __shfl_xor_sync(0xffffffffu, s, mm);
      if (valid) {
        const float mn = fmaxf(m[g], s);
        const float alpha = exp2f(m[g] - mn);
        const float p = exp2f(s - mn);
        l[g] = l[g] * alpha + p;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[g][e] = o[g][e] * alpha + p * vf[e];
        m[g] = mn;
      }
    }
  }
  // Merge the per-half-warp states of the CTA.
  if (lir == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[grp][g] = m[g];
      s_l[grp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) s_o[grp][g][lir * 8 + e] = o[g][e];
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    float mx = -INFINITY;
    for (int k = 0; k < kGroups; ++k) mx = fmaxf(mx, s_m[k][g]);
    float lsum = 0.f, acc = 0.f;
    if (mx != -INFINITY) {
      for (int k = 0; k < kGroups; ++k) {
        const float w = exp2f(s_m[k][g] - mx);
        lsum += s_l[k][g] * w;
        acc += s_o[k][g][d] * w;
      }
    }
    const int h = kvh * G + g;
    if (splits == 1) {
      out[int64_t(b) * out_tok_stride + int64_t(h) * D + d] = rn(lsum > 0.f ? acc / lsum : 0.f);
    } else {
      const int64_t rec = (int64_t(b) * Hq + h) * splits + split;
      part_o[rec * D + d] = acc;
      if (d == 0) {
        part_ml[rec * 2] = mx;
        part_ml[rec * 2 + 1] = lsum;
      }
    }
  }
}

template <int D>
__global__ void merge_splits_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                    int Hq, int splits, bf16* __restrict__ out, int64_t out_tok_stride) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t rec0 = (int64_t(b) * Hq + h) * splits;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, part_ml[(rec0 + s) * 2]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float lsum = 0.f, acc = 0.f;
    if (mx != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const float w = exp2f(part_ml[(rec0 + s) * 2] - mx);
        lsum += part_ml[(rec0 + s) * 2 + 1] * w;
        acc += part_o[(rec0 + s) * D + d] * w;
      }
    }
    out[int64_t(b) * out_tok_stride + int64_t(h) * D + d] = rn(lsum > 0.f ? acc / lsum : 0.f);
  }
}

template <int D>
void launch_decode(int G, dim3 grid, cudaStream_t st, const bf16* q, int64_t qs, const bf16* kc, const bf16* vc,
                   int64_t bs_, int64_t ts, int64_t hs, const int32_t* bt, int64_t bts, const int32_t* ctx,
                   int block_size, int Hq, int splits, int chunk, float sl2, float* po, float* pml, bf16* out,
                   int64_t os) {
#define KVS_DEC_CASE(GG)                                                                                     \
  case GG:                                                                                                   \
    paged_decode_kernel<D, GG><<<grid, kThreads, 0, st>>>(q, qs, kc, vc, bs_, ts, hs, bt, bts, ctx,         \
                                                          block_size, Hq, splits, chunk, sl2, po, pml, out, os); \
    break;
  switch (G) {
    KVS_DEC_CASE(1)
    KVS_DEC_CASE(2)
    KVS_DEC_CASE(4)
    KVS_DEC_CASE(8)
    default: throw std::invalid_argument("paged decode: query heads per KV head must be 1, 2, 4 or 8");
  }
#undef KVS_DEC_CASE
}

}  // namespace
}  // namespace kvs
