// Kernels of the split-K paged decode attention, shared by the regular
// entry point (attention_decode.cu) and the allocation-free C entry point
// (paged_decode_noalloc.cu).  See attention_decode.cu for the design.
#pragma once
#include "common.cuh"

namespace kvs {
namespace {

constexpr int kThreads = 128;

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One CTA = one (split, kv head, sequence).  A token row of K or V (D bf16)
// is spread over D/8 lanes (16 bytes each); every row group handles U
// consecutive tokens per step and issues all 2U of its 16-byte loads before
// using any of them (16 KB per CTA in flight, 3 CTAs per SM).  The U scores of a
// step share one online-softmax update per query head.
template <int D, int G>
__global__ void __launch_bounds__(kThreads) paged_decode_kernel(
    const bf16* __restrict__ q, int64_t q_tok_stride, const bf16* __restrict__ kc, const bf16* __restrict__ vc,
    int64_t blk_stride, int64_t tok_stride, int64_t head_stride, const int32_t* __restrict__ block_tables,
    int64_t bt_stride, const int32_t* __restrict__ ctx_lens, int block_size, int Hq, int splits, int chunk,
    float scale_log2, float* __restrict__ part_o, float* __restrict__ part_ml, bf16* __restrict__ out,
    int64_t out_tok_stride) {
  pdl_trigger();
  constexpr int LANES = D / 8;          // lanes per token row
  constexpr int TPW = 32 / LANES;       // row groups per warp
  constexpr int kGroups = (kThreads / 32) * TPW;
  constexpr int U = G >= 8 ? 2 : (G >= 4 ? 4 : 8);  // tokens per row group per step
  constexpr int STEP = kGroups * U;
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
  const int64_t head_off = int64_t(kvh) * head_stride + lir * 8;
  for (int t0 = t_begin; t0 < t_end; t0 += STEP) {
    const int tg = t0 + grp * U;
    uint4 kr[U], vr[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = tg + u;
      if (t < t_end) {
        const int64_t off = int64_t(bt[t / block_size]) * blk_stride + int64_t(t % block_size) * tok_stride +
                            head_off;
        kr[u] = ld_stream16(kc + off);
        vr[u] = ld_stream16(vc + off);
      } else {
        kr[u] = make_uint4(0, 0, 0, 0);
        vr[u] = make_uint4(0, 0, 0, 0);
      }
    }
    float s[U][G];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[8];
      const __nv_bfloat162* kh = reinterpret_cast<const __nv_bfloat162*>(&kr[u]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __bfloat1622float2(kh[e]);
        kf[2 * e] = a.x;
        kf[2 * e + 1] = a.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(qf[g][e], kf[e], acc);
        s[u][g] = acc;
      }
    }
#pragma unroll
    for (int mm = 1; mm < LANES; mm <<= 1)
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffffu, s[u][g], mm);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = m[g];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (tg + u < t_end) mx = fmaxf(mx, s[u][g]);
      // no valid token seen yet (mx = -inf): nothing to rescale
      const float alpha = (mx == -INFINITY) ? 1.0f : fast_ex2(m[g] - mx);
      l[g] *= alpha;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[g][e] *= alpha;
      m[g] = mx;
#pragma unroll
      for (int u = 0; u < U; ++u) s[u][g] = (tg + u < t_end) ? fast_ex2(s[u][g] - mx) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vr[u]);
      float vf[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 c = __bfloat1622float2(vh[e]);
        vf[2 * e] = c.x;
        vf[2 * e + 1] = c.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        l[g] += s[u][g];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[g][e] = fmaf(s[u][g], vf[e], o[g][e]);
      }
    }
  }
  // Merge the per-row-group states of the CTA.
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
        const float w = fast_ex2(s_m[k][g] - mx);
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
  pdl_trigger();
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
    KVS_DEC_CASE(3)
    KVS_DEC_CASE(4)
    KVS_DEC_CASE(5)
    KVS_DEC_CASE(6)
    KVS_DEC_CASE(7)   // Qwen2.5-7B: 28 query heads over 4 KV heads
    KVS_DEC_CASE(8)
    default: throw std::invalid_argument("paged decode: query heads per KV head must be 1..8");
  }
#undef KVS_DEC_CASE
}

}  // namespace
}  // namespace kvs
