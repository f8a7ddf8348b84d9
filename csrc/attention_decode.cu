// Paged decode attention (one new query token per sequence, GQA) with a
// split-K ("flash-decoding") schedule: grid (splits, kv_heads, batch); each
// CTA streams a contiguous range of the sequence's paged K/V blocks for one
// KV head and all of its query heads, keeps an online softmax per half-warp,
// merges in shared memory and writes a partial (max, sum, acc) record; a
// second tiny kernel merges the splits.  Memory-bound by design: every K/V
// byte is read once with 16-byte loads.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "ops.h"

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

int64_t paged_decode_splits(int64_t batch, int64_t hkv, int64_t max_ctx) {
  const int64_t want = std::max<int64_t>(1, (2 * kNumSMs) / std::max<int64_t>(1, batch * hkv));
  const int64_t by_len = std::max<int64_t>(1, max_ctx / 128);
  return std::min<int64_t>(std::min<int64_t>(want, by_len), 64);
}

void paged_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache,
                            torch::Tensor block_tables, torch::Tensor ctx_lens, int64_t max_ctx, double scale,
                            torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml, int64_t splits) {
  KVS_CHECK_ARG(q.dim() == 3 && q.stride(2) == 1 && out.dim() == 3 && out.stride(2) == 1 &&
                    q.scalar_type() == at::kBFloat16,
                "paged decode: q/out [B, Hq, D] bf16");
  KVS_CHECK_ARG(k_cache.dim() == 4 && k_cache.stride(3) == 1 && v_cache.strides() == k_cache.strides(),
                "paged decode: caches [num_blocks, block_size, Hkv, D] with equal strides");
  const int B = int(q.size(0)), Hq = int(q.size(1)), D = int(q.size(2));
  const int Hkv = int(k_cache.size(2)), bsz = int(k_cache.size(1));
  KVS_CHECK_ARG(Hq % Hkv == 0 && q.stride(1) == D && out.stride(1) == D, "paged decode: head layout");
  KVS_CHECK_ARG(block_tables.scalar_type() == at::kInt && ctx_lens.scalar_type() == at::kInt, "int32 tables");
  if (B == 0) return;
  const int G = Hq / Hkv;
  const int chunk = int(std::max<int64_t>(16, ((max_ctx + splits - 1) / splits + 15) / 16 * 16));
  splits = (max_ctx + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  if (splits > 1)
    KVS_CHECK_ARG(part_o.numel() >= int64_t(B) * Hq * splits * D && part_ml.numel() >= int64_t(B) * Hq * splits * 2,
                  "paged decode: split scratch too small");
  dim3 grid(int(splits), Hkv, B);
  const float sl2 = float(scale) * 1.4426950408889634f;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto qp = reinterpret_cast<const bf16*>(q.data_ptr());
  auto kp = reinterpret_cast<const bf16*>(k_cache.data_ptr());
  auto vp = reinterpret_cast<const bf16*>(v_cache.data_ptr());
  auto op = reinterpret_cast<bf16*>(out.data_ptr());
  float* po = splits > 1 ? part_o.data_ptr<float>() : nullptr;
  float* pml = splits > 1 ? part_ml.data_ptr<float>() : nullptr;
  if (D == 128)
    launch_decode<128>(G, grid, st, qp, q.stride(0), kp, vp, k_cache.stride(0), k_cache.stride(1),
                       k_cache.stride(2), block_tables.data_ptr<int32_t>(), block_tables.stride(0),
                       ctx_lens.data_ptr<int32_t>(), bsz, Hq, int(splits), chunk, sl2, po, pml, op, out.stride(0));
  else if (D == 64)
    launch_decode<64>(G, grid, st, qp, q.stride(0), kp, vp, k_cache.stride(0), k_cache.stride(1),
                      k_cache.stride(2), block_tables.data_ptr<int32_t>(), block_tables.stride(0),
                      ctx_lens.data_ptr<int32_t>(), bsz, Hq, int(splits), chunk, sl2, po, pml, op, out.stride(0));
  else
    throw std::invalid_argument("paged decode: head_dim must be 64 or 128");
  if (splits > 1) {
    dim3 g2(Hq, B);
    if (D == 128)
      merge_splits_kernel<128><<<g2, 128, 0, st>>>(po, pml, Hq, int(splits), op, out.stride(0));
    else
      merge_splits_kernel<64><<<g2, 64, 0, st>>>(po, pml, Hq, int(splits), op, out.stride(0));
  }
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
