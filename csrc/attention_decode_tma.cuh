// TMA-fed paged decode attention for head_dim 128 and 16-token paged blocks
// stored contiguously ([num_blocks, 16, Hkv, 128]).
//
// One CTA = one (split, kv head, sequence), 160 threads (with kv_shift = 1
// a "kv head" index covers half of a real KV head's G query heads: 8 query
// heads per KV head run as two CTAs of 4, each streaming the KV once):
//   warp 4      producer: one 2-D TMA load per paged block for K and one for V
//               (16 rows x 256 bytes each) into an 8-stage shared-memory ring;
//   warps 0..3  consumers: thread (t, q) = token slot t (0..15) of every block
//               and 16-dim slice q (0..7); scores are reduced over the 8 slice
//               threads with three xor shuffles.
// Every token slot keeps its own online-softmax state with lazy rescaling
// (the reference max only moves when a score exceeds it by 2^8); the 16 slot
// states are merged through shared memory at the end and written either to
// the output (one split) or to the split's partial record, exactly like the
// generic kernel, so the same merge kernel follows.
#pragma once
#include "common.cuh"
#include "sm100.cuh"

namespace kvs {
namespace {

constexpr int kTmaStages = 8;
constexpr int kTmaThreads = 160;
constexpr int kTmaBlk = 16;                       // tokens per paged block
constexpr int kTmaTile = kTmaBlk * 128 * 2;       // bytes of one K (or V) block tile
constexpr int kTmaSmem = kTmaStages * 2 * kTmaTile + 256;

template <int G>
__global__ void __launch_bounds__(kTmaThreads) paged_decode_tma_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const bf16* __restrict__ q,
    int64_t q_tok_stride, const int32_t* __restrict__ block_tables, int64_t bt_stride,
    const int32_t* __restrict__ ctx_lens, int Hq, int splits, int chunk, float scale_log2,
    float* __restrict__ part_o, float* __restrict__ part_ml, bf16* __restrict__ out, int64_t out_tok_stride,
    uint32_t* err, int kv_shift) {
  pdl_trigger();
  using namespace sm100;
  constexpr int D = 128;
  extern __shared__ __align__(128) uint8_t dsm[];
  uint8_t* sK = dsm;
  uint8_t* sV = dsm + kTmaStages * kTmaTile;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + 2 * kTmaStages * kTmaTile);
  uint64_t* empty = full + kTmaStages;
  __shared__ float s_m[kTmaBlk][G], s_l[kTmaBlk][G];

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int ctx = ctx_lens[b];
  const int t_begin = split * chunk;
  const int t_end = min(ctx, t_begin + chunk);
  const int blk_begin = t_begin / kTmaBlk;
  const int nblk = t_end > t_begin ? (t_end - 1) / kTmaBlk - blk_begin + 1 : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t* bt = block_tables + int64_t(b) * bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmaStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 4) {
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int issued = 0;
      for (int i = 0; i < nblk; ++i) {
        const int s = i % kTmaStages;
        const uint32_t ph = (i / kTmaStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, err)) break;
        const int row = bt[blk_begin + i] * kTmaBlk;
        mbar_arrive_expect_tx(&full[s], 2 * kTmaTile);
        tma_load_2d(sK + s * kTmaTile, &tmK, (kvh >> kv_shift) * D, row, &full[s]);
        tma_load_2d(sV + s * kTmaTile, &tmV, (kvh >> kv_shift) * D, row, &full[s]);
        issued = i + 1;
      }
      // every issued copy lands before the CTA may exit
      for (int i = max(0, issued - kTmaStages); i < issued; ++i)
        mbar_wait(&full[i % kTmaStages], (i / kTmaStages) & 1, nullptr);
    }
    return;
  }

  const int t = threadIdx.x >> 3, qd = threadIdx.x & 7;
  float qf[G][16];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const bf16* qp = q + int64_t(b) * q_tok_stride + int64_t(kvh * G + g) * D + qd * 16;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qp + 8 * h);
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(hh[e]);
        qf[g][8 * h + 2 * e] = f.x * scale_log2;
        qf[g][8 * h + 2 * e + 1] = f.y * scale_log2;
      }
    }
  }
  float m[G], l[G], o[G][16];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) o[g][e] = 0.f;
  }
  bool ok = true;
  for (int i = 0; i < nblk; ++i) {
    const int s = i % kTmaStages;
    if (!mbar_wait(&full[s], (i / kTmaStages) & 1, err)) ok = false;
    if (!__all_sync(0xffffffffu, ok)) break;
    const bf16* kr = reinterpret_cast<const bf16*>(sK + s * kTmaTile) + t * D + qd * 16;
    const bf16* vr = reinterpret_cast<const bf16*>(sV + s * kTmaTile) + t * D + qd * 16;
    float kf[16], vf[16];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 kk = *reinterpret_cast<const uint4*>(kr + 8 * h);
      const uint4 vv = *reinterpret_cast<const uint4*>(vr + 8 * h);
      const __nv_bfloat162* kh = reinterpret_cast<const __nv_bfloat162*>(&kk);
      const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&vv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __bfloat1622float2(kh[e]), c = __bfloat1622float2(vh[e]);
        kf[8 * h + 2 * e] = a.x;
        kf[8 * h + 2 * e + 1] = a.y;
        vf[8 * h + 2 * e] = c.x;
        vf[8 * h + 2 * e + 1] = c.y;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);  // the stage's data are in registers
    const bool valid = (blk_begin + i) * kTmaBlk + t < t_end && (blk_begin + i) * kTmaBlk + t >= t_begin;
    float sc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) acc = fmaf(qf[g][e], kf[e], acc);
      sc[g] = acc;
    }
#pragma unroll
    for (int mm = 1; mm < 8; mm <<= 1)
#pragma unroll
      for (int g = 0; g < G; ++g) sc[g] += __shfl_xor_sync(0xffffffffu, sc[g], mm);
    if (valid) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        if (sc[g] > m[g] + 8.0f) {  // lazy rescale: the reference max moves rarely
          const float alpha = (m[g] == -INFINITY) ? 0.f : fast_ex2(m[g] - sc[g]);
          l[g] *= alpha;
#pragma unroll
          for (int e = 0; e < 16; ++e) o[g][e] *= alpha;
          m[g] = sc[g];
        }
        const float p = fast_ex2(sc[g] - m[g]);
        l[g] += p;
#pragma unroll
        for (int e = 0; e < 16; ++e) o[g][e] = fmaf(p, vf[e], o[g][e]);
      }
    }
  }
  // ---- merge the 16 token-slot states (stage memory is free now) ----
  asm volatile("bar.sync 1, 128;" ::: "memory");  // consumers only
  float* s_o = reinterpret_cast<float*>(dsm);      // [16][G][128]
  if (qd == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s_m[t][g] = m[g];
      s_l[t][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < 16; ++e) s_o[(t * G + g) * D + qd * 16 + e] = o[g][e];
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (int idx = threadIdx.x; idx < G * D; idx += 128) {
    const int g = idx / D, d = idx % D;
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kTmaBlk; ++k) mx = fmaxf(mx, s_m[k][g]);
    float lsum = 0.f, acc = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int k = 0; k < kTmaBlk; ++k) {
        const float w = s_m[k][g] == -INFINITY ? 0.f : fast_ex2(s_m[k][g] - mx);
        lsum += s_l[k][g] * w;
        acc += s_o[(k * G + g) * D + d] * w;
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

}  // namespace
}  // namespace kvs
