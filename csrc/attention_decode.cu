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
#include "attention_decode_kernels.cuh"
#include "attention_decode_tma.cuh"

namespace kvs {

int64_t paged_decode_splits(int64_t batch, int64_t hkv, int64_t max_ctx) {
  const int64_t want = std::max<int64_t>(1, (3 * kNumSMs) / std::max<int64_t>(1, batch * hkv));
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
  // TMA-fed kernel: head_dim 128, 16-token blocks stored contiguously, 1, 2,
  // 4 or 8 query heads per KV head.
  const bool tma_ok = D == 128 && bsz == kTmaBlk && k_cache.stride(2) == D && k_cache.stride(1) == Hkv * D &&
                      k_cache.stride(0) == int64_t(bsz) * Hkv * D && v_cache.strides() == k_cache.strides() &&
                      (G == 1 || G == 2 || G == 4 || G == 8) &&
                      (reinterpret_cast<uintptr_t>(k_cache.data_ptr()) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(v_cache.data_ptr()) & 15) == 0;
  // 8 query heads per KV head: two CTAs of 4 query heads per KV head (the
  // TMA kernel keeps 4 heads' queries and accumulators in registers)
  const int kv_shift = (tma_ok && G == 8) ? 1 : 0;
  const int Gl = G >> kv_shift, Hl = Hkv << kv_shift;
  // it holds two CTAs per SM: one wave of 2 x 148 CTAs
  if (tma_ok) splits = std::max<int64_t>(1, std::min<int64_t>(splits, (2 * kNumSMs) / std::max(1, B * Hl)));
  const int chunk = int(std::max<int64_t>(16, ((max_ctx + splits - 1) / splits + 15) / 16 * 16));
  splits = (max_ctx + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  if (splits > 1)
    KVS_CHECK_ARG(part_o.numel() >= int64_t(B) * Hq * splits * D && part_ml.numel() >= int64_t(B) * Hq * splits * 2,
                  "paged decode: split scratch too small");
  dim3 grid(int(splits), tma_ok ? Hl : Hkv, B);
  const float sl2 = float(scale) * 1.4426950408889634f;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  float* po0 = splits > 1 ? part_o.data_ptr<float>() : nullptr;
  float* pml0 = splits > 1 ? part_ml.data_ptr<float>() : nullptr;
  if (tma_ok) {
    const uint64_t rows = uint64_t(k_cache.size(0)) * bsz;
    const CUtensorMap tk = make_tmap_2d_bf16(k_cache.data_ptr(), uint64_t(Hkv) * D, rows, uint64_t(Hkv) * D * 2,
                                             128, kTmaBlk, false);
    const CUtensorMap tv = make_tmap_2d_bf16(v_cache.data_ptr(), uint64_t(Hkv) * D, rows, uint64_t(Hkv) * D * 2,
                                             128, kTmaBlk, false);
    auto qp = reinterpret_cast<const bf16*>(q.data_ptr());
    auto op = reinterpret_cast<bf16*>(out.data_ptr());
    const int32_t* btp = block_tables.data_ptr<int32_t>();
    const int32_t* clp = ctx_lens.data_ptr<int32_t>();
#define KVS_TMA_CASE(GG)                                                                                       \
  case GG: {                                                                                                   \
    static bool set = false;                                                                                   \
    if (!set) {                                                                                                \
      KVS_CUDA_CHECK(cudaFuncSetAttribute(paged_decode_tma_kernel<GG>,                                         \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kTmaSmem));             \
      set = true;                                                                                              \
    }                                                                                                          \
    paged_decode_tma_kernel<GG><<<grid, kTmaThreads, kTmaSmem, st>>>(tk, tv, qp, q.stride(0), btp,             \
                                                                     block_tables.stride(0), clp, Hq,          \
                                                                     int(splits), chunk, sl2, po0, pml0, op,   \
                                                                     out.stride(0), nullptr, kv_shift);        \
    break;                                                                                                     \
  }
    switch (Gl) {
      KVS_TMA_CASE(1)
      KVS_TMA_CASE(2)
      KVS_TMA_CASE(4)
    }
#undef KVS_TMA_CASE
    if (splits > 1) {
      dim3 g2(Hq, B);
      merge_splits_kernel<128><<<g2, 128, 0, st>>>(po0, pml0, Hq, int(splits), op, out.stride(0));
    }
    KVS_CUDA_CHECK(cudaGetLastError());
    return;
  }
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
