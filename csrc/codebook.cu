// Centred Gaussian codebook quantiser of the modular pipeline
// (behaviour of kvserve_v1/compression/quantizer/centered_codebook.py:
// keys per (head, channel) over groups of `group` tokens, values per
// (token, head) over the head dimension; mean, RMS scale times alpha rounded
// to bf16, optional least-squares scale refinements, symbol = index of the
// Lloyd-Max cell of (x - mean) / scale).
//
//   * cb_quant_keys:   one CTA per (token group, head), one thread per
//     channel; the group's [G, D] slice is read once from HBM and the later
//     passes (RMS, refinements, symbols) hit L1.
//   * cb_quant_values: one warp per (token, head); every statistic is a warp
//     reduction over the D values held in registers.
//   * cb_dequant:      elementwise centers[q] * scale + mean for both parts.
//
// Numerics follow the PyTorch formulation exactly where it matters for the
// symbols: fp32 statistics, IEEE division by the clamped scale, cell index =
// number of cell bounds strictly below the value (torch.bucketize, right=False),
// mean rounded to its storage dtype and scales to bf16 before use.  Invalid
// symbols on dequantisation set a status word instead of trapping.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "ops.h"

namespace kvs {
namespace {

constexpr int kCbMaxLevels = 16;

struct CbTable {
  float centers[kCbMaxLevels];
  float bounds[kCbMaxLevels - 1];
  int levels;
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<bf16>(bf16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }

__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ int cell_of(float v, const CbTable& tb) {
  int q = 0;
#pragma unroll
  for (int i = 0; i < kCbMaxLevels - 1; ++i)
    if (i < tb.levels - 1 && tb.bounds[i] < v) ++q;
  return q;
}

__device__ __forceinline__ float center_of(int q, const CbTable& tb) {
  float c = tb.centers[0];
#pragma unroll
  for (int i = 1; i < kCbMaxLevels; ++i)
    if (q == i) c = tb.centers[i];
  return c;
}

// ---------------------------------------------------------------- keys
template <typename T>
__global__ void __launch_bounds__(128) cb_quant_keys_kernel(const T* __restrict__ x, int64_t total, int heads,
                                                            int dim, int group, int refinements, float alpha,
                                                            int mean_bf16, CbTable tb, uint8_t* __restrict__ q,
                                                            void* mean_out, bf16* __restrict__ scale_out) {
  const int g = blockIdx.x, h = blockIdx.y;
  const int ng = gridDim.x;
  const int64_t t0 = int64_t(g) * group;
  const int cnt = int(total - t0 < int64_t(group) ? total - t0 : int64_t(group));
  const int64_t row = int64_t(heads) * dim;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    const T* col = x + t0 * row + int64_t(h) * dim + d;
    float s = 0.f;
    for (int t = 0; t < cnt; ++t) s += to_f(col[t * row]);
    float mean = s / float(cnt);
    mean = mean_bf16 ? round_bf16(mean) : mean;
    float ss = 0.f;
    for (int t = 0; t < cnt; ++t) {
      const float r = to_f(col[t * row]) - mean;
      ss = fmaf(r, r, ss);
    }
    float scale = round_bf16(sqrtf(ss / float(cnt)) * alpha);
    for (int it = 0; it < refinements; ++it) {
      const float den_s = fmaxf(scale, 1e-20f);
      float num = 0.f, den = 0.f;
      for (int t = 0; t < cnt; ++t) {
        const float r = to_f(col[t * row]) - mean;
        const float c = center_of(cell_of(r / den_s, tb), tb);
        num = fmaf(r, c, num);
        den = fmaf(c, c, den);
      }
      scale = round_bf16(fmaxf(num / fmaxf(den, 1e-20f), 0.f));
    }
    const float den_s = fmaxf(scale, 1e-20f);
    uint8_t* qc = q + t0 * row + int64_t(h) * dim + d;
    for (int t = 0; t < cnt; ++t) qc[t * row] = uint8_t(cell_of((to_f(col[t * row]) - mean) / den_s, tb));
    const int64_t pidx = (int64_t(h) * ng + g) * dim + d;  // [heads, ng, dim]
    if (mean_bf16)
      reinterpret_cast<bf16*>(mean_out)[pidx] = __float2bfloat16_rn(mean);
    else
      reinterpret_cast<float*>(mean_out)[pidx] = mean;
    scale_out[pidx] = __float2bfloat16_rn(scale);
  }
}

// -------------------------------------------------------------- values
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

template <typename T, int PER>
__global__ void __launch_bounds__(256) cb_quant_values_kernel(const T* __restrict__ x, int64_t total, int heads,
                                                              int dim, int refinements, float alpha, int mean_bf16,
                                                              CbTable tb, uint8_t* __restrict__ q, void* mean_out,
                                                              bf16* __restrict__ scale_out) {
  const int lane = threadIdx.x & 31;
  const int64_t w = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= total * heads) return;
  const int64_t t = w / heads;
  const int h = int(w - t * heads);
  const T* src = x + w * dim;
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane + 32 * i;
    v[i] = d < dim ? to_f(src[d]) : 0.f;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) s += v[i];
  float mean = warp_sum(s) / float(dim);
  mean = mean_bf16 ? round_bf16(mean) : mean;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i)
    if (lane + 32 * i < dim) {
      const float r = v[i] - mean;
      ss = fmaf(r, r, ss);
    }
  float scale = round_bf16(sqrtf(warp_sum(ss) / float(dim)) * alpha);
  for (int it = 0; it < refinements; ++it) {
    const float den_s = fmaxf(scale, 1e-20f);
    float num = 0.f, den = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i < dim) {
        const float r = v[i] - mean;
        const float c = center_of(cell_of(r / den_s, tb), tb);
        num = fmaf(r, c, num);
        den = fmaf(c, c, den);
      }
    num = warp_sum(num);
    den = warp_sum(den);
    scale = round_bf16(fmaxf(num / fmaxf(den, 1e-20f), 0.f));
  }
  const float den_s = fmaxf(scale, 1e-20f);
  uint8_t* qr = q + w * dim;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int d = lane + 32 * i;
    if (d < dim) qr[d] = uint8_t(cell_of((v[i] - mean) / den_s, tb));
  }
  if (lane == 0) {
    const int64_t pidx = int64_t(h) * total + t;  // [heads, total]
    if (mean_bf16)
      reinterpret_cast<bf16*>(mean_out)[pidx] = __float2bfloat16_rn(mean);
    else
      reinterpret_cast<float*>(mean_out)[pidx] = mean;
    scale_out[pidx] = __float2bfloat16_rn(scale);
  }
}

// ------------------------------------------------------------- dequant
// part 0 (keys): params [heads, ng, dim]; part 1 (values): [heads, total]
template <typename T>
__global__ void cb_dequant_kernel(const uint8_t* __restrict__ q, int64_t total, int heads, int dim, int group,
                                  int part, const void* mean_in, int mean_bf16, const bf16* __restrict__ scale_in,
                                  CbTable tb, T* __restrict__ out, uint32_t* status) {
  const int64_t n = total * heads * dim;
  const int ng = int((total + group - 1) / group);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int d = int(i % dim);
    const int64_t th = i / dim;
    const int h = int(th % heads);
    const int64_t t = th / heads;
    const int64_t pidx = part == 0 ? (int64_t(h) * ng + t / group) * dim + d : int64_t(h) * total + t;
    const float mean = mean_bf16 ? __bfloat162float(reinterpret_cast<const bf16*>(mean_in)[pidx])
                                 : reinterpret_cast<const float*>(mean_in)[pidx];
    const float sc = __bfloat162float(scale_in[pidx]);
    int s = q[i];
    if (s >= tb.levels) {
      atomicCAS(status, 0u, uint32_t(kStatusBadSymbol));
      s = tb.levels - 1;
    }
    // product and sum rounded separately (no FMA contraction), as in PyTorch
    out[i] = from_f<T>(__fadd_rn(__fmul_rn(center_of(s, tb), sc), mean));
  }
}

CbTable make_table(const torch::Tensor& centers) {
  KVS_CHECK_ARG(centers.device().is_cpu() && centers.scalar_type() == at::kFloat && centers.dim() == 1 &&
                    centers.numel() >= 2 && centers.numel() <= kCbMaxLevels,
                "codebook: centers must be a CPU float32 vector of 2..16 entries");
  CbTable tb{};
  const float* c = centers.data_ptr<float>();
  tb.levels = int(centers.numel());
  for (int i = 0; i < tb.levels; ++i) tb.centers[i] = c[i];
  // cell bounds are the midpoints of adjacent centres, in fp32 as in PyTorch
  for (int i = 0; i + 1 < tb.levels; ++i) tb.bounds[i] = (c[i] + c[i + 1]) / 2.0f;
  return tb;
}

#define KVS_CB_DISPATCH(dtype, T, ...)                                  \
  if (dtype == at::kBFloat16) {                                         \
    using T = bf16;                                                     \
    __VA_ARGS__;                                                        \
  } else if (dtype == at::kHalf) {                                      \
    using T = __half;                                                   \
    __VA_ARGS__;                                                        \
  } else if (dtype == at::kFloat) {                                     \
    using T = float;                                                    \
    __VA_ARGS__;                                                        \
  } else {                                                              \
    KVS_CHECK_ARG(false, "codebook: bf16, fp16 or fp32 input");         \
  }

}  // namespace

void codebook_quantize(torch::Tensor x, int64_t part, int64_t group, int64_t refinements, double alpha,
                       torch::Tensor centers, torch::Tensor q, torch::Tensor mean, torch::Tensor scale) {
  KVS_CHECK_ARG(x.is_cuda() && x.dim() == 3 && x.is_contiguous(), "codebook: x [tokens, heads, dim] contiguous CUDA");
  KVS_CHECK_ARG(q.is_cuda() && q.scalar_type() == at::kByte && q.is_contiguous() && q.numel() == x.numel(),
                "codebook: q uint8 like x");
  KVS_CHECK_ARG(scale.scalar_type() == at::kBFloat16 && scale.is_contiguous() &&
                    (mean.scalar_type() == at::kBFloat16 || mean.scalar_type() == at::kFloat) &&
                    mean.is_contiguous() && mean.numel() == scale.numel(),
                "codebook: bf16 scale and bf16/fp32 mean");
  const int64_t total = x.size(0);
  const int heads = int(x.size(1)), dim = int(x.size(2));
  KVS_CHECK_ARG(dim >= 1 && dim <= 512 && refinements >= 0 && refinements <= 2, "codebook: dim 1..512, 0..2 refinements");
  const CbTable tb = make_table(centers);
  const int mean_bf16 = mean.scalar_type() == at::kBFloat16;
  if (total == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (part == 0) {
    KVS_CHECK_ARG(group >= 1, "codebook: group size");
    const int64_t ng = (total + group - 1) / group;
    KVS_CHECK_ARG(scale.numel() == ng * heads * dim, "codebook: key params [heads, groups, dim]");
    KVS_CB_DISPATCH(x.scalar_type(), T,
                    cb_quant_keys_kernel<T><<<dim3(unsigned(ng), unsigned(heads)), 128, 0, st>>>(
                        reinterpret_cast<const T*>(x.data_ptr()), total, heads, dim, int(group), int(refinements),
                        float(alpha), mean_bf16, tb, q.data_ptr<uint8_t>(), mean.data_ptr(),
                        reinterpret_cast<bf16*>(scale.data_ptr())));
  } else {
    KVS_CHECK_ARG(scale.numel() == total * heads, "codebook: value params [heads, tokens]");
    const int64_t warps = total * heads;
    const unsigned blocks = unsigned((warps + 7) / 8);
#define KVS_CB_V(PER)                                                                                             \
  KVS_CB_DISPATCH(x.scalar_type(), T,                                                                             \
                  cb_quant_values_kernel<T, PER><<<blocks, 256, 0, st>>>(                                         \
                      reinterpret_cast<const T*>(x.data_ptr()), total, heads, dim, int(refinements), float(alpha), \
                      mean_bf16, tb, q.data_ptr<uint8_t>(), mean.data_ptr(), reinterpret_cast<bf16*>(scale.data_ptr())))
    if (dim <= 64) {
      KVS_CB_V(2)
    } else if (dim <= 128) {
      KVS_CB_V(4)
    } else if (dim <= 256) {
      KVS_CB_V(8)
    } else {
      KVS_CB_V(16)
    }
#undef KVS_CB_V
  }
  KVS_CUDA_CHECK(cudaGetLastError());
}

void codebook_dequantize(torch::Tensor q, int64_t part, int64_t group, torch::Tensor centers, torch::Tensor mean,
                         torch::Tensor scale, torch::Tensor out, torch::Tensor status) {
  KVS_CHECK_ARG(q.is_cuda() && q.dim() == 3 && q.is_contiguous() && q.scalar_type() == at::kByte,
                "codebook: q uint8 [tokens, heads, dim]");
  KVS_CHECK_ARG(out.is_cuda() && out.is_contiguous() && out.numel() == q.numel(), "codebook: out like q");
  KVS_CHECK_ARG(scale.scalar_type() == at::kBFloat16 && scale.is_contiguous() && mean.is_contiguous() &&
                    (mean.scalar_type() == at::kBFloat16 || mean.scalar_type() == at::kFloat) &&
                    mean.numel() == scale.numel(),
                "codebook: bf16 scale and bf16/fp32 mean");
  const int64_t total = q.size(0);
  const int heads = int(q.size(1)), dim = int(q.size(2));
  const int64_t ng = part == 0 ? (total + group - 1) / std::max<int64_t>(group, 1) : 0;
  KVS_CHECK_ARG(part == 0 ? (group >= 1 && scale.numel() == ng * heads * dim) : scale.numel() == total * heads,
                "codebook: parameter shape");
  const CbTable tb = make_table(centers);
  const int64_t n = q.numel();
  if (n == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const unsigned blocks = unsigned(std::min<int64_t>((n + 255) / 256, 148 * 16));
  const int mean_bf16 = mean.scalar_type() == at::kBFloat16;
  KVS_CB_DISPATCH(out.scalar_type(), T,
                  cb_dequant_kernel<T><<<blocks, 256, 0, st>>>(
                      q.data_ptr<uint8_t>(), total, heads, dim, int(std::max<int64_t>(group, 1)), int(part),
                      mean.data_ptr(), mean_bf16, reinterpret_cast<const bf16*>(scale.data_ptr()), tb,
                      reinterpret_cast<T*>(out.data_ptr()), reinterpret_cast<uint32_t*>(status.data_ptr<int32_t>())));
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
