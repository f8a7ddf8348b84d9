// Memory-bound engine kernels for the standalone PD engine (sm_100a):
// RMSNorm (optionally fused with the residual add), RoPE fused with the K/V
// write into the sequence buffer or the paged cache, SiLU-and-multiply,
// embedding gather, greedy argmax.  All loads/stores are 16-byte vectors.
// (The reference delegates all of these to vLLM; they are required by the
// standalone engine of this framework.)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cstdlib>

#include "common.cuh"
#include "ops.h"

namespace kvs {

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("KVSERVE_PDL");
    return !(e && (e[0] == '0' || e[0] == 'n' || e[0] == 'N' || e[0] == 'f' || e[0] == 'F'));
  }();
  return on;
}

namespace {

__device__ __forceinline__ void unpack8(const uint4& raw, float (&v)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 out;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  return out;
}

template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kThreads / 32 ? red[lane] : 0.f;
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) t += __shfl_xor_sync(0xffffffffu, t, m);
  __syncthreads();
  return t;
}

// out = rmsnorm(x [+ residual]) * w; when residual != null the sum is
// rounded to bf16 and written back into residual (the new residual stream).
template <int kThreads, int kVec>
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const bf16* __restrict__ x,
                                                           bf16* __restrict__ residual,
                                                           const bf16* __restrict__ w,
                                                           bf16* __restrict__ out, int hidden,
                                                           float eps) {
  pdl_trigger();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const bf16* xr = x + row * hidden;
  float v[kVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = (i * kThreads + threadIdx.x) * 8;
    if (c < hidden) {
      unpack8(*reinterpret_cast<const uint4*>(xr + c), v[i]);
      if (residual) {
        float r[8];
        unpack8(*reinterpret_cast<const uint4*>(residual + row * hidden + c), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = rnf(v[i][e] + r[e]);
        *reinterpret_cast<uint4*>(residual + row * hidden + c) = pack8(v[i]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
    }
  }
  const float tot = block_sum<kThreads>(ss, red);
  const float inv = rsqrtf(tot / float(hidden) + eps);
#pragma unroll
  for (int i = 0; i < kVec; ++i) {
    const int c = (i * kThreads + threadIdx.x) * 8;
    if (c < hidden) {
      float wv[8];
      unpack8(*reinterpret_cast<const uint4*>(w + c), wv);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = rnf(v[i][e] * inv) * wv[e];
      *reinterpret_cast<uint4*>(out + row * hidden + c) = pack8(o);
    }
  }
}

// Rotary embedding (rotate-half / NeoX pairing (i, i + D/2)) applied in place
// to the q and k heads of a fused QKV row, plus a copy of the rotated k and
// of v into a destination addressed by slot: dst + slot*token_stride +
// head*head_stride.  slot = slot_mapping[t] (paged cache) or slot_base + t.
__global__ void rope_qkv_kernel(bf16* __restrict__ qkv, int64_t qkv_stride, int T, int Hq, int Hkv,
                                int D, const int32_t* __restrict__ positions,
                                const float* __restrict__ cos_sin, bf16* __restrict__ k_dst,
                                bf16* __restrict__ v_dst, int64_t dst_token_stride,
                                int64_t dst_head_stride, const int32_t* __restrict__ slot_mapping,
                                int64_t slot_base) {
  pdl_trigger();
  const int t = blockIdx.x;
  if (t >= T) return;
  const int half = D / 2;
  const int pos = positions[t];
  const float* cs = cos_sin + int64_t(pos) * D;  // cos[half] | sin[half]
  bf16* row = qkv + int64_t(t) * qkv_stride;
  const int pairs_q = Hq * half, pairs_k = Hkv * half;
  for (int i = threadIdx.x; i < pairs_q + pairs_k; i += blockDim.x) {
    const bool is_k = i >= pairs_q;
    const int ii = is_k ? i - pairs_q : i;
    const int h = ii / half, d = ii % half;
    bf16* base = row + (is_k ? (Hq + h) * D : h * D);
    const float x1 = to_f32(base[d]), x2 = to_f32(base[d + half]);
    const float c = cs[d], s = cs[half + d];
    const bf16 o1 = rn(x1 * c - x2 * s), o2 = rn(x2 * c + x1 * s);
    base[d] = o1;
    base[d + half] = o2;
    if (is_k && k_dst) {
      const int64_t slot = slot_mapping ? int64_t(slot_mapping[t]) : slot_base + t;
      bf16* kd = k_dst + slot * dst_token_stride + int64_t(h) * dst_head_stride;
      kd[d] = o1;
      kd[d + half] = o2;
    }
  }
  if (v_dst) {
    const int64_t slot = slot_mapping ? int64_t(slot_mapping[t]) : slot_base + t;
    const bf16* vr = row + (Hq + Hkv) * D;
    for (int i = threadIdx.x * 8; i < Hkv * D; i += blockDim.x * 8) {
      const int h = i / D, d = i % D;
      *reinterpret_cast<uint4*>(v_dst + slot * dst_token_stride + int64_t(h) * dst_head_stride + d) =
          *reinterpret_cast<const uint4*>(vr + i);
    }
  }
}

// out[r, c] = silu(gate[r, c]) * up[r, c].  blk == 0: gate = gu[:, :inter],
// up = gu[:, inter:]; blk > 0: gate/up interleaved in blocks of blk columns
// (the layout the fused GEMM epilogue consumes).
__global__ void silu_mul_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int64_t rows,
                                int inter, int blk) {
  pdl_trigger();
  const int64_t groups = rows * (inter / 8);
  for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
       g += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = g / (inter / 8);
    const int c = int(g % (inter / 8)) * 8;
    float a[8], b[8], o[8];
    const int gc = blk ? (c / blk) * 2 * blk + c % blk : c;
    const int uc = blk ? gc + blk : inter + c;
    unpack8(*reinterpret_cast<const uint4*>(gu + r * 2 * inter + gc), a);
    unpack8(*reinterpret_cast<const uint4*>(gu + r * 2 * inter + uc), b);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float sg = a[e] / (1.0f + __expf(-a[e]));
      o[e] = rnf(sg) * b[e];
    }
    *reinterpret_cast<uint4*>(out + r * inter + c) = pack8(o);
  }
}

__global__ void embedding_kernel(const int32_t* __restrict__ ids, const bf16* __restrict__ table,
                                 bf16* __restrict__ out, int T, int hidden, int64_t vocab_begin,
                                 int64_t vocab_rows) {
  pdl_trigger();
  const int t = blockIdx.x;
  const int64_t id = int64_t(ids[t]) - vocab_begin;
  const bool mine = id >= 0 && id < vocab_rows;
  for (int c = threadIdx.x * 8; c < hidden; c += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (mine) v = *reinterpret_cast<const uint4*>(table + id * hidden + c);
    *reinterpret_cast<uint4*>(out + int64_t(t) * hidden + c) = v;
  }
}

// Greedy sampling: index of the maximum logit per row (lowest index wins ties).
__global__ void argmax_kernel(const bf16* __restrict__ logits, int64_t row_stride, int V,
                              int32_t* __restrict__ out, float* __restrict__ out_val,
                              int64_t index_offset) {
  pdl_trigger();
  __shared__ float sv[32];
  __shared__ int si[32];
  const bf16* r = logits + int64_t(blockIdx.x) * row_stride;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = to_f32(r[i]);
    if (x > best || (x == best && i < bi)) { best = x; bi = i; }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = lane < int(blockDim.x / 32) ? sv[lane] : -INFINITY;
    bi = lane < int(blockDim.x / 32) ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      out[blockIdx.x] = int32_t(bi + index_offset);
      if (out_val) out_val[blockIdx.x] = best;
    }
  }
}

// Per decode step bookkeeping, captured together with the step in one CUDA
// graph: feed the sampled token back, record it, advance position / context
// length and compute the next cache slot from the block table.
__global__ void decode_advance_kernel(const int32_t* __restrict__ tok, int32_t* __restrict__ ids,
                                      int32_t* __restrict__ pos, int32_t* __restrict__ ctx,
                                      int32_t* __restrict__ slot, const int32_t* __restrict__ table,
                                      int64_t table_stride, int block_size, int32_t* __restrict__ out_tokens,
                                      int32_t* __restrict__ step, int max_steps, int B) {
  pdl_trigger();
  const int b = threadIdx.x;
  const int s = *step;
  __syncthreads();
  if (b < B) {
    const int32_t t = tok[b];
    ids[b] = t;
    if (s < max_steps) out_tokens[int64_t(s) * B + b] = t;
    const int p = pos[b] + 1;
    pos[b] = p;
    ctx[b] = ctx[b] + 1;
    slot[b] = table[b * table_stride + p / block_size] * block_size + p % block_size;
  }
  __syncthreads();
  if (b == 0) *step = s + 1;
}

// Continuous-batching variant: every row is its own request with its own
// token count.  Rows with active[b] == 0 are padding (they point at a scratch
// block and do not advance); out_tokens is [B, ld] with row b's t-th token at
// out_tokens[b * ld + t].
__global__ void batch_advance_kernel(const int32_t* __restrict__ tok, const int32_t* __restrict__ active,
                                     int32_t* __restrict__ ids, int32_t* __restrict__ pos,
                                     int32_t* __restrict__ ctx, int32_t* __restrict__ slot,
                                     const int32_t* __restrict__ table, int64_t table_stride, int block_size,
                                     int32_t* __restrict__ out_tokens, int64_t ld, int32_t* __restrict__ steps,
                                     int B) {
  pdl_trigger();
  const int b = threadIdx.x;
  if (b >= B || !active[b]) return;
  const int32_t t = tok[b];
  ids[b] = t;
  const int s = steps[b];
  if (s < ld) out_tokens[int64_t(b) * ld + s] = t;
  steps[b] = s + 1;
  const int p = pos[b] + 1;
  pos[b] = p;
  ctx[b] = ctx[b] + 1;
  slot[b] = table[b * table_stride + p / block_size] * block_size + p % block_size;
}

}  // namespace

void batch_advance(torch::Tensor tok, torch::Tensor active, torch::Tensor ids, torch::Tensor pos, torch::Tensor ctx,
                   torch::Tensor slot, torch::Tensor table, int64_t block_size, torch::Tensor out_tokens,
                   torch::Tensor steps) {
  const int B = int(ids.numel());
  KVS_CHECK_ARG(B >= 1 && B <= 1024 && table.dim() == 2 && table.size(0) >= B && out_tokens.dim() == 2 &&
                    out_tokens.size(0) >= B && out_tokens.stride(1) == 1 && active.numel() >= B &&
                    steps.numel() >= B && tok.numel() >= B,
                "batch_advance: per-row state of B rows");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  batch_advance_kernel<<<1, std::max(32, B), 0, st>>>(
      tok.data_ptr<int32_t>(), active.data_ptr<int32_t>(), ids.data_ptr<int32_t>(), pos.data_ptr<int32_t>(),
      ctx.data_ptr<int32_t>(), slot.data_ptr<int32_t>(), table.data_ptr<int32_t>(), table.stride(0),
      int(block_size), out_tokens.data_ptr<int32_t>(), out_tokens.stride(0), steps.data_ptr<int32_t>(), B);
  KVS_CUDA_CHECK(cudaGetLastError());
}

void decode_advance(torch::Tensor tok, torch::Tensor ids, torch::Tensor pos, torch::Tensor ctx, torch::Tensor slot,
                    torch::Tensor table, int64_t block_size, torch::Tensor out_tokens, torch::Tensor step) {
  const int B = int(ids.numel());
  KVS_CHECK_ARG(B >= 1 && B <= 1024 && table.dim() == 2, "decode_advance: batch / table");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  decode_advance_kernel<<<1, std::max(32, B), 0, st>>>(
      tok.data_ptr<int32_t>(), ids.data_ptr<int32_t>(), pos.data_ptr<int32_t>(), ctx.data_ptr<int32_t>(),
      slot.data_ptr<int32_t>(), table.data_ptr<int32_t>(), table.stride(0), int(block_size),
      out_tokens.data_ptr<int32_t>(), step.data_ptr<int32_t>(), int(out_tokens.numel() / B), B);
  KVS_CUDA_CHECK(cudaGetLastError());
}

void rmsnorm(torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor w, torch::Tensor out,
             double eps) {
  KVS_CHECK_ARG(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.is_contiguous() && out.is_contiguous(),
                "rmsnorm: contiguous CUDA bf16");
  const int hidden = int(x.size(-1));
  KVS_CHECK_ARG(hidden % 8 == 0 && hidden <= 16384, "rmsnorm: hidden must be a multiple of 8, <= 16384");
  const int64_t rows = x.numel() / hidden;
  if (rows == 0) return;
  bf16* res = nullptr;
  if (residual.has_value()) {
    KVS_CHECK_ARG(residual->is_contiguous() && residual->numel() == x.numel(), "rmsnorm: residual shape");
    res = reinterpret_cast<bf16*>(residual->data_ptr());
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto op = reinterpret_cast<bf16*>(out.data_ptr());
  if (hidden <= 256 * 8)
    rmsnorm_kernel<256, 1><<<rows, 256, 0, st>>>(xp, res, wp, op, hidden, float(eps));
  else if (hidden <= 512 * 8)
    rmsnorm_kernel<512, 1><<<rows, 512, 0, st>>>(xp, res, wp, op, hidden, float(eps));
  else
    rmsnorm_kernel<512, 4><<<rows, 512, 0, st>>>(xp, res, wp, op, hidden, float(eps));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void rope_qkv(torch::Tensor qkv, int64_t Hq, int64_t Hkv, int64_t D, torch::Tensor positions,
              torch::Tensor cos_sin, c10::optional<torch::Tensor> k_dst, c10::optional<torch::Tensor> v_dst,
              int64_t dst_token_stride, int64_t dst_head_stride, c10::optional<torch::Tensor> slot_mapping,
              int64_t slot_base) {
  KVS_CHECK_ARG(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1,
                "rope_qkv: qkv must be [T, (Hq+2Hkv)*D] bf16");
  KVS_CHECK_ARG(qkv.size(1) == (Hq + 2 * Hkv) * D && D % 16 == 0, "rope_qkv: width mismatch");
  KVS_CHECK_ARG(positions.scalar_type() == at::kInt && cos_sin.scalar_type() == at::kFloat, "rope_qkv: dtypes");
  const int T = int(qkv.size(0));
  if (T == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  rope_qkv_kernel<<<T, 256, 0, st>>>(
      reinterpret_cast<bf16*>(qkv.data_ptr()), qkv.stride(0), T, int(Hq), int(Hkv), int(D),
      positions.data_ptr<int32_t>(), cos_sin.data_ptr<float>(),
      k_dst.has_value() ? reinterpret_cast<bf16*>(k_dst->data_ptr()) : nullptr,
      v_dst.has_value() ? reinterpret_cast<bf16*>(v_dst->data_ptr()) : nullptr, dst_token_stride,
      dst_head_stride, slot_mapping.has_value() ? slot_mapping->data_ptr<int32_t>() : nullptr, slot_base);
  KVS_CUDA_CHECK(cudaGetLastError());
}

void silu_mul(torch::Tensor gate_up, torch::Tensor out, int64_t blk) {
  const int inter = int(out.size(-1));
  KVS_CHECK_ARG(gate_up.size(-1) == 2 * inter && inter % 8 == 0 && gate_up.is_contiguous() && out.is_contiguous(),
                "silu_mul: shapes");
  KVS_CHECK_ARG(blk == 0 || (blk % 8 == 0 && inter % blk == 0), "silu_mul: interleave block");
  const int64_t rows = out.numel() / inter;
  if (rows == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  const int64_t groups = rows * (inter / 8);
  const int grid = int(std::min<int64_t>(ceil_div(groups, 256), 148 * 16));
  silu_mul_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const bf16*>(gate_up.data_ptr()),
                                        reinterpret_cast<bf16*>(out.data_ptr()), rows, inter, int(blk));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out, int64_t vocab_begin) {
  KVS_CHECK_ARG(ids.scalar_type() == at::kInt && table.is_contiguous() && out.is_contiguous(), "embedding: args");
  const int T = int(ids.numel());
  const int hidden = int(table.size(1));
  if (T == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  embedding_kernel<<<T, 256, 0, st>>>(ids.data_ptr<int32_t>(), reinterpret_cast<const bf16*>(table.data_ptr()),
                                      reinterpret_cast<bf16*>(out.data_ptr()), T, hidden, vocab_begin,
                                      table.size(0));
  KVS_CUDA_CHECK(cudaGetLastError());
}

void argmax_rows(torch::Tensor logits, torch::Tensor out, c10::optional<torch::Tensor> out_val,
                 int64_t index_offset) {
  KVS_CHECK_ARG(logits.dim() == 2 && logits.stride(1) == 1 && logits.scalar_type() == at::kBFloat16,
                "argmax: logits [B, V] bf16");
  const int B = int(logits.size(0));
  if (B == 0) return;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  argmax_kernel<<<B, 1024, 0, st>>>(reinterpret_cast<const bf16*>(logits.data_ptr()), logits.stride(0),
                                    int(logits.size(1)), out.data_ptr<int32_t>(),
                                    out_val.has_value() ? out_val->data_ptr<float>() : nullptr, index_offset);
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
