// Frame -> paged KV decode with the inverse Hadamard transform on the tensor
// cores (head_dim 128, quantised sections).  Included by kv_codec.cu after
// the frame helpers and DecodeArgs.
//
// Work unit = (layer, part, head slot, 128-token tile).  For a unit the CTA
//   1. dequantises the packed symbols of the tile into a bf16 A tile in
//      shared memory (K: per-channel parameters, V: per-token parameters),
//      written in the 128-byte-swizzled K-major layout the UMMA reads;
//   2. issues eight tcgen05.mma (M=128 tokens, N=128, K=16) against the
//      +-1 Sylvester Hadamard matrix H (built once per CTA, B operand),
//      accumulating fp32 in 128 TMEM columns;
//   3. reads the rows back (thread = token), applies 1/sqrt(D) and the
//      head's random signs, and stores the 256-byte bf16 row into the
//      token's paged block.
// Units are visited layer-major, so with publish flags a CTA waits (bounded)
// for a layer only when it reaches that layer's first unit.  The dequantised
// values are rounded to bf16 before the transform; products with +-1 are
// exact and sums are fp32, so the result differs from the register FWHT by
// about one bf16 rounding.
#pragma once
#include "sm100.cuh"

namespace kvs {
namespace {

constexpr int kMmaDecThreads = 256;
constexpr int kMmaPanel = 128 * 128;          // bytes: 128 rows x 64 bf16 (one SW128 panel)
constexpr int kMmaTile = 2 * kMmaPanel;       // 128 x 128 bf16
constexpr int kMmaOffA = 0;
constexpr int kMmaOffB = kMmaTile;
constexpr int kMmaOffPar = 2 * kMmaTile;      // K params: min[128], scale[128] fp32
constexpr int kMmaOffBar = kMmaOffPar + 2 * 128 * 4;
constexpr int kMmaSmem = kMmaOffBar + 64 + 1024;

// byte offset of element (row, col) inside a 128x128 bf16 SW128 K-major tile
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk16) {
  return uint32_t((chunk16 >> 3) * kMmaPanel + row * 128 + (((chunk16 & 7) ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kMmaDecThreads) kv_decode_mma_kernel(DecodeArgs a) {
  using namespace sm100;
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* kpar = reinterpret_cast<float*>(smem + kMmaOffPar);
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(smem + kMmaOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kMmaOffBar + 8);
  __shared__ int s_ok;
  __shared__ int s_layer;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // H[e][d] = (-1)^popc(e & d), B operand rows e, K-major
  for (int i = tid; i < 128 * 16; i += kMmaDecThreads) {
    const int e = i >> 4, c16 = i & 15;
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int d0 = c16 * 8 + 2 * q;
      const uint16_t h0 = (__popc(e & d0) & 1) ? 0xBF80u : 0x3F80u;        // bf16 -1 / +1
      const uint16_t h1 = (__popc(e & (d0 + 1)) & 1) ? 0xBF80u : 0x3F80u;
      w[q] = uint32_t(h0) | (uint32_t(h1) << 16);
    }
    *reinterpret_cast<uint4*>(smem + kMmaOffB + sw128_off(e, c16)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (tid == 0) {
    mbar_init(mma_bar, 1);
    fence_barrier_init();
    s_layer = -1;
    s_ok = 1;
  }
  if (warp == 0) tmem_alloc<128>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t a_base = smem_u32(smem + kMmaOffA), b_base = smem_u32(smem + kMmaOffB);
  constexpr uint32_t idesc = idesc_bf16(128, 128, false);
  const float scale = inv_sqrt_d<D>();
  const int bshift = (a.block_size & (a.block_size - 1)) == 0 ? __ffs(a.block_size) - 1 : -1;

  const int nparts = a.part_mask == 3 ? 2 : 1;
  const int ntile = (a.g.T + 127) / 128;
  const int per_layer = nparts * a.g.H * ntile;
  const int64_t total = int64_t(per_layer) * a.num_layers;
  uint32_t phase = 0;
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    const int li = int(u / per_layer);
    int rem = int(u % per_layer);
    const int pi = rem / (a.g.H * ntile);
    rem %= a.g.H * ntile;
    const int j = rem / ntile, tt = rem % ntile;
    const int part = a.part_mask == 2 ? 1 : pi;
    const int layer = a.layer_begin + li;
    FrameGeom g = a.g;
    if (a.n_lows != nullptr) {
      g.n_low = a.n_lows[layer];
      frame_geom_finalize(g);
    }
    const uint8_t* frame = a.frame_base + int64_t(li) * a.frame_stride;
    if (tid == 0 && s_layer != layer) {
      int ok = 1;
      if (a.flags != nullptr && !wait_flag_geq(a.flags + layer, a.seq, a.timeout_ns)) {
        atomicCAS(a.status, 0u, uint32_t(kStatusTimeout));
        ok = 0;
      }
      if (ok) {
        const FrameHeader* h = reinterpret_cast<const FrameHeader*>(frame);
        if (__ldcg(&h->magic) != kFrameMagic || __ldcg(&h->seq) != a.seq || __ldcg(&h->tokens) != uint32_t(g.T) ||
            __ldcg(&h->layer) != uint32_t(layer)) {
          atomicCAS(a.status, 0u, uint32_t(kStatusBadHeader));
          ok = 0;
        }
      }
      if (ok) asm volatile("fence.acq_rel.sys;" ::: "memory");
      s_ok = ok;
      s_layer = layer;
    }
    __syncthreads();
    if (!s_ok) break;

    int s, js, hs;
    slot_section(g, j, s, js, hs);
    const int bits = gbits(g, part, s);
    const int64_t pay = gpayload(g, part, s) + 16;
    const int h = a.orders[int64_t(layer) * g.H + j];
    if (part == 0) {  // K parameters of slot j (channels j*D .. j*D+127)
      const bf16* kmin = reinterpret_cast<const bf16*>(frame + g.k_aux);
      for (int c = tid; c < 2 * D; c += kMmaDecThreads) {
        const int64_t idx = (c < D ? 0 : int64_t(g.H) * D) + int64_t(j) * D + (c & (D - 1));
        kpar[c] = __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(kmin + idx))));
      }
      __syncthreads();
    }
    const bf16* vaux = reinterpret_cast<const bf16*>(frame + gvaux(g, s));
    const int t0 = tt * 128;
    const int t1 = min(g.T, t0 + 128);
    const uint64_t mask = (1ull << bits) - 1ull;
    // 1. dequantise into the A tile: 128 rows x 16 chunks of 8 values
#pragma unroll 2
    for (int i = tid; i < 128 * 16; i += kMmaDecThreads) {
      const int row = i >> 4, c16 = i & 15;
      const int t = t0 + row;
      uint4 out = make_uint4(0, 0, 0, 0);
      if (t < t1) {
        const int64_t sym = (int64_t(t) * hs + js) * D + c16 * 8;
        const uint64_t acc = load_packed(frame + pay + sym * bits / 8, bits);
        float mn[8], sc[8];
        if (part == 0) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            mn[e] = kpar[c16 * 8 + e];
            sc[e] = kpar[D + c16 * 8 + e];
          }
        } else {
          const float m = __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(vaux + t))));
          const float q = __bfloat162float(
              __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(vaux + g.T + t))));
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            mn[e] = m;
            sc[e] = q;
          }
        }
        __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v0 = mn[2 * e] + float((acc >> (2 * e * bits)) & mask) * sc[2 * e];
          const float v1 = mn[2 * e + 1] + float((acc >> ((2 * e + 1) * bits)) & mask) * sc[2 * e + 1];
          o2[e] = __floats2bfloat162_rn(v0, v1);
        }
      }
      *reinterpret_cast<uint4*>(smem + kMmaOffA + sw128_off(row, c16)) = out;
    }
    fence_proxy_async_smem();
    __syncthreads();
    // 2. Y = A * H on the tensor cores
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kMmaPanel + (kk & 3) * 32;
        umma_f16(tmem, smem_desc_sw128(a_base + off, 16, 1024), smem_desc_sw128(b_base + off, 16, 1024), idesc,
                 kk > 0 ? 1u : 0u);
      }
      umma_commit(mma_bar);
    }
    const bool done = mbar_wait(mma_bar, phase, a.status);
    if (!__syncthreads_and(done)) {
      // the MMA did not retire in time: wait once more (bounded) so TMEM is
      // never released under an MMA in flight, then give up
      if (tid == 0) mbar_wait(mma_bar, phase, nullptr);
      break;
    }
    phase ^= 1u;
    tc_fence_after();
    // 3. epilogue: warps 0..3, thread = token row
    if (warp < 4) {
      const int row = warp * 32 + lane;
      const int t = t0 + row;
      const uint32_t* sb = a.sign_bits + (int64_t(layer) * g.H + h) * (D / 32);
      bf16* dst = nullptr;
      if (t < t1) {
        bf16* cache = a.layer_ptrs != nullptr
                          ? reinterpret_cast<bf16*>(a.layer_ptrs[2 * layer + part])
                          : a.cache + int64_t(layer) * a.layer_stride + int64_t(part) * a.part_stride;
        int bi, bo;
        split_pos(a.tok_offset + t, a.block_size, bshift, bi, bo);
        dst = cache + int64_t(a.block_table[bi]) * a.block_stride + int64_t(bo) * a.token_stride +
              int64_t(h) * a.head_stride;
      }
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c * 32), r);
        tmem_wait_ld();
        const uint32_t sw = sb[c];
        if (dst != nullptr) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 o;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int d = v * 8 + 2 * e;
              float x0 = __uint_as_float(r[d]) * scale, x1 = __uint_as_float(r[d + 1]) * scale;
              if ((sw >> d) & 1u) x0 = -x0;
              if ((sw >> (d + 1)) & 1u) x1 = -x1;
              o2[e] = __floats2bfloat162_rn(x0, x1);
            }
            *reinterpret_cast<uint4*>(dst + c * 32 + v * 8) = o;
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // A tile, K params and TMEM are reused by the next unit
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<128>(tmem);
  }
}

}  // namespace
}  // namespace kvs
