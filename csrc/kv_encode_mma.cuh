// Frame encode with the random-sign Hadamard transform on the tensor cores
// (head_dim 128, quantised sections).  Included by kv_codec.cu after the
// frame helpers, EncodeArgs, encode_signal_done and the MMA decoder (whose
// sw128_off / tile constants it shares).
//
// Work unit = (part, head slot j, 128-token tile).  For a unit the CTA
//   1. loads the tile's 128 bf16 rows of head order[j] with 16-byte loads,
//      flips the signs of the head's random-sign channels (exact: the sign
//      bit of a bf16) and stores them in the 128-byte-swizzled K-major
//      layout the UMMA reads;
//   2. issues eight tcgen05.mma against the +-1 Sylvester Hadamard matrix H
//      (built once per CTA) into 128 TMEM columns;
//   3. reads the accumulator back.
//
// Two launches per layer, as in the SIMT path:
//   * kv_stats_mma_kernel:  K units compute D^T = H (s.K)^T, so TMEM lane =
//     channel and the per-channel min/max over the tile's tokens is a
//     register reduction per thread; V units compute (s.V) H with lane =
//     token and reduce each token's 128 values of the head.  Both end in
//     ordered-integer atomics on the layer's statistics (K: [2][H*D],
//     V: [2 sections][2][T]).
//   * kv_quant_mma_kernel:  every unit computes (s.X) H with lane = token,
//     quantises with the per-channel (K) or per-token (V) bf16 parameters
//     derived from the statistics, packs the token's 128 symbols LSB-first
//     and stores them into the frame (local or a peer's receive slot); the
//     last CTA writes the header, resets the statistics and publishes.
// Products with +-1 are exact and sums are fp32, so the transformed values
// equal the register butterfly's up to fp32 summation order.
#pragma once
#include "sm100.cuh"

namespace kvs {
namespace {

constexpr int kEncMmaThreads = 128;
constexpr int kEncOffA = 0;                       // token tile (A or B operand)
constexpr int kEncOffH = kMmaTile;                // Hadamard matrix
constexpr int kEncOffPar = 2 * kMmaTile;          // K params of every slot: min[H*D], inv[H*D] fp32
constexpr int kEncMaxHD = 8 * 128;
constexpr int kEncOffBar = kEncOffPar + 2 * kEncMaxHD * 4;
constexpr int kEncSmem = kEncOffBar + 64 + 1024;

struct EncUnit {
  int part, j, tile;
};

// Units: all K units (slot-major within a tile row of the grid) then all V units.
__device__ __forceinline__ EncUnit enc_unit(int64_t u, int H, int ntile, int part_mask) {
  const int per_part = H * ntile;
  EncUnit e;
  int p = int(u / per_part);
  if (part_mask == 2) p = 1;
  const int r = int(u % per_part);
  e.part = p;
  e.j = r / ntile;
  e.tile = r % ntile;
  return e;
}

__device__ __forceinline__ void enc_build_h(uint8_t* smem, int tid, int nthreads) {
  for (int i = tid; i < 128 * 16; i += nthreads) {
    const int e = i >> 4, c16 = i & 15;
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int d0 = c16 * 8 + 2 * q;
      const uint16_t h0 = (__popc(e & d0) & 1) ? 0xBF80u : 0x3F80u;
      const uint16_t h1 = (__popc(e & (d0 + 1)) & 1) ? 0xBF80u : 0x3F80u;
      w[q] = uint32_t(h0) | (uint32_t(h1) << 16);
    }
    *reinterpret_cast<uint4*>(smem + kEncOffH + sw128_off(e, c16)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

constexpr int kEncRowsPerPass = kEncMmaThreads / 16;   // 8 rows of 16 x 16-byte chunks per pass
constexpr int kEncLoads = 128 / kEncRowsPerPass;        // 16 loads per thread per tile

// Issues the 16 loads of this thread's chunks of a 128-token tile of head
// slot j (rows past T read as zero); the data are consumed by enc_put_tile,
// so the loads of the next unit overlap the current unit's epilogue.
__device__ __forceinline__ void enc_fetch_tile(const EncodeArgs& a, int part, int j, int t0, int tid,
                                               uint4 (&buf)[kEncLoads]) {
  const bf16* base = part ? a.v : a.k;
  const int64_t tok_stride = part ? a.v_tok_stride : a.k_tok_stride;
  const int64_t head_stride = part ? a.v_head_stride : a.k_head_stride;
  const int64_t block_stride = part ? a.v_block_stride : a.k_block_stride;
  const int hsrc = a.order[j];
  const int c16 = tid & 15;
#pragma unroll
  for (int i = 0; i < kEncLoads; ++i) {
    const int t = t0 + i * kEncRowsPerPass + (tid >> 4);
    buf[i] = make_uint4(0, 0, 0, 0);
    if (t < a.g.T)
      buf[i] = __ldg(reinterpret_cast<const uint4*>(
          src_row(base, t, hsrc, tok_stride, head_stride, a.block_table, a.block_size, block_stride) + c16 * 8));
  }
}

// Sign flip (the bf16 sign bit of the head's negative channels; rows past T
// stay zero) and store into the SW128 tile.
__device__ __forceinline__ void enc_put_tile(const EncodeArgs& a, uint8_t* smem, int j, int tid,
                                             const uint4 (&buf)[kEncLoads]) {
  const uint32_t* sb = a.sign_bits + a.order[j] * 4;
  const int c16 = tid & 15;
  const uint32_t sbyte = (sb[c16 >> 2] >> ((c16 & 3) * 8)) & 0xffu;
  uint4 flip;
  flip.x = ((sbyte & 1u) ? 0x8000u : 0u) | ((sbyte & 2u) ? 0x80000000u : 0u);
  flip.y = ((sbyte & 4u) ? 0x8000u : 0u) | ((sbyte & 8u) ? 0x80000000u : 0u);
  flip.z = ((sbyte & 16u) ? 0x8000u : 0u) | ((sbyte & 32u) ? 0x80000000u : 0u);
  flip.w = ((sbyte & 64u) ? 0x8000u : 0u) | ((sbyte & 128u) ? 0x80000000u : 0u);
#pragma unroll
  for (int i = 0; i < kEncLoads; ++i) {
    const int row = i * kEncRowsPerPass + (tid >> 4);
    uint4 x = buf[i];
    x.x ^= flip.x;   // zero rows flip to -0.0, which the transform treats as 0
    x.y ^= flip.y;
    x.z ^= flip.z;
    x.w ^= flip.w;
    *reinterpret_cast<uint4*>(smem + kEncOffA + sw128_off(row, c16)) = x;
  }
}

// D = A * B^T over K = 128 (eight K=16 steps), both operands SW128 K-major.
__device__ __forceinline__ void enc_mma(uint32_t tmem, uint32_t a_base, uint32_t b_base, uint64_t* bar) {
  using namespace sm100;
  constexpr uint32_t idesc = idesc_bf16(128, 128, false);
  tc_fence_after();
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t off = (kk >> 2) * kMmaPanel + (kk & 3) * 32;
    umma_f16(tmem, smem_desc_sw128(a_base + off, 16, 1024), smem_desc_sw128(b_base + off, 16, 1024), idesc,
             kk > 0 ? 1u : 0u);
  }
  umma_commit(bar);
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kEncMmaThreads) kv_stats_mma_kernel(EncodeArgs a) {
  using namespace sm100;
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kEncOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kEncOffBar + 8);
  const int tid = threadIdx.x, warp = tid >> 5;
  const FrameGeom& g = a.g;
  const int ntile = (g.T + 127) / 128;
  const int nparts = a.part_mask == 3 ? 2 : 1;
  const int64_t total = int64_t(nparts) * g.H * ntile;
  uint4 buf[kEncLoads];
  EncUnit e{};
  if (blockIdx.x < total) {  // the first tile's loads overlap the set-up
    e = enc_unit(blockIdx.x, g.H, ntile, a.part_mask);
    enc_fetch_tile(a, e.part, e.j, e.tile * 128, tid, buf);
  }
  enc_build_h(smem, tid, kEncMmaThreads);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc<128>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tile_s = smem_u32(smem + kEncOffA), h_s = smem_u32(smem + kEncOffH);
  const float scale = inv_sqrt_d<D>();
  const int HD = g.H * D;
  uint32_t phase = 0;
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    const int t0 = e.tile * 128;
    const int nvalid = min(128, g.T - t0);
    enc_put_tile(a, smem, e.j, tid, buf);
    fence_proxy_async_smem();
    __syncthreads();
    // K: D^T = H (s.K)^T (lane = channel); V: D = (s.V) H (lane = token)
    if (tid == 0) {
      if (e.part == 0) enc_mma(tmem, h_s, tile_s, bar);
      else enc_mma(tmem, tile_s, h_s, bar);
    }
    const EncUnit cur = e;
    if (u + gridDim.x < total) {  // next unit's loads run under this unit's MMA and epilogue
      e = enc_unit(u + gridDim.x, g.H, ntile, a.part_mask);
      enc_fetch_tile(a, e.part, e.j, e.tile * 128, tid, buf);
    }
    const bool done = mbar_wait(bar, phase, a.counter + 1);
    if (!__syncthreads_and(done)) {
      if (tid == 0) mbar_wait(bar, phase, nullptr);
      break;
    }
    phase ^= 1u;
    tc_fence_after();
    const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
    float lo = INFINITY, hi = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(trow + uint32_t(c * 32), r);
      tmem_wait_ld();
      if (cur.part == 0) {
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if (c * 32 + q < nvalid) {
            lo = fminf(lo, __uint_as_float(r[q]));
            hi = fmaxf(hi, __uint_as_float(r[q]));
          }
      } else {
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          lo = fminf(lo, __uint_as_float(r[q]));
          hi = fmaxf(hi, __uint_as_float(r[q]));
        }
      }
    }
    if (cur.part == 0) {
      const int c = cur.j * D + tid;  // lane = channel
      atomicMin(&a.stats[c], float_to_ordered(lo * scale));
      atomicMax(&a.stats[HD + c], float_to_ordered(hi * scale));
    } else if (tid < nvalid) {
      const int s = cur.j < g.n_low ? 0 : 1;
      uint32_t* vs = a.stats + 2 * HD + int64_t(s) * 2 * g.T;
      atomicMin(&vs[t0 + tid], float_to_ordered(lo * scale));
      atomicMax(&vs[g.T + t0 + tid], float_to_ordered(hi * scale));
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<128>(tmem);
  }
}

// Packs 32 symbols of `bits` each (LSB-first) into `bits` 32-bit words.
template <int BITS>
__device__ __forceinline__ void pack32(const uint32_t (&q)[32], uint32_t* dst) {
  uint32_t w[BITS];
#pragma unroll
  for (int i = 0; i < BITS; ++i) w[i] = 0;
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int bit = e * BITS;
    w[bit >> 5] |= q[e] << (bit & 31);
    if ((bit & 31) + BITS > 32) w[(bit >> 5) + 1] |= q[e] >> (32 - (bit & 31));
  }
  if constexpr (BITS % 4 == 0) {
#pragma unroll
    for (int i = 0; i < BITS; i += 4) *reinterpret_cast<uint4*>(dst + i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
  } else if constexpr (BITS % 2 == 0) {
#pragma unroll
    for (int i = 0; i < BITS; i += 2) *reinterpret_cast<uint2*>(dst + i) = make_uint2(w[i], w[i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < BITS; ++i) dst[i] = w[i];
  }
}

__device__ __forceinline__ void pack32_any(const uint32_t (&q)[32], uint32_t* dst, int bits) {
  switch (bits) {
    case 1: pack32<1>(q, dst); break;
    case 2: pack32<2>(q, dst); break;
    case 3: pack32<3>(q, dst); break;
    case 4: pack32<4>(q, dst); break;
    case 5: pack32<5>(q, dst); break;
    case 6: pack32<6>(q, dst); break;
    case 7: pack32<7>(q, dst); break;
    default: pack32<8>(q, dst); break;
  }
}

__global__ void __launch_bounds__(kEncMmaThreads) kv_quant_mma_kernel(EncodeArgs a) {
  using namespace sm100;
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* kmin = reinterpret_cast<float*>(smem + kEncOffPar);
  float* kinv = kmin + kEncMaxHD;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kEncOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kEncOffBar + 8);
  const int tid = threadIdx.x, warp = tid >> 5;
  const FrameGeom& g = a.g;
  const int HD = g.H * D;
  const int ntile = (g.T + 127) / 128;
  const int nparts = a.part_mask == 3 ? 2 : 1;
  const int64_t total = int64_t(nparts) * g.H * ntile;
  uint4 buf[kEncLoads];
  EncUnit e{};
  if (blockIdx.x < total) {  // the first tile's loads overlap the set-up
    e = enc_unit(blockIdx.x, g.H, ntile, a.part_mask);
    enc_fetch_tile(a, e.part, e.j, e.tile * 128, tid, buf);
  }
  enc_build_h(smem, tid, kEncMmaThreads);
  // K parameters of every slot from the statistics (block 0 also writes them
  // and the section headers into the frame)
  if (a.part_mask & 1) {
    bf16* fmin = reinterpret_cast<bf16*>(a.frame + g.k_aux);
    bf16* fscl = fmin + HD;
    for (int c = tid; c < HD; c += kEncMmaThreads) {
      const int s = c / D < g.n_low ? 0 : 1;
      const float lo = ordered_to_float(a.stats[c]);
      const float hi = ordered_to_float(a.stats[HD + c]);
      const bf16 minb = rn(lo);
      const bf16 sclb = rn(fmaxf(hi - to_f32(minb), 1e-5f) / float(glevels(g, 0, s) - 1));
      kmin[c] = to_f32(minb);
      kinv[c] = 1.0f / to_f32(sclb);
      if (blockIdx.x == 0) {
        fmin[c] = minb;
        fscl[c] = sclb;
      }
    }
  }
  if (blockIdx.x == 0 && tid < 4) {
    const int p = tid >> 1, s = tid & 1;
    if (((a.part_mask >> p) & 1) && section_heads(g, s) > 0)
      write_bitpack_header(a.frame + gpayload(g, p, s), gbits(g, p, s), uint64_t(g.T) * section_heads(g, s) * D);
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc<128>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tile_s = smem_u32(smem + kEncOffA), h_s = smem_u32(smem + kEncOffH);
  const float scale = inv_sqrt_d<D>();
  uint32_t phase = 0;
  for (int64_t u = blockIdx.x; u < total; u += gridDim.x) {
    const int t0 = e.tile * 128;
    enc_put_tile(a, smem, e.j, tid, buf);
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) enc_mma(tmem, tile_s, h_s, bar);   // lane = token
    const EncUnit cur = e;
    if (u + gridDim.x < total) {  // next unit's loads run under this unit's MMA and epilogue
      e = enc_unit(u + gridDim.x, g.H, ntile, a.part_mask);
      enc_fetch_tile(a, e.part, e.j, e.tile * 128, tid, buf);
    }
    const bool done = mbar_wait(bar, phase, a.counter + 1);
    if (!__syncthreads_and(done)) {
      if (tid == 0) mbar_wait(bar, phase, nullptr);
      break;
    }
    phase ^= 1u;
    tc_fence_after();
    int s, js, hs;
    slot_section(g, cur.j, s, js, hs);
    const int bits = gbits(g, cur.part, s);
    const float top = float(glevels(g, cur.part, s) - 1);
    const int t = t0 + tid;
    const bool valid = t < g.T;
    float vmn = 0.f, vinv = 0.f;
    if (cur.part == 1 && valid) {
      const uint32_t* vs = a.stats + 2 * HD + int64_t(s) * 2 * g.T;
      const bf16 minb = rn(ordered_to_float(vs[t]));
      const bf16 sclb = rn(fmaxf(ordered_to_float(vs[g.T + t]) - to_f32(minb), 1e-5f) / top);
      vmn = to_f32(minb);
      vinv = 1.0f / to_f32(sclb);
      if (js == 0) {
        bf16* aux = reinterpret_cast<bf16*>(a.frame + gvaux(g, s));
        aux[t] = minb;
        aux[g.T + t] = sclb;
      }
    }
    const int64_t sym = (int64_t(t) * hs + js) * D;
    uint32_t* dst = reinterpret_cast<uint32_t*>(a.frame + gpayload(g, cur.part, s) + 16 + sym * bits / 8);
    const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld32(trow + uint32_t(c * 32), r);
      tmem_wait_ld();
      if (!valid) continue;
      uint32_t q[32];
      if (cur.part == 0) {
        const float* mn = kmin + cur.j * D + c * 32;
        const float* iv = kinv + cur.j * D + c * 32;
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const float y = rintf((__uint_as_float(r[x]) * scale - mn[x]) * iv[x]);
          q[x] = uint32_t(fminf(fmaxf(y, 0.0f), top));
        }
      } else {
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const float y = rintf((__uint_as_float(r[x]) * scale - vmn) * vinv);
          q[x] = uint32_t(fminf(fmaxf(y, 0.0f), top));
        }
      }
      pack32_any(q, dst + c * bits, bits);
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc<128>(tmem);
  }
  encode_signal_done(a);
}

}  // namespace
}  // namespace kvs
