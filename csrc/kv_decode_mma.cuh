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
      if (ok && a.trace != nullptr) trace_start(a.trace + 4 * layer + 2);
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


// ---------------------------------------------------------------------------
// Warp-specialised variant (the default): one persistent CTA per SM,
// 544 threads.
//   warps 0-11  three builder warpgroups taking units in turn: for a new
//               layer, thread 0 of the group acquire-waits (bounded) on the
//               layer's publish flag and checks the header; then every
//               thread dequantises one token row (its packed symbols are
//               16*bits contiguous bytes) into the SW128 A tile of a
//               4-stage ring;
//   warp 12     MMA issuer: A tile x H into one of four 128-column TMEM
//               accumulators;
//   warps 13-16 epilogue warpgroup: 1/sqrt(D), the head's signs, bf16,
//               256-byte row store into the paged block.
// A timed-out flag or a bad header sets the status word and a CTA-wide
// "bad" mark; the pipeline then keeps its protocol (no wait is left
// pending) but no row is stored.
constexpr int kDwGroups = 3;       // builder warpgroups (dequantisation is the heavier side)
constexpr int kDwEpi = 1;          // epilogue warpgroups
constexpr int kDwStages = 4;
constexpr int kDwAcc = 4;
constexpr int kDwThreads = 128 * kDwGroups + 32 + 128 * kDwEpi;
constexpr int kDwOffH = kDwStages * kMmaTile;
constexpr int kDwOffPar = kDwOffH + kMmaTile;                 // per builder group: K min[128], scale[128]
constexpr int kDwOffBar = kDwOffPar + kDwGroups * 2 * 128 * 4;
constexpr int kDwSmem = kDwOffBar + 256 + 1024;

template <int BITS>
__device__ __forceinline__ void dw_unpack_row(const uint32_t* w, const float* mn, const float* sc, bool per_chan,
                                              float vmin, float vscl, uint8_t* tile, int row) {
#pragma unroll
  for (int c16 = 0; c16 < 16; ++c16) {
    uint4 out;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float v[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int idx = c16 * 8 + 2 * e + h;
        const int bit = idx * BITS;
        uint32_t q = w[bit >> 5] >> (bit & 31);
        if ((bit & 31) + BITS > 32) q |= w[(bit >> 5) + 1] << (32 - (bit & 31));
        q &= (1u << BITS) - 1u;
        v[h] = per_chan ? mn[idx] + float(q) * sc[idx] : vmin + float(q) * vscl;
      }
      o2[e] = __floats2bfloat162_rn(v[0], v[1]);
    }
    *reinterpret_cast<uint4*>(tile + sw128_off(row, c16)) = out;
  }
}

__global__ void __launch_bounds__(kDwThreads, 1) kv_decode_ws_kernel(DecodeArgs a) {
  using namespace sm100;
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDwOffBar);
  uint64_t* empty = full + kDwStages;
  uint64_t* tfull = empty + kDwStages;   // [kDwAcc] is the abort drain
  uint64_t* tempty = tfull + kDwAcc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + kDwAcc);
  __shared__ int s_bad;
  __shared__ int s_ok[kDwGroups];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int kMmaWarp = 4 * kDwGroups;
  // H[e][d] = (-1)^popc(e & d), B operand rows e, K-major
  for (int i = tid; i < 128 * 16; i += kDwThreads) {
    const int e = i >> 4, c16 = i & 15;
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int d0 = c16 * 8 + 2 * q;
      const uint16_t h0 = (__popc(e & d0) & 1) ? 0xBF80u : 0x3F80u;
      const uint16_t h1 = (__popc(e & (d0 + 1)) & 1) ? 0xBF80u : 0x3F80u;
      w[q] = uint32_t(h0) | (uint32_t(h1) << 16);
    }
    *reinterpret_cast<uint4*>(smem + kDwOffH + sw128_off(e, c16)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (tid == 0) {
    for (int s = 0; s < kDwStages; ++s) {
      mbar_init(&full[s], 128);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kDwAcc; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(&tfull[kDwAcc], 1);
    fence_barrier_init();
    s_bad = 0;
  }
  if (warp == kMmaWarp) tmem_alloc<512>(tmem_slot);
  fence_proxy_async_smem();   // H is read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const FrameGeom g0 = a.g;
  const int nparts = a.part_mask == 3 ? 2 : 1;
  const int ntile = (g0.T + 127) / 128;
  const int per_layer = nparts * g0.H * ntile;
  const int64_t total = int64_t(per_layer) * a.num_layers;

  if (warp < kMmaWarp) {
    // ---------------------------------------------------------------- builders
    const int grp = warp >> 2, gt = tid & 127;
    float* kmn = reinterpret_cast<float*>(smem + kDwOffPar) + grp * 256;
    float* ksc = kmn + 128;
    int cur_layer = -1;
    int64_t n = grp;
    for (int64_t u = blockIdx.x + grp * int64_t(gridDim.x); u < total;
         u += kDwGroups * int64_t(gridDim.x), n += kDwGroups) {
      const int li = int(u / per_layer);
      int rem = int(u % per_layer);
      const int pi = rem / (g0.H * ntile);
      rem %= g0.H * ntile;
      const int j = rem / ntile, tt = rem % ntile;
      const int part = a.part_mask == 2 ? 1 : pi;
      const int layer = a.layer_begin + li;
      FrameGeom g = g0;
      if (a.n_lows != nullptr) {
        g.n_low = a.n_lows[layer];
        frame_geom_finalize(g);
      }
      const uint8_t* frame = a.frame_base + int64_t(li) * a.frame_stride;
      if (layer != cur_layer) {
        if (gt == 0) {
          int ok = s_bad == 0;
          if (ok && a.flags != nullptr && !wait_flag_geq(a.flags + layer, a.seq, a.timeout_ns)) {
            atomicCAS(a.status, 0u, uint32_t(kStatusTimeout));
            ok = 0;
          }
          if (ok) {
            const FrameHeader* hd = reinterpret_cast<const FrameHeader*>(frame);
            if (__ldcg(&hd->magic) != kFrameMagic || __ldcg(&hd->seq) != a.seq ||
                __ldcg(&hd->tokens) != uint32_t(g.T) || __ldcg(&hd->layer) != uint32_t(layer)) {
              atomicCAS(a.status, 0u, uint32_t(kStatusBadHeader));
              ok = 0;
            }
          }
          if (ok) asm volatile("fence.acq_rel.sys;" ::: "memory");
          else s_bad = 1;
          if (ok && a.trace != nullptr) trace_start(a.trace + 4 * layer + 2);
          s_ok[grp] = ok;
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory");
        cur_layer = layer;
      }
      const bool ok = s_ok[grp] != 0;
      const int stage = int(n % kDwStages);
      const uint32_t sphase = uint32_t(n / kDwStages) & 1u;
      // the stage is free once the MMA that read it retired (bounded wait)
      if (!mbar_wait(&empty[stage], sphase ^ 1u, a.status)) {
        if (gt == 0) s_bad = 1;
      }
      int s, js, hs;
      slot_section(g, j, s, js, hs);
      const int bits = gbits(g, part, s);
      const int64_t pay = gpayload(g, part, s) + 16;
      uint8_t* tile = smem + stage * kMmaTile;
      // every thread of the group is done reading the previous unit's K parameters
      asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory");
      if (ok && part == 0) {  // K parameters of slot j
        const bf16* kmin = reinterpret_cast<const bf16*>(frame + g.k_aux);
        const int64_t idx = int64_t(j) * D + gt;
        kmn[gt] = __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(kmin + idx))));
        ksc[gt] = __bfloat162float(__ushort_as_bfloat16(
            __ldcg(reinterpret_cast<const unsigned short*>(kmin + int64_t(g.H) * D + idx))));
      }
      asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory");
      const int t = tt * 128 + gt;
      if (ok && t < g.T) {
        float vmin = 0.f, vscl = 0.f;
        if (part == 1) {
          const bf16* vaux = reinterpret_cast<const bf16*>(frame + gvaux(g, s));
          vmin = __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(vaux + t))));
          vscl = __bfloat162float(
              __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(vaux + g.T + t))));
        }
        // the row's 128 symbols: 16 * bits contiguous bytes, 16-byte aligned
        const uint4* src = reinterpret_cast<const uint4*>(frame + pay + ((int64_t(t) * hs + js) * D) * bits / 8);
        uint32_t w[33];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (i < bits) {
            const uint4 x = __ldcg(src + i);
            w[4 * i] = x.x;
            w[4 * i + 1] = x.y;
            w[4 * i + 2] = x.z;
            w[4 * i + 3] = x.w;
          }
        }
        w[32] = 0;
        const bool pc = part == 0;
        switch (bits) {
          case 1: dw_unpack_row<1>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          case 2: dw_unpack_row<2>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          case 3: dw_unpack_row<3>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          case 4: dw_unpack_row<4>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          case 5: dw_unpack_row<5>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          case 6: dw_unpack_row<6>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          case 7: dw_unpack_row<7>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
          default: dw_unpack_row<8>(w, kmn, ksc, pc, vmin, vscl, tile, gt); break;
        }
      } else {
#pragma unroll
        for (int c16 = 0; c16 < 16; ++c16) *reinterpret_cast<uint4*>(tile + sw128_off(gt, c16)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      mbar_arrive(&full[stage]);
    }
  } else if (warp == kMmaWarp) {
    // -------------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, 128, false);
      const uint32_t h_s = smem_u32(smem + kDwOffH);
      bool okp = true;
      int64_t n = 0;
      for (int64_t u = blockIdx.x; u < total; u += gridDim.x, ++n) {
        const int stage = int(n % kDwStages), acc = int(n % kDwAcc);
        if (!mbar_wait(&tempty[acc], (uint32_t(n / kDwAcc) & 1u) ^ 1u, a.status)) { okp = false; break; }
        if (!mbar_wait(&full[stage], uint32_t(n / kDwStages) & 1u, a.status)) { okp = false; break; }
        tc_fence_after();
        const uint32_t a_s = smem_u32(smem + stage * kMmaTile);
        const uint32_t d = tmem_base + uint32_t(acc * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kMmaPanel + (kk & 3) * 32;
          umma_f16(d, smem_desc_sw128(a_s + off, 16, 1024), smem_desc_sw128(h_s + off, 16, 1024), idesc,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        umma_commit(&tfull[acc]);
      }
      if (!okp) {
        s_bad = 1;
        umma_commit(&tfull[kDwAcc]);
        mbar_wait(&tfull[kDwAcc], 0, nullptr);
      }
    }
  } else {
    // --------------------------------------------------------------- epilogue
    const int ew = warp - kMmaWarp - 1;        // 0 .. 4*kDwEpi-1
    const int grp = ew >> 2;
    const int quarter = warp & 3;              // TMEM lanes quarter*32 .. +31
    const int row = quarter * 32 + lane;
    const float scale = inv_sqrt_d<D>();
    const int bshift = (a.block_size & (a.block_size - 1)) == 0 ? __ffs(a.block_size) - 1 : -1;
    int64_t n = grp;
    for (int64_t u = blockIdx.x + grp * int64_t(gridDim.x); u < total;
         u += kDwEpi * int64_t(gridDim.x), n += kDwEpi) {
      const int acc = int(n % kDwAcc);
      const bool ready = mbar_wait(&tfull[acc], uint32_t(n / kDwAcc) & 1u, a.status);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int li = int(u / per_layer);
      int rem = int(u % per_layer);
      const int pi = rem / (g0.H * ntile);
      rem %= g0.H * ntile;
      const int j = rem / ntile, tt = rem % ntile;
      const int part = a.part_mask == 2 ? 1 : pi;
      const int layer = a.layer_begin + li;
      const int h = a.orders[int64_t(layer) * g0.H + j];
      const int t = tt * 128 + row;
      const uint32_t* sb = a.sign_bits + (int64_t(layer) * g0.H + h) * (D / 32);
      bf16* dst = nullptr;
      if (t < g0.T && s_bad == 0) {
        bf16* cache = a.layer_ptrs != nullptr
                          ? reinterpret_cast<bf16*>(a.layer_ptrs[2 * layer + part])
                          : a.cache + int64_t(layer) * a.layer_stride + int64_t(part) * a.part_stride;
        int bi, bo;
        split_pos(a.tok_offset + t, a.block_size, bshift, bi, bo);
        dst = cache + int64_t(a.block_table[bi]) * a.block_stride + int64_t(bo) * a.token_stride +
              int64_t(h) * a.head_stride;
      }
      const uint32_t trow = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * 128);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + uint32_t(c * 32), r);
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
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (quarter == 0 && lane == 0 && dst != nullptr && a.trace != nullptr) trace_end(a.trace + 4 * layer + 3);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc<512>(tmem_base);
  }
}

}  // namespace
}  // namespace kvs
