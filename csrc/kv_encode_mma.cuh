// Frame encode with the random-sign Hadamard transform on the tensor cores
// (head_dim 128, contiguous [T, H, D] K/V, quantised sections).  Included by
// kv_codec.cu after the frame helpers, EncodeArgs, encode_signal_done and the
// MMA decoder (whose SW128 tile constants it shares).
//
// The random signs are folded into the transform matrix: for every (layer,
// head) M[o][i] = H[o][i] * s[i] (H the +-1 Sylvester matrix), built once
// into a bf16 table.  The transformed row of token t is then X[t] M^T, and
// the same M is the B operand of (X M^T) and the A operand of (M X^T).
//
// Work unit = (part, head slot j, 128-token tile).  One persistent,
// warp-specialised CTA per SM (320 threads) takes a contiguous range of
// units (consecutive units mostly share a head):
//   warp 0     TMA producer: per unit the X tile (two 64-column SW128 boxes
//              of the K or V rows of head order[j]; rows past T are zero
//              filled) into a 3-stage ring, and M of the head into one of
//              two M buffers only when the head changes;
//   warp 1     MMA issuer: eight tcgen05.mma (K = 16 each) into one of four
//              128-column TMEM accumulators (all 512 columns);
//   warps 2-9  two epilogue warpgroups taking alternate units, so two
//              epilogues run while the next units load and multiply.
// kv_encode_ws_kernel<true> (statistics): K units compute M X^T (TMEM lane =
// channel: per-channel min/max over the tile's tokens is a register
// reduction); V units compute X M^T (lane = token); both end in
// ordered-integer atomics on the layer's statistics (K: [2][H*D], V:
// [2 sections][2][T]).  kv_encode_ws_kernel<false> (quantise): X M^T for
// every unit, quantised with the per-channel (K) or per-token (V) bf16
// parameters derived from the statistics, packed LSB-first and stored into
// the frame (local or a peer's receive slot); the last CTA writes the
// header, resets the statistics and publishes.
// Products with +-1 are exact and sums are fp32, so the transformed values
// equal the register butterfly's up to fp32 summation order.
#pragma once
#include "sm100.cuh"

namespace kvs {
namespace {

constexpr int kWsEpiGroups = 2;                        // epilogue warpgroups (alternate units)
constexpr int kWsAcc = 4;                              // 128-column TMEM accumulators
constexpr int kWsThreads = 64 + 128 * kWsEpiGroups;
constexpr int kWsStages = 3;                           // ring of X tiles (32 KB each)
constexpr int kWsStage = kMmaTile;
constexpr int kWsOffM = kWsStages * kWsStage;          // two 32 KB buffers of a head's signed transform M
constexpr int kEncMaxHD = 8 * 128;
constexpr int kWsOffPar = kWsOffM + 2 * kMmaTile;      // K params: min[H*D], inv[H*D] fp32
constexpr int kWsStgWarp = 32 * (128 + 16);            // per epilogue warp: 32 packed rows of <= 128 bytes,
                                                       // each padded by 16 bytes (spreads the bank groups)
constexpr int kWsOffStg = kWsOffPar + 2 * kEncMaxHD * 4;
constexpr int kWsOffBar = kWsOffStg + 4 * kWsEpiGroups * kWsStgWarp;
constexpr int kWsSmem = kWsOffBar + 256 + 1024;
static_assert(kWsAcc % kWsEpiGroups == 0, "each warpgroup keeps its own accumulators");

struct EncUnit {
  int part, j, tile;
};

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

// Signed transform table: rows (h * 128 + o), columns i: H[o][i] * s_h[i].
__global__ void kv_signed_hadamard_kernel(const uint32_t* __restrict__ sign_bits, int heads,
                                          bf16* __restrict__ out) {
  const int64_t n = int64_t(heads) * 128 * 128;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int col = int(i & 127), o = int((i >> 7) & 127);
    const int h = int(i >> 14);
    const bool neg = ((__popc(o & col) & 1) != 0) ^ (((sign_bits[h * 4 + (col >> 5)] >> (col & 31)) & 1u) != 0);
    out[i] = __ushort_as_bfloat16(neg ? 0xBF80u : 0x3F80u);
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


template <bool kStats>
__global__ void __launch_bounds__(kWsThreads, 1)
    kv_encode_ws_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmM, EncodeArgs a, int m_head0) {
  using namespace sm100;
  constexpr int D = 128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* kmin = reinterpret_cast<float*>(smem + kWsOffPar);
  float* kinv = kmin + kEncMaxHD;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kWsOffBar);
  uint64_t* empty = full + kWsStages;
  uint64_t* mfull = empty + kWsStages;   // [2] M buffer loaded
  uint64_t* mempty = mfull + 2;          // [2] M buffer free (its MMAs retired)
  uint64_t* tfull = mempty + 2;          // [0, kWsAcc): accumulator ready; [kWsAcc]: abort drain
  uint64_t* tempty = tfull + kWsAcc + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + kWsAcc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0 && a.trace != nullptr) trace_start(a.trace);
  const FrameGeom& g = a.g;
  const int HD = g.H * D;
  const int ntile = (g.T + 127) / 128;
  const int64_t total = int64_t(a.part_mask == 3 ? 2 : 1) * g.H * ntile;
  // a contiguous range of units per CTA: consecutive units mostly share a
  // head, so its transform matrix is loaded once for several tiles
  const int64_t u_begin = total * blockIdx.x / gridDim.x, u_end = total * (blockIdx.x + 1) / gridDim.x;
  if (!kStats) {
    // K parameters of every slot (block 0 also writes them and the section
    // headers into the frame)
    if (a.part_mask & 1) {
      bf16* fmin = reinterpret_cast<bf16*>(a.frame + g.k_aux);
      bf16* fscl = fmin + HD;
      for (int c = tid; c < HD; c += kWsThreads) {
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
  }
  if (tid == 0) {
    for (int s = 0; s < kWsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&mfull[b], 1);
      mbar_init(&mempty[b], 1);
    }
    for (int b = 0; b < kWsAcc; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(&tfull[kWsAcc], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmM);
  }
  if (warp == 1) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0, prev_h = -1;
      uint32_t phase = 0, mloads = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int64_t u = u_begin; u < u_end; ++u) {
        const EncUnit e = enc_unit(u, g.H, ntile, a.part_mask);
        const int h = a.order[e.j];
        if (h != prev_h) {   // the head's signed transform into the next M buffer
          const int mb = int(mloads & 1u);
          if (!mbar_wait(&mempty[mb], ((mloads >> 1) & 1u) ^ 1u, a.counter + 1)) { ok = false; break; }
          uint8_t* mdst = smem + kWsOffM + mb * kMmaTile;
          mbar_arrive_expect_tx(&mfull[mb], kMmaTile);
          tma_load_2d(mdst, &tmM, 0, (m_head0 + h) * 128, &mfull[mb]);
          tma_load_2d(mdst + kMmaPanel, &tmM, 64, (m_head0 + h) * 128, &mfull[mb]);
          ++mloads;
          prev_h = h;
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, a.counter + 1)) { ok = false; break; }
        uint8_t* st = smem + stage * kWsStage;
        mbar_arrive_expect_tx(&full[stage], kWsStage);
        const CUtensorMap* tx = e.part ? &tmV : &tmK;
        tma_load_2d(st, tx, h * D, e.tile * 128, &full[stage]);
        tma_load_2d(st + kMmaPanel, tx, h * D + 64, e.tile * 128, &full[stage]);
        issued_mask |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kWsStages) { stage = 0; phase ^= 1; }
      }
      if (!ok) {  // every issued copy lands before the CTA may exit
        for (int i = 0; i < kWsStages; ++i)
          if (issued_mask & (1u << i)) mbar_wait(&full[i], (issued_parity >> i) & 1u, nullptr);
        for (uint32_t k = (mloads > 2 ? mloads - 2 : 0); k < mloads; ++k)
          mbar_wait(&mfull[k & 1u], (k >> 1) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(128, 128, false);
      int stage = 0, acc = 0, prev_h = -1, mb = 0;
      uint32_t phase = 0, acc_phase = 0, mloads = 0;
      bool ok = true;
      for (int64_t u = u_begin; u < u_end; ++u) {
        const EncUnit e = enc_unit(u, g.H, ntile, a.part_mask);
        const int h = a.order[e.j];
        if (h != prev_h) {
          // the previous head's M buffer is free once its MMAs retire
          if (prev_h >= 0) umma_commit(&mempty[mb]);
          mb = int(mloads & 1u);
          if (!mbar_wait(&mfull[mb], (mloads >> 1) & 1u, a.counter + 1)) { ok = false; break; }
          ++mloads;
          prev_h = h;
        }
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, a.counter + 1)) { ok = false; break; }
        if (!mbar_wait(&full[stage], phase, a.counter + 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t x_s = smem_u32(smem + stage * kWsStage), m_s = smem_u32(smem + kWsOffM + mb * kMmaTile);
        // statistics of K: M X^T (lane = channel); everything else X M^T (lane = token)
        const bool chan = kStats && e.part == 0;
        const uint32_t a_s = chan ? m_s : x_s, b_s = chan ? x_s : m_s;
        const uint32_t d = tmem_base + uint32_t(acc * 128);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kMmaPanel + (kk & 3) * 32;
          umma_f16(d, smem_desc_sw128(a_s + off, 16, 1024), smem_desc_sw128(b_s + off, 16, 1024), idesc,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(&empty[stage]);
        umma_commit(&tfull[acc]);
        if (++stage == kWsStages) { stage = 0; phase ^= 1; }
        if (++acc == kWsAcc) { acc = 0; acc_phase ^= 1; }
      }
      if (!ok) {  // every issued MMA retires before TMEM is freed
        umma_commit(&tfull[kWsAcc]);
        mbar_wait(&tfull[kWsAcc], 0, nullptr);
      }
    }
  } else {
    const int quarter = warp & 3;          // TMEM lanes quarter*32 .. +31
    const int r = quarter * 32 + lane;     // token (or channel) of this thread
    const int grp = (warp - 2) >> 2;       // this warpgroup takes local units grp, grp + 2, ...
    const float scale = inv_sqrt_d<D>();
    int64_t n = grp;
    for (int64_t u = u_begin + grp; u < u_end; u += kWsEpiGroups, n += kWsEpiGroups) {
      const EncUnit e = enc_unit(u, g.H, ntile, a.part_mask);
      const int acc = int(n % kWsAcc);
      const uint32_t acc_phase = uint32_t(n / kWsAcc) & 1u;
      const bool ready = mbar_wait(&tfull[acc], acc_phase, a.counter + 1);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * 128);
      const int t0 = e.tile * 128;
      const int nvalid = min(128, g.T - t0);
      int s, js, hs;
      slot_section(g, e.j, s, js, hs);
      if (kStats) {
        float lo = INFINITY, hi = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(trow + uint32_t(c * 32), v);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 32; ++q)
            if (e.part != 0 || c * 32 + q < nvalid) {
              lo = fminf(lo, __uint_as_float(v[q]));
              hi = fmaxf(hi, __uint_as_float(v[q]));
            }
        }
        if (e.part == 0) {
          const int c = e.j * D + r;  // lane = channel
          atomicMin(&a.stats[c], float_to_ordered(lo * scale));
          atomicMax(&a.stats[HD + c], float_to_ordered(hi * scale));
        } else if (r < nvalid) {
          uint32_t* vs = a.stats + 2 * HD + int64_t(s) * 2 * g.T;
          atomicMin(&vs[t0 + r], float_to_ordered(lo * scale));
          atomicMax(&vs[g.T + t0 + r], float_to_ordered(hi * scale));
        }
      } else {
        const int bits = gbits(g, e.part, s);
        const float top = float(glevels(g, e.part, s) - 1);
        const int t = t0 + r;
        const bool valid = r < nvalid;
        float vmn = 0.f, vinv = 0.f;
        if (e.part == 1 && valid) {
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
        uint8_t* rows = a.frame + gpayload(g, e.part, s) + 16;   // row of token t at (t*hs + js) * 16*bits
        const int64_t row_stride = int64_t(hs) * 16 * bits;
        const int64_t row0 = (int64_t(t0) * hs + js) * 16 * bits;
        // power-of-two widths: the warp's 32 packed rows go through shared
        // memory so that each store instruction writes whole row pieces
        // (16*bits contiguous bytes) instead of 16 bytes of 32 rows -- the
        // frame is often a peer GPU's memory, where small writes waste NVLink
        const bool staged = (bits & (bits - 1)) == 0;
        uint32_t* stg = reinterpret_cast<uint32_t*>(smem + kWsOffStg + (warp - 2) * kWsStgWarp) + lane * 4 * (bits + 1);
        uint32_t* dst = reinterpret_cast<uint32_t*>(rows + row0 + int64_t(r) * row_stride);
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(trow + uint32_t(c * 32), v);
          tmem_wait_ld();
          uint32_t q[32];
          if (e.part == 0) {
            const float* mn = kmin + e.j * D + c * 32;
            const float* iv = kinv + e.j * D + c * 32;
#pragma unroll
            for (int x = 0; x < 32; ++x) {
              const float y = rintf((__uint_as_float(v[x]) * scale - mn[x]) * iv[x]);
              q[x] = uint32_t(fminf(fmaxf(y, 0.0f), top));
            }
          } else {
#pragma unroll
            for (int x = 0; x < 32; ++x) {
              const float y = rintf((__uint_as_float(v[x]) * scale - vmn) * vinv);
              q[x] = uint32_t(fminf(fmaxf(y, 0.0f), top));
            }
          }
          if (staged) pack32_any(q, stg + c * bits, bits);
          else if (valid) pack32_any(q, dst + c * bits, bits);
        }
        if (staged) {
          __syncwarp();
          // row pieces of 16*bits bytes = bits 16-byte chunks; 32/bits rows per instruction
          const uint4* sp = reinterpret_cast<const uint4*>(smem + kWsOffStg + (warp - 2) * kWsStgWarp);
          const int rows_per = 32 / bits;
          for (int i = 0; i < bits; ++i) {
            const int rr = i * rows_per + lane / bits, ck = lane % bits;
            if (t0 + quarter * 32 + rr < g.T) {
              const uint4 val = sp[rr * (bits + 1) + ck];
              *reinterpret_cast<uint4*>(rows + row0 + int64_t(quarter * 32 + rr) * row_stride + ck * 16) = val;
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<512>(tmem_base);
  }
  if (!kStats) encode_signal_done(a);
}

}  // namespace
}  // namespace kvs
