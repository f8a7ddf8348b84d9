// Causal GQA prefill flash attention on tcgen05 tensor cores (head_dim 128).
//
// One CTA per SM holds two 128-row query tiles of one head (a "pair") and
// streams the pair's K/V tiles; pairs are launched heaviest-first.  K tiles
// go through a ring of 2 (default) or 3 stages, V tiles through 2.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cstdlib>

#include "common.cuh"
#include "ops.h"
#include "sm100.cuh"

namespace kvs {
namespace {

constexpr int D = 128;
constexpr int BQ = 128, BKV = 128;
constexpr int PANEL = 128 * 128;          // bytes: 128 rows x 64 bf16
constexpr int TILE = 2 * PANEL;           // 32 KB: 128 rows x 128 bf16
constexpr float kRescaleThreshold = 8.0f;

struct AttnArgs {
  bf16* out;
  int64_t ldo;
  int T, Hq, Hkv;
  float scale_log2;
  uint32_t* err;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// Two query tiles per CTA in ping-pong (one CTA per SM).
//   warps 0..3  softmax of query tile 0 (rows q0 .. q0+127)
//   warps 4..7  softmax of query tile 1 (rows q0+128 .. q0+255)
//   warp 8      TMA producer (Q0, Q1; K and V double buffered)
//   warp 9      MMA issuer
// TMEM (512 columns): S0/P0 | S1/P1 | O0 | O1.  The MMA issue order
//   S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ...
// keeps the tensor pipe on one tile while the other tile's softmax runs.
// A commit after S_i(j+1) also covers PV_i(j), so when a softmax group sees
// its next S tile, its O accumulator is quiescent and may be rescaled in
// place.  The softmax keeps the whole S row in registers (one TMEM pass),
// uses packed f32x2 FMA/ADD, a 3-input max; a compile-time mask can move a
// fixed subset of the exponentials to a cubic on the FMA pipes (off by
// default: the MUFU is not the bottleneck).
// ---------------------------------------------------------------------------
namespace v3 {
constexpr int kThreads = 320;
constexpr int OFF_Q0 = 0;
constexpr int OFF_Q1 = TILE;
constexpr int OFF_K = 2 * TILE;  // KS stages of K, then 2 of V
template <int KS>
struct Layout {
  static constexpr int OFF_V = (2 + KS) * TILE;
  static constexpr int OFF_BAR = (4 + KS) * TILE;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[2], v_empty[2],
  // s_full[2], p_full[2], o_done[2], drain; then the TMEM address
  static constexpr int B_KFULL = 1, B_KEMPTY = 1 + KS, B_VFULL = 1 + 2 * KS, B_VEMPTY = 3 + 2 * KS,
                       B_SFULL = 5 + 2 * KS, B_PFULL = 7 + 2 * KS, B_ODONE = 9 + 2 * KS, B_DRAIN = 11 + 2 * KS,
                       NUM_BARS = 12 + 2 * KS;
};
static_assert(Layout<3>::SMEM_BYTES <= 232448, "3 K stages must fit in shared memory");
constexpr uint32_t kTmemCols = 512;
// Of every 16 consecutive key columns (8 pairs), pairs whose bit is set in
// the kernel's POLY mask take the polynomial exponential on the FMA pipes.
// Measured at T = 8192 (TFLOP/s): none 1130, 2 of 8 pairs 1080, 4 of 8 906,
// all 563 — the softmax is bound by its issue slots, not by the MUFU, so
// the default evaluates every exponential with ex2.approx.
constexpr uint32_t kPolyPairs = 0x00u;

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x on the FMA pipes: 2^x = 2^n * 2^f with n = round(x) (1.5 * 2^23
// rounding trick), f in [-0.5, 0.5]; 2^f by a cubic whose coefficients were
// fitted for this kernel by relative-error-weighted least squares on
// [-0.5, 0.5] (max relative error 8e-5, far below the bf16 rounding of P).
// Arguments are clamped below at -120 so the exponent never underflows.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -120.0f);
  const float t = x + 12582912.0f;
  const float n = t - 12582912.0f;
  const float f = x - n;
  float p = fmaf(f, 0.05516014f, 0.24258275f);
  p = fmaf(f, p, 0.69326055f);
  p = fmaf(f, p, 0.99993020f);
  const int e = __float_as_int(t) - 0x4B400000;
  return __int_as_float(__float_as_int(p) + (e << 23));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}
// (d0, d1) = (a0, a1) * b + (c, c) in one packed instruction.
__device__ __forceinline__ void fma2s(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{.reg .b64 ra, rb, rc, rd;\n"
      "mov.b64 ra, {%2,%3};\n"
      "mov.b64 rb, {%4,%4};\n"
      "mov.b64 rc, {%5,%5};\n"
      "fma.rn.f32x2 rd, ra, rb, rc;\n"
      "mov.b64 {%0,%1}, rd;}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
__device__ __forceinline__ void add2(float& s0, float& s1, float a0, float a1) {
  asm("{.reg .b64 ra, rb, rd;\n"
      "mov.b64 ra, {%0,%1};\n"
      "mov.b64 rb, {%2,%3};\n"
      "add.rn.f32x2 rd, ra, rb;\n"
      "mov.b64 {%0,%1}, rd;}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}
}  // namespace v3

// TMA producer of both flash kernels (one thread): Q0, Q1, then K and V of
// each KV tile into two-stage rings.
template <int KS>
__device__ __forceinline__ void flash_produce(uint8_t* smem, const CUtensorMap* tmp, const AttnArgs& a, int h,
                                              int kvh, int q0, int n1, uint64_t* q_full, uint64_t* k_full,
                                              uint64_t* k_empty, uint64_t* v_full, uint64_t* v_empty) {
  using namespace sm100;
  const CUtensorMap& tm = *tmp;
  const int xq = h * D, xk = (a.Hq + kvh) * D, xv = (a.Hq + a.Hkv + kvh) * D;
  mbar_arrive_expect_tx(q_full, 2 * TILE);
  tma_load_2d(smem + v3::OFF_Q0, &tm, xq, q0, q_full);
  tma_load_2d(smem + v3::OFF_Q0 + PANEL, &tm, xq + 64, q0, q_full);
  tma_load_2d(smem + v3::OFF_Q1, &tm, xq, q0 + BQ, q_full);
  tma_load_2d(smem + v3::OFF_Q1 + PANEL, &tm, xq + 64, q0 + BQ, q_full);
  int kdone = -1, vdone = -1;
  for (int j = 0; j < n1; ++j) {
    const int ks = j % KS, vs = j & 1;
    const uint32_t kph = (j / KS) & 1, vph = (j >> 1) & 1;
    const int k0 = j * BKV;
    if (!mbar_wait(&k_empty[ks], kph ^ 1, a.err)) break;
    mbar_arrive_expect_tx(&k_full[ks], TILE);
    tma_load_2d(smem + v3::OFF_K + ks * TILE, &tm, xk, k0, &k_full[ks]);
    tma_load_2d(smem + v3::OFF_K + ks * TILE + PANEL, &tm, xk + 64, k0, &k_full[ks]);
    kdone = j;
    if (!mbar_wait(&v_empty[vs], vph ^ 1, a.err)) break;
    mbar_arrive_expect_tx(&v_full[vs], TILE);
    tma_load_2d(smem + v3::Layout<KS>::OFF_V + vs * TILE, &tm, xv, k0, &v_full[vs]);
    tma_load_2d(smem + v3::Layout<KS>::OFF_V + vs * TILE + PANEL, &tm, xv + 64, k0, &v_full[vs]);
    vdone = j;
  }
  // every issued copy lands before the CTA may exit (the last use of each
  // stage is the newest phase of its barrier)
  mbar_wait(q_full, 0, nullptr);
  for (int j = (kdone >= KS ? kdone - KS + 1 : 0); j <= kdone; ++j) mbar_wait(&k_full[j % KS], (j / KS) & 1, nullptr);
  for (int j = (vdone > 0 ? vdone - 1 : 0); j <= vdone; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr);
}

// MMA issuer of both flash kernels (one thread): S_i = Q_i K^T into TMEM and
// O_i += P_i V with P read from TMEM, in the ping-pong order described above.
template <int KS>
__device__ __forceinline__ void flash_mma(uint8_t* smem, const AttnArgs& a, uint32_t tmem, int n0, int n1,
                                          uint64_t* q_full, uint64_t* k_full, uint64_t* k_empty, uint64_t* v_full,
                                          uint64_t* v_empty, uint64_t* s_full, uint64_t* p_full, uint64_t* o_done,
                                          uint64_t* drain) {
  using namespace sm100;
  constexpr uint32_t idesc_qk = idesc_bf16(BQ, BKV, false);
  constexpr uint32_t idesc_pv = idesc_bf16(BQ, D, true);
  const uint32_t q0a = smem_u32(smem + v3::OFF_Q0), q1a = smem_u32(smem + v3::OFF_Q1);
  const uint32_t kb0 = smem_u32(smem + v3::OFF_K), vb0 = smem_u32(smem + v3::Layout<KS>::OFF_V);
  auto qk = [&](uint32_t dst, uint32_t qa, int j) {
    const uint32_t kb = kb0 + (j % KS) * TILE;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * PANEL + (kk & 3) * 32;
      umma_f16(dst, smem_desc_sw128(qa + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc_qk,
               kk > 0 ? 1u : 0u);
    }
  };
  auto pv = [&](uint32_t dst, uint32_t p_tmem, int j) {
    const uint32_t vb = vb0 + (j & 1) * TILE;
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk)
      umma_f16_ta(dst, p_tmem + kk * 8, smem_desc_sw128(vb + kk * 2048, PANEL, 1024), idesc_pv,
                  (j > 0 || kk > 0) ? 1u : 0u);
  };
  const uint32_t tS0 = tmem, tS1 = tmem + 128, tO0 = tmem + 256, tO1 = tmem + 384;
  bool ok = mbar_wait(q_full, 0, a.err) && mbar_wait(&k_full[0], 0, a.err);
  if (ok) {
    tc_fence_after();
    qk(tS0, q0a, 0);
    umma_commit(&s_full[0]);
    qk(tS1, q1a, 0);
    umma_commit(&s_full[1]);
    umma_commit(&k_empty[0]);
  }
  for (int j = 0; j < n1 && ok; ++j) {
    const int st = j & 1;
    const uint32_t par = j & 1;
    if (!mbar_wait(&v_full[st], (j >> 1) & 1, a.err)) { ok = false; break; }
    bool k_next_ready = false;
    if (j < n0) {
      if (!mbar_wait(&p_full[0], par, a.err)) { ok = false; break; }
      tc_fence_after();
      pv(tO0, tS0, j);
      if (j == n0 - 1) umma_commit(&o_done[0]);
      if (j + 1 < n0) {
        if (!mbar_wait(&k_full[(j + 1) % KS], ((j + 1) / KS) & 1, a.err)) { ok = false; break; }
        k_next_ready = true;
        tc_fence_after();
        qk(tS0, q0a, j + 1);
        umma_commit(&s_full[0]);
      }
    }
    if (!mbar_wait(&p_full[1], par, a.err)) { ok = false; break; }
    tc_fence_after();
    pv(tO1, tS1, j);
    umma_commit(&v_empty[st]);
    if (j == n1 - 1) umma_commit(&o_done[1]);
    if (j + 1 < n1) {
      if (!k_next_ready && !mbar_wait(&k_full[(j + 1) % KS], ((j + 1) / KS) & 1, a.err)) { ok = false; break; }
      tc_fence_after();
      qk(tS1, q1a, j + 1);
      umma_commit(&s_full[1]);
      umma_commit(&k_empty[(j + 1) % KS]);
    }
  }
  umma_commit(drain);
  mbar_wait(drain, 0, nullptr);
}


template <int KS, uint32_t POLY>
__global__ void __launch_bounds__(v3::kThreads, 1)
    flash_prefill_v3_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  using Lay = v3::Layout<KS>;
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Lay::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + Lay::B_KFULL;     // [KS]
  uint64_t* k_empty = bars + Lay::B_KEMPTY;   // [KS]
  uint64_t* v_full = bars + Lay::B_VFULL;     // [2]
  uint64_t* v_empty = bars + Lay::B_VEMPTY;   // [2]
  uint64_t* s_full = bars + Lay::B_SFULL;     // [2] per query tile
  uint64_t* p_full = bars + Lay::B_PFULL;     // [2] per query tile (128 arrivals)
  uint64_t* o_done = bars + Lay::B_ODONE;     // [2] per query tile
  uint64_t* drain = bars + Lay::B_DRAIN;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Lay::NUM_BARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int npairs = (a.T + 2 * BQ - 1) / (2 * BQ);
  const int pair = npairs - 1 - int(blockIdx.y);
  const int q0 = pair * 2 * BQ;
  const int kvh = h / (a.Hq / a.Hkv);
  const int n0 = q0 / BKV + 1;  // KV tiles seen by query tile 0
  const int n1 = n0 + 1;        // ... and by query tile 1

  if (threadIdx.x == 0) {
    for (int i = 0; i < Lay::NUM_BARS; ++i)
      mbar_init(&bars[i], (i == Lay::B_PFULL || i == Lay::B_PFULL + 1) ? 128 : 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 9) tmem_alloc<v3::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) flash_produce<KS>(smem, &tm, a, h, kvh, q0, n1, q_full, k_full, k_empty, v_full, v_empty);
  } else if (warp == 9) {
    if (lane == 0) flash_mma<KS>(smem, a, tmem, n0, n1, q_full, k_full, k_empty, v_full, v_empty, s_full, p_full,
                                 o_done, drain);
  } else {
    const int wg = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + wg * 128, tO = tmem + 256 + wg * 128;
    const int qrow0 = q0 + wg * BQ;
    const int q_abs = qrow0 + row;
    const int nkv = qrow0 / BKV + 1;
    const float sl2 = a.scale_log2;
    float m_ref = -INFINITY, l0 = 0.f, l1 = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const bool diag = (j == nkv - 1);
      if (!mbar_wait(&s_full[wg], j & 1, a.err)) ok = false;
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, r[c]);
      tmem_wait_ld();
      if (diag) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (c * 32 + e > row) r[c][e] = __float_as_uint(-INFINITY);
      }
      // row max as 8 independent 3-input-max chains (a single chain of 64
      // dependent max3 put its latency on every tile's critical path)
      float mxa[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxa[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 2)
          mxa[c * 2 + (e >> 4)] = v3::max3(mxa[c * 2 + (e >> 4)], __uint_as_float(r[c][e]),
                                           __uint_as_float(r[c][e + 1]));
      const float mx = fmaxf(v3::max3(mxa[0], mxa[1], mxa[2]), v3::max3(mxa[3], mxa[4], v3::max3(mxa[5], mxa[6],
                                                                                                 mxa[7])));
      const float mxs = mx * sl2;
      const bool rescale = mxs > m_ref + kRescaleThreshold;
      const float m_use = rescale ? mxs : m_ref;
      const float neg_m = -m_use;
      // row sum: one packed accumulator pair per 32-key chunk (independent chains)
      float sa[4][2];
#pragma unroll
      for (int c = 0; c < 4; ++c) sa[c][0] = sa[c][1] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float x0, x1;
          v3::fma2s(x0, x1, __uint_as_float(r[c][2 * e]), __uint_as_float(r[c][2 * e + 1]), sl2, neg_m);
          float p0, p1;
          if ((POLY >> (e & 7)) & 1u) {
            p0 = v3::ex2_poly(x0);
            p1 = v3::ex2_poly(x1);
            if (diag) {  // the polynomial does not map -inf to 0
              if (c * 32 + 2 * e > row) p0 = 0.f;
              if (c * 32 + 2 * e + 1 > row) p1 = 0.f;
            }
          } else {
            p0 = v3::ex2_mufu(x0);
            p1 = v3::ex2_mufu(x1);
          }
          v3::add2(sa[c][0], sa[c][1], p0, p1);
          pk[e] = pack_bf16x2(p0, p1);
        }
        // P chunk c (keys 32c .. 32c+31) -> columns [16c, 16c+16) of S; the
        // whole S row is already in registers.
        tmem_st16(tS + lane_off + c * 16, pk);
      }
      const float s0 = (sa[0][0] + sa[1][0]) + (sa[2][0] + sa[3][0]);
      const float s1 = (sa[0][1] + sa[1][1]) + (sa[2][1] + sa[3][1]);
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? v3::ex2_mufu(m_ref - m_use) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + lane_off + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(tO + lane_off + c * 32, o);
        }
        l0 *= f;
        l1 *= f;
      }
      tmem_wait_st();
      if (rescale) m_ref = m_use;
      l0 += s0;
      l1 += s1;
      tc_fence_before();
      mbar_arrive(&p_full[wg]);
    }
    if (ok) {
      const bool done = mbar_wait(&o_done[wg], 0, a.err);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        const float l = l0 + l1;
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        bf16* orow = a.out + int64_t(q_abs) * a.ldo + int64_t(h) * D;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + lane_off + c * 32, o);
          tmem_wait_ld();
          if (q_abs < a.T) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
              w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
              w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
              w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = w;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc<v3::kTmemCols>(tmem);
  }
}


}  // namespace

// K-tile stages of the kernel: 2 (default) or 3 (KVSERVE_FLASH_KSTAGES=3;
// measured equal at T=8192, so the smaller ring stays the default);
// `kstages` 0 takes that default.
static int flash_default_kstages() {
  static const int v = [] {
    const char* e = std::getenv("KVSERVE_FLASH_KSTAGES");
    return (e && e[0] == '3') ? 3 : 2;
  }();
  return v;
}

void flash_prefill(torch::Tensor qkv, int64_t Hq, int64_t Hkv, double scale, torch::Tensor out, torch::Tensor err,
                   int64_t kstages, int64_t poly) {
  KVS_CHECK_ARG(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.stride(1) == 1,
                "flash_prefill: qkv [T, (Hq+2Hkv)*128] bf16");
  KVS_CHECK_ARG(qkv.size(1) == (Hq + 2 * Hkv) * D && Hq % Hkv == 0, "flash_prefill: head_dim 128 only");
  KVS_CHECK_ARG(out.dim() == 2 && out.size(0) == qkv.size(0) && out.size(1) == Hq * D && out.stride(1) == 1 &&
                    out.stride(0) % 8 == 0,
                "flash_prefill: out [T, Hq*128]");
  const int T = int(qkv.size(0));
  if (T == 0) return;
  AttnArgs a{};
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.T = T;
  a.Hq = int(Hq);
  a.Hkv = int(Hkv);
  a.scale_log2 = float(scale) * 1.4426950408889634f;
  a.err = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  const CUtensorMap tm =
      make_tmap_2d_bf16(qkv.data_ptr(), uint64_t(qkv.size(1)), uint64_t(T), uint64_t(qkv.stride(0)) * 2, 64, 128);
  if (kstages == 0) kstages = flash_default_kstages();
  if (poly == 0) poly = 0x100;   // default mix: no polynomial exponentials
  KVS_CHECK_ARG(kstages == 2 || kstages == 3, "flash_prefill: K-tile stages must be 2 or 3");
  KVS_CHECK_ARG(kstages == 2 || poly == 0x100, "flash_prefill: 3 K stages use the default exponential mix");
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  dim3 grid(int(Hq), (T + 2 * BQ - 1) / (2 * BQ));
#define KVS_FLASH_LAUNCH(KS, PM)                                                                                 \
  {                                                                                                            \
    static bool set = false;                                                                                   \
    if (!set) {                                                                                                \
      KVS_CUDA_CHECK(cudaFuncSetAttribute(flash_prefill_v3_kernel<KS, PM>,                                     \
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, v3::Layout<KS>::SMEM_BYTES)); \
      set = true;                                                                                              \
    }                                                                                                          \
    flash_prefill_v3_kernel<KS, PM><<<grid, v3::kThreads, v3::Layout<KS>::SMEM_BYTES, st>>>(tm, a);            \
  }
  if (kstages == 3) KVS_FLASH_LAUNCH(3, 0x00u)
  else if (poly == 0x11) KVS_FLASH_LAUNCH(2, 0x11u)
  else if (poly == 0x100) KVS_FLASH_LAUNCH(2, 0x00u)
  else if (poly == 0x55) KVS_FLASH_LAUNCH(2, 0x55u)
  else if (poly == 0xFF) KVS_FLASH_LAUNCH(2, 0xFFu)
  else KVS_CHECK_ARG(false, "flash_prefill: polynomial-exponential mask must be 0x11, 0x55, 0xFF or 0x100 (none)");
#undef KVS_FLASH_LAUNCH
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
