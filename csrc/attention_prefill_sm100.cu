// Causal GQA prefill flash attention on tcgen05 tensor cores (head_dim 128).
//
// One CTA per (query tile of 128 rows, query head); tiles are launched
// heaviest-first.  Warp roles (192 threads):
//   warps 0..3  softmax + epilogue: thread = one query row = one TMEM lane.
//   warp 4      TMA producer: Q (2 x 64-col swizzled panels), K/V double
//               buffered straight out of the fused QKV activation.
//   warp 5      MMA issuer: S = Q K^T into a double-buffered TMEM S tile,
//               O += P V with P (bf16, swizzled K-major) written by the
//               softmax warps into shared memory and V used as an MN-major
//               operand; O accumulates in TMEM.
// Online softmax with lazy rescaling: the reference max of a row only moves
// when the new max exceeds it by more than 2^8, so O (in TMEM) is rarely
// rescaled; exp2 arguments are bounded by 8 so p <= 256 stays exact enough.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "ops.h"
#include "sm100.cuh"

#include <cstdlib>

namespace kvs {
namespace {

constexpr int D = 128;
constexpr int BQ = 128, BKV = 128;
constexpr int PANEL = 128 * 128;          // bytes: 128 rows x 64 bf16
constexpr int TILE = 2 * PANEL;           // 32 KB: 128 rows x 128 bf16
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE;       // 2 stages
constexpr int OFF_V = OFF_K + 2 * TILE;   // 2 stages
constexpr int OFF_P = OFF_V + 2 * TILE;   // 2 buffers
constexpr int OFF_BAR = OFF_P + 2 * TILE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;       // S0 | S1 | O | (unused)
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

__global__ void __launch_bounds__(kThreads, 1)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars;        // 1
  uint64_t* k_full = bars + 1;    // 2
  uint64_t* v_full = bars + 3;    // 2
  uint64_t* kv_empty = bars + 5;  // 2
  uint64_t* s_full = bars + 7;    // 2
  uint64_t* s_empty = bars + 9;   // 2
  uint64_t* p_full = bars + 11;   // 2
  uint64_t* pv_done = bars + 13;  // 2
  uint64_t* drain = bars + 15;    // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int ntiles = (a.T + BQ - 1) / BQ;
  const int qt = ntiles - 1 - int(blockIdx.y);
  const int q0 = qt * BQ;
  const int kvh = h / (a.Hq / a.Hkv);
  const int nkv = qt + 1;  // causal: key tiles 0..qt

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 5) tmem_alloc<kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int xq = h * D, xk = (a.Hq + kvh) * D, xv = (a.Hq + a.Hkv + kvh) * D;
      uint32_t issued = 0, parity = 0;
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_2d(smem + OFF_Q, &tm, xq, q0, q_full);
      tma_load_2d(smem + OFF_Q + PANEL, &tm, xq + 64, q0, q_full);
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, a.err)) { ok = false; break; }
        const int k0 = j * BKV;
        mbar_arrive_expect_tx(&k_full[st], TILE);
        tma_load_2d(smem + OFF_K + st * TILE, &tm, xk, k0, &k_full[st]);
        tma_load_2d(smem + OFF_K + st * TILE + PANEL, &tm, xk + 64, k0, &k_full[st]);
        mbar_arrive_expect_tx(&v_full[st], TILE);
        tma_load_2d(smem + OFF_V + st * TILE, &tm, xv, k0, &v_full[st]);
        tma_load_2d(smem + OFF_V + st * TILE + PANEL, &tm, xv + 64, k0, &v_full[st]);
        issued |= 1u << st;
        parity = (parity & ~(1u << st)) | (uint32_t((j >> 1) & 1) << st);
      }
      // Always make sure our copies have landed before the CTA may exit.
      mbar_wait(q_full, 0, nullptr);
      for (int st = 0; st < 2; ++st)
        if (issued & (1u << st)) {
          mbar_wait(&k_full[st], (parity >> st) & 1u, nullptr);
          mbar_wait(&v_full[st], (parity >> st) & 1u, nullptr);
        }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(BQ, BKV, false);
      constexpr uint32_t idesc_pv = idesc_bf16(BQ, D, true);
      bool ok = mbar_wait(q_full, 0, a.err);
      for (int j = 0; j <= nkv && ok; ++j) {
        if (j < nkv) {
          const int st = j & 1;
          if (!mbar_wait(&k_full[st], (j >> 1) & 1, a.err) ||
              !mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qa = smem_u32(smem + OFF_Q), kb = smem_u32(smem + OFF_K + st * TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * PANEL + (kk & 3) * 32;
            umma_f16(tS[st], smem_desc_sw128(qa + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc_qk,
                     kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
        }
        if (j >= 1) {
          const int jj = j - 1, pb = jj & 1;
          if (!mbar_wait(&p_full[pb], (jj >> 1) & 1, a.err) || !mbar_wait(&v_full[pb], (jj >> 1) & 1, a.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t pa = smem_u32(smem + OFF_P + pb * TILE), vb = smem_u32(smem + OFF_V + pb * TILE);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint32_t aoff = (kk >> 2) * PANEL + (kk & 3) * 32;
            umma_f16(tO, smem_desc_sw128(pa + aoff, 16, 1024), smem_desc_sw128(vb + kk * 2048, PANEL, 1024),
                     idesc_pv, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&pv_done[pb]);
          umma_commit(&kv_empty[pb]);
        }
      }
      // Retire every issued MMA before TMEM can be released.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int row = warp * 32 + lane;  // warps 0..3 own TMEM lane quarters 0..3
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    const int q_abs = q0 + row;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      const int sb = j & 1;
      const bool diag = (j == qt);
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, a.err)) ok = false;
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      tc_fence_after();
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS[sb] + lane_off + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int col = c * 32 + e;
          const float s = __uint_as_float(r[e]) * a.scale_log2;
          if (!diag || col <= row) mx = fmaxf(mx, s);
        }
      }
      const bool rescale = mx > m_ref + kRescaleThreshold;
      const float m_use = rescale ? mx : m_ref;
      // P buffer sb was last read by PV_{j-2}.
      if (j >= 2 && !mbar_wait(&pv_done[sb], ((j - 2) >> 1) & 1, a.err)) ok = false;
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      // pass 2: probabilities -> bf16 P (128-byte swizzled, K-major over keys)
      float rsum = 0.f;
      uint8_t* pbase = smem + OFF_P + sb * TILE;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS[sb] + lane_off + c * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int col = c * 32 + 2 * e;
          float p0 = exp2f(__uint_as_float(r[2 * e]) * a.scale_log2 - m_use);
          float p1 = exp2f(__uint_as_float(r[2 * e + 1]) * a.scale_log2 - m_use);
          if (diag && col > row) p0 = 0.f;
          if (diag && col + 1 > row) p1 = 0.f;
          rsum += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        uint8_t* panel = pbase + (c >> 1) * PANEL + row * 128;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const int chunk = (c & 1) * 4 + v;  // 16-byte chunk within the 128-byte row
          *reinterpret_cast<uint4*>(panel + ((chunk ^ (row & 7)) << 4)) =
              make_uint4(pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      // tcgen05.ld/st are warp-collective (.sync.aligned): the O rescale must
      // be taken by the whole warp; rows that do not need it use factor 1.
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? exp2f(m_ref - mx) : 1.0f;
        if (!mbar_wait(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.err)) ok = false;
        if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * f);
          tmem_st32(tO + lane_off + c * 32, r);
        }
        tmem_wait_st();
        l *= f;
      }
      if (rescale) m_ref = mx;
      l += rsum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    if (ok) {
      const int last = nkv - 1;
      const bool done = mbar_wait(&pv_done[last & 1], (last >> 1) & 1, a.err);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        bf16* orow = a.out + int64_t(q_abs) * a.ldo + int64_t(h) * D;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_wait_ld();
          if (q_abs < a.T) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
              o.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
              o.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
              o.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc<kTmemCols>(tmem);
  }
}

// ---------------------------------------------------------------------------
// Variant 2: two CTAs per SM.  P is written back into the S columns of TMEM
// (bf16 pairs) and consumed by the PV MMA straight from tensor memory, so a
// CTA needs only Q + one K + one V tile of shared memory (96 KB) and 256 TMEM
// columns; the second resident CTA's softmax overlaps this CTA's MMAs.
// ---------------------------------------------------------------------------
namespace v2 {
constexpr int OFF_Q = 0;
constexpr int OFF_K = TILE;
constexpr int OFF_V = 2 * TILE;
constexpr int OFF_BAR = 3 * TILE;
constexpr int SMEM_BYTES = OFF_BAR + 128 + 1024;
constexpr uint32_t kTmemCols = 256;  // S/P | O
}  // namespace v2

__global__ void __launch_bounds__(kThreads, 2)
    flash_prefill_v2_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + v2::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = bars + 2;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_empty = bars + 4;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* pv_done = bars + 7;
  uint64_t* drain = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int ntiles = (a.T + BQ - 1) / BQ;
  const int qt = ntiles - 1 - int(blockIdx.y);
  const int q0 = qt * BQ;
  const int kvh = h / (a.Hq / a.Hkv);
  const int nkv = qt + 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 8; ++i) mbar_init(&bars[i], (i == 6) ? 128 : 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 5) tmem_alloc<v2::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 4) {
    if (lane == 0) {
      const int xq = h * D, xk = (a.Hq + kvh) * D, xv = (a.Hq + a.Hkv + kvh) * D;
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_2d(smem + v2::OFF_Q, &tm, xq, q0, q_full);
      tma_load_2d(smem + v2::OFF_Q + PANEL, &tm, xq + 64, q0, q_full);
      int kdone = -1, vdone = -1;
      for (int j = 0; j < nkv; ++j) {
        const int k0 = j * BKV;
        if (!mbar_wait(k_empty, (j & 1) ^ 1, a.err)) break;
        mbar_arrive_expect_tx(k_full, TILE);
        tma_load_2d(smem + v2::OFF_K, &tm, xk, k0, k_full);
        tma_load_2d(smem + v2::OFF_K + PANEL, &tm, xk + 64, k0, k_full);
        kdone = j;
        if (!mbar_wait(v_empty, (j & 1) ^ 1, a.err)) break;
        mbar_arrive_expect_tx(v_full, TILE);
        tma_load_2d(smem + v2::OFF_V, &tm, xv, k0, v_full);
        tma_load_2d(smem + v2::OFF_V + PANEL, &tm, xv + 64, k0, v_full);
        vdone = j;
      }
      // make sure every issued copy has landed before the CTA can exit
      mbar_wait(q_full, 0, nullptr);
      if (kdone >= 0) mbar_wait(k_full, kdone & 1, nullptr);
      if (vdone >= 0) mbar_wait(v_full, vdone & 1, nullptr);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(BQ, BKV, false);
      constexpr uint32_t idesc_pv = idesc_bf16(BQ, D, true);
      bool ok = mbar_wait(q_full, 0, a.err);
      const uint32_t qa = smem_u32(smem + v2::OFF_Q), kb = smem_u32(smem + v2::OFF_K);
      const uint32_t vb = smem_u32(smem + v2::OFF_V);
      for (int j = 0; j < nkv && ok; ++j) {
        // S_j = Q K_j^T (overwrites P_{j-1}: PV_{j-1} was issued before, the
        // tensor pipe executes in order)
        if (!mbar_wait(k_full, j & 1, a.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * PANEL + (kk & 3) * 32;
          umma_f16(tS, smem_desc_sw128(qa + off, 16, 1024), smem_desc_sw128(kb + off, 16, 1024), idesc_qk,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        umma_commit(k_empty);
        // O += P_j V_j with P_j read from TMEM
        if (!mbar_wait(p_full, j & 1, a.err) || !mbar_wait(v_full, j & 1, a.err)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_f16_ta(tO, tS + kk * 8, smem_desc_sw128(vb + kk * 2048, PANEL, 1024), idesc_pv,
                      (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pv_done);
        umma_commit(v_empty);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    const int row = warp * 32 + lane;
    const uint32_t lane_off = uint32_t(warp * 32) << 16;
    const int q_abs = q0 + row;
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const bool diag = (j == qt);
      // s_full_j also implies PV_{j-1} has retired (committed after it).
      if (!mbar_wait(s_full, j & 1, a.err)) ok = false;
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      tc_fence_after();
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float sv = __uint_as_float(r[e]) * a.scale_log2;
          if (!diag || c * 32 + e <= row) mx = fmaxf(mx, sv);
        }
      }
      const bool rescale = mx > m_ref + kRescaleThreshold;
      const float m_use = rescale ? mx : m_ref;
      float rsum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tS + lane_off + c * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int col = c * 32 + 2 * e;
          float p0 = exp2f(__uint_as_float(r[2 * e]) * a.scale_log2 - m_use);
          float p1 = exp2f(__uint_as_float(r[2 * e + 1]) * a.scale_log2 - m_use);
          if (diag && col > row) p0 = 0.f;
          if (diag && col + 1 > row) p1 = 0.f;
          rsum += p0 + p1;
          pk[e] = pack_bf16x2(p0, p1);
        }
        // P chunk c (keys 32c..32c+31) -> columns [16c, 16c+16): only columns
        // of S chunks already read are overwritten.
        tmem_st16(tS + lane_off + c * 16, pk);
      }
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? exp2f(m_ref - mx) : 1.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * f);
          tmem_st32(tO + lane_off + c * 32, r);
        }
        l *= f;
      }
      tmem_wait_st();
      if (rescale) m_ref = mx;
      l += rsum;
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok) {
      const bool done = mbar_wait(pv_done, (nkv - 1) & 1, a.err);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        bf16* orow = a.out + int64_t(q_abs) * a.ldo + int64_t(h) * D;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tO + lane_off + c * 32, r);
          tmem_wait_ld();
          if (q_abs < a.T) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 o;
              o.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
              o.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
              o.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
              o.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + v * 8) = o;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc<v2::kTmemCols>(tmem);
  }
}

// ---------------------------------------------------------------------------
// Variant 3: two query tiles per CTA in ping-pong (one CTA per SM).
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
// uses packed f32x2 FMA/ADD, a 3-input max, and evaluates a fixed subset of
// the exponentials with a cubic on the FMA pipes to offload the MUFU.
// ---------------------------------------------------------------------------
namespace v3 {
constexpr int kThreads = 320;
constexpr int OFF_Q0 = 0;
constexpr int OFF_Q1 = TILE;
constexpr int OFF_K = 2 * TILE;  // 2 stages
constexpr int OFF_V = 4 * TILE;  // 2 stages
constexpr int OFF_BAR = 6 * TILE;
constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t kTmemCols = 512;
// Of every 16 consecutive key columns (8 pairs), pairs whose bit is set in
// this mask take the polynomial exponential.
constexpr uint32_t kPolyPairs = 0x11u;  // 2 of 8 pairs = 25 %

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}
// Packed f32x2 helpers on 64-bit registers (two fp32 lanes).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t addv2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t subv2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Loop-invariant operands of the softmax, packed once per tile row.
struct PolyConsts {
  uint64_t magic, c3, c2, c1, c0;
};
__device__ __forceinline__ PolyConsts poly_consts() {
  PolyConsts k;
  k.magic = pk2(12582912.0f, 12582912.0f);
  k.c3 = pk2(0.05516014f, 0.05516014f);
  k.c2 = pk2(0.24258275f, 0.24258275f);
  k.c1 = pk2(0.69326055f, 0.69326055f);
  k.c0 = pk2(0.99993020f, 0.99993020f);
  return k;
}
// Two exponentials on the FMA pipes, in packed arithmetic:
// 2^x = 2^n * 2^f with n = round(x) and f = x - n in [-0.5, 0.5].  With
// t = x + 1.5*2^23 the integer n sits in t's low mantissa bits, and
// (bits(t) << 23) == n << 23 modulo 2^32, so the exponent is added with one
// shift-add per lane.  2^f is a cubic whose coefficients were fitted for this
// kernel by relative-error-weighted least squares on [-0.5, 0.5] (max
// relative error 8e-5, far below the bf16 rounding of P).  Arguments are
// clamped below at -120 so the exponent never underflows.
__device__ __forceinline__ void ex2_poly2(uint64_t x2, const PolyConsts& k, float& p0, float& p1) {
  float x0, x1;
  upk2(x2, x0, x1);
  const uint64_t xc = pk2(fmaxf(x0, -120.0f), fmaxf(x1, -120.0f));
  const uint64_t t = addv2(xc, k.magic);
  const uint64_t n = subv2(t, k.magic);
  const uint64_t f = subv2(xc, n);
  uint64_t p = fma2(f, k.c3, k.c2);
  p = fma2(f, p, k.c1);
  p = fma2(f, p, k.c0);
  float pf0, pf1, tf0, tf1;
  upk2(p, pf0, pf1);
  upk2(t, tf0, tf1);
  p0 = __int_as_float(__float_as_int(pf0) + (__float_as_int(tf0) << 23));
  p1 = __int_as_float(__float_as_int(pf1) + (__float_as_int(tf1) << 23));
}
}  // namespace v3

__global__ void __launch_bounds__(v3::kThreads, 1)
    flash_prefill_v3_kernel(const __grid_constant__ CUtensorMap tm, AttnArgs a) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + v3::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2] per query tile
  uint64_t* p_full = bars + 11;  // [2] per query tile (128 arrivals)
  uint64_t* o_done = bars + 13;  // [2] per query tile
  uint64_t* drain = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int npairs = (a.T + 2 * BQ - 1) / (2 * BQ);
  const int pair = npairs - 1 - int(blockIdx.y);
  const int q0 = pair * 2 * BQ;
  const int kvh = h / (a.Hq / a.Hkv);
  const int n0 = q0 / BKV + 1;  // KV tiles seen by query tile 0
  const int n1 = n0 + 1;        // ... and by query tile 1

  if (threadIdx.x == 0) {
    for (int i = 0; i < 15; ++i) mbar_init(&bars[i], (i == 11 || i == 12) ? 128 : 1);
    mbar_init(drain, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm);
  }
  if (warp == 9) tmem_alloc<v3::kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      const int xq = h * D, xk = (a.Hq + kvh) * D, xv = (a.Hq + a.Hkv + kvh) * D;
      mbar_arrive_expect_tx(q_full, 2 * TILE);
      tma_load_2d(smem + v3::OFF_Q0, &tm, xq, q0, q_full);
      tma_load_2d(smem + v3::OFF_Q0 + PANEL, &tm, xq + 64, q0, q_full);
      tma_load_2d(smem + v3::OFF_Q1, &tm, xq, q0 + BQ, q_full);
      tma_load_2d(smem + v3::OFF_Q1 + PANEL, &tm, xq + 64, q0 + BQ, q_full);
      int kdone = -1, vdone = -1;
      for (int j = 0; j < n1; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        const int k0 = j * BKV;
        if (!mbar_wait(&k_empty[st], ph ^ 1, a.err)) break;
        mbar_arrive_expect_tx(&k_full[st], TILE);
        tma_load_2d(smem + v3::OFF_K + st * TILE, &tm, xk, k0, &k_full[st]);
        tma_load_2d(smem + v3::OFF_K + st * TILE + PANEL, &tm, xk + 64, k0, &k_full[st]);
        kdone = j;
        if (!mbar_wait(&v_empty[st], ph ^ 1, a.err)) break;
        mbar_arrive_expect_tx(&v_full[st], TILE);
        tma_load_2d(smem + v3::OFF_V + st * TILE, &tm, xv, k0, &v_full[st]);
        tma_load_2d(smem + v3::OFF_V + st * TILE + PANEL, &tm, xv + 64, k0, &v_full[st]);
        vdone = j;
      }
      // every issued copy lands before the CTA may exit (the last use of each
      // stage is the newest phase of its barrier)
      mbar_wait(q_full, 0, nullptr);
      for (int j = (kdone > 0 ? kdone - 1 : 0); j <= kdone; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr);
      for (int j = (vdone > 0 ? vdone - 1 : 0); j <= vdone; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_bf16(BQ, BKV, false);
      constexpr uint32_t idesc_pv = idesc_bf16(BQ, D, true);
      const uint32_t q0a = smem_u32(smem + v3::OFF_Q0), q1a = smem_u32(smem + v3::OFF_Q1);
      const uint32_t kb0 = smem_u32(smem + v3::OFF_K), vb0 = smem_u32(smem + v3::OFF_V);
      auto qk = [&](uint32_t dst, uint32_t qa, int j) {
        const uint32_t kb = kb0 + (j & 1) * TILE;
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
            if (!mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, a.err)) { ok = false; break; }
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
          if (!k_next_ready && !mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, a.err)) { ok = false; break; }
          tc_fence_after();
          qk(tS1, q1a, j + 1);
          umma_commit(&s_full[1]);
          umma_commit(&k_empty[(j + 1) & 1]);
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr);
    }
  } else {
    const int wg = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = uint32_t((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + wg * 128, tO = tmem + 256 + wg * 128;
    const int qrow0 = q0 + wg * BQ;
    const int q_abs = qrow0 + row;
    const int nkv = qrow0 / BKV + 1;
    const float sl2 = a.scale_log2;
    const v3::PolyConsts pk_consts = v3::poly_consts();
    float m_ref = -INFINITY, l0 = 0.f, l1 = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const bool diag = (j == nkv - 1);
      if (!mbar_wait(&s_full[wg], j & 1, a.err)) ok = false;
      if (__any_sync(0xffffffffu, !ok)) { ok = false; break; }
      tc_fence_after();
      // Pass 1: the row maximum over the whole S row.
      float mx = -INFINITY;
      {
        uint32_t r[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + lane_off + c * 32, r[c]);
        tmem_wait_ld();
        if (!diag) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; e += 2)
              mx = v3::max3(mx, __uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1]));
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (c * 32 + e <= row) mx = fmaxf(mx, __uint_as_float(r[c][e]));
        }
      }
      const float mxs = mx * sl2;
      const bool rescale = mxs > m_ref + kRescaleThreshold;
      const float m_use = rescale ? mxs : m_ref;
      const uint64_t scale2 = v3::pk2(sl2, sl2), negm2 = v3::pk2(-m_use, -m_use);
      uint64_t sum2 = v3::pk2(0.f, 0.f);
      // Pass 2: S is re-read chunk by chunk; the TMEM load of chunk c+1 is in
      // flight while chunk c is exponentiated.  P chunk c goes to columns
      // [16c, 16c+16), always below the S columns still to be read.
      uint32_t rb[2][32];
      tmem_ld32(tS + lane_off, rb[0]);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_wait_ld();
        if (c + 1 < 4) tmem_ld32(tS + lane_off + (c + 1) * 32, rb[(c + 1) & 1]);
        const uint32_t* rc = rb[c & 1];
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint64_t x2 = v3::fma2(v3::pk2(__uint_as_float(rc[2 * e]), __uint_as_float(rc[2 * e + 1])),
                                       scale2, negm2);
          float p0, p1;
          if ((v3::kPolyPairs >> (e & 7)) & 1u) {
            v3::ex2_poly2(x2, pk_consts, p0, p1);
          } else {
            float x0, x1;
            v3::upk2(x2, x0, x1);
            p0 = v3::ex2_mufu(x0);
            p1 = v3::ex2_mufu(x1);
          }
          if (diag) {
            if (c * 32 + 2 * e > row) p0 = 0.f;
            if (c * 32 + 2 * e + 1 > row) p1 = 0.f;
          }
          sum2 = v3::addv2(sum2, v3::pk2(p0, p1));
          pk[e] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tS + lane_off + c * 16, pk);
      }
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
      {
        float s0, s1;
        v3::upk2(sum2, s0, s1);
        l0 += s0;
        l1 += s1;
      }
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

void flash_prefill(torch::Tensor qkv, int64_t Hq, int64_t Hkv, double scale, torch::Tensor out, torch::Tensor err) {
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
  static bool attr = false;
  if (!attr) {
    KVS_CUDA_CHECK(cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    KVS_CUDA_CHECK(cudaFuncSetAttribute(flash_prefill_v2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        v2::SMEM_BYTES));
    KVS_CUDA_CHECK(cudaFuncSetAttribute(flash_prefill_v3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        v3::SMEM_BYTES));
    attr = true;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  static const int variant = [] {
    const char* e = std::getenv("KVS_ATTN_VARIANT");
    return e ? std::atoi(e) : 3;
  }();
  if (variant == 3) {
    dim3 grid(int(Hq), (T + 2 * BQ - 1) / (2 * BQ));
    flash_prefill_v3_kernel<<<grid, v3::kThreads, v3::SMEM_BYTES, st>>>(tm, a);
  } else {
    dim3 grid(int(Hq), (T + BQ - 1) / BQ);
    if (variant == 1)
      flash_prefill_kernel<<<grid, kThreads, SMEM_BYTES, st>>>(tm, a);
    else
      flash_prefill_v2_kernel<<<grid, kThreads, v2::SMEM_BYTES, st>>>(tm, a);
  }
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
