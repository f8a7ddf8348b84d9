// Persistent, warp-specialised bf16 GEMM on the 5th-generation tensor cores:
//   C[M, N] = A[M, K] * B[N, K]^T  (+ R[M, N])          (fp32 accumulate)
// A = activations (row-major, K contiguous), B = nn.Linear weight [out, in].
//
//   warp 0      TMA producer (one lane): 128x64 A and 256x64 B tiles with
//               128-byte swizzle into a 4-stage shared-memory ring.
//   warp 1      MMA issuer (one lane): tcgen05.mma M=128 N=256 K=16 into a
//               double-buffered TMEM accumulator (2 x 256 columns).
//   warps 2..5  epilogue: tcgen05.ld 32x32b -> bf16 -> global, overlapped
//               with the next tile's main loop.
// One CTA per SM, grid = min(tiles, #SMs).  Tiles are rastered in groups of
// kGroupM row blocks (m fastest inside a group), so the ~148 tiles in flight
// share 16 A row blocks and ~9 B column blocks: a weight much larger than L2
// (e.g. the 235 MB gate/up projection) is streamed num_m / 16 times instead
// of num_m times.
// Epilogue mode 3 fuses the tensor-parallel all-reduce of a row-parallel
// projection into the same launch (see the block comment above the kernel).
// No cluster multicast is used anywhere (this kernel may run in multi-GPU
// processes and reads only this GPU's memory through TMA).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "ops.h"
#include "sm100.cuh"

namespace kvs {

namespace {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_BYTES = BN * BK * 2;   // 32 KB
constexpr int SMEM_BYTES = STAGES * (A_BYTES + B_BYTES) + 1024 /*align*/ + 256 /*barriers*/;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;

constexpr int kGroupM = 16;
constexpr int kMaxTp = 8;                        // ranks of a fused all-reduce
constexpr int kEpiBytes = 4 * 32 * 64 * 2;       // per epilogue warp: a 32 x 64 bf16 slab

// Rank that reduces tile `tile` in mode 3.  Tile t belongs to CTA t % grid
// (round t / grid); the owner rotates with the round, so every CTA owns
// 1/world of its tiles and the NVLink bytes per CTA are balanced.
__device__ __forceinline__ int tile_owner(int tile, int grid, int world) {
  return (tile % grid + tile / grid) % world;
}

// The j-th tile of this CTA (n = its tile count).  Plain launches walk the
// rounds in order.  In mode 3 a CTA first computes the tiles it pushes to
// other ranks, then the ones it owns: by the time it reduces an owned tile
// the peers (who push first too) have already delivered their partials, so
// the owner rarely waits and NVLink carries partials during the first half
// and results during the second.
__device__ __forceinline__ int cta_tile(int j, int n, int act, int world, int rank) {
  const int cta = blockIdx.x, grid = gridDim.x;
  int k = j;
  if (act == 3 && world > 1) {
    const int k0 = ((rank - cta) % world + world) % world;  // first owned round
    const int owned = k0 < n ? (n - 1 - k0) / world + 1 : 0;
    const int pushed = n - owned;
    if (j < pushed) {
      const int b = j / (world - 1), q = j % (world - 1);
      k = b * world + q + (q >= k0 ? 1 : 0);
    } else {
      k = k0 + (j - pushed) * world;
    }
  }
  return cta + k * grid;
}

// Named barrier over the 128 epilogue threads (warps 2..5).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// The same barrier, returning the AND of `v` over the 128 threads.
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t out;
  asm volatile(
      "{\n.reg .pred pi, po;\n"
      "setp.ne.u32 pi, %1, 0;\n"
      "bar.red.and.pred po, 1, 128, pi;\n"
      "selp.u32 %0, 1, 0, po;\n}"
      : "=r"(out)
      : "r"(uint32_t(v))
      : "memory");
  return out != 0;
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int r = tile - group * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

struct GemmArgs {
  bf16* C;
  const bf16* R;
  const bf16* bias;
  int M, N, K;
  int act;  // 1: C[:, n] = silu(gate) * up, gate/up rows of B interleaved in blocks of BN/2
            // 2: fused QKV projection: bias, rotary embedding on q/k heads, k/v copies
  int64_t ldc, ldr;
  uint32_t* err;
  // act == 2 (head_dim 128, NeoX rotate-half; cos_sin [max_pos, 128] = cos[64] | sin[64])
  const float* cos_sin;
  const int32_t* positions;
  int hq, hkv;
  bf16* k_dst;
  bf16* v_dst;
  int64_t dst_tok_stride, dst_head_stride;
  // act == 3: C = sum over `world` tensor-parallel ranks of A_r * B_r^T, all
  // ranks receive the sum (C has the same shape and ldc on every rank)
  int world, rank;
  uint32_t epoch;             // this launch's sequence number (identical on every rank)
  uint64_t peer_timeout_ns;   // bound of every wait on a peer
  int max_tiles;              // tile capacity of the staging and flag regions
  bf16* out_peer[kMaxTp];     // every rank's C; out_peer[rank] == C
  bf16* stage_peer[kMaxTp];   // every rank's staging: [world-1 source slots][max_tiles][BM*BN]
  uint32_t* flag_peer[kMaxTp];  // every rank's flags: [world-1][max_tiles] partial, then [max_tiles] final
};

// Stores 32 consecutive bf16 (64 bytes) from fp32 values.
__device__ __forceinline__ void store32_bf16(bf16* dst, const float (&f)[32]) {
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) oh[e] = __floats2bfloat162_rn(f[8 * v + 2 * e], f[8 * v + 2 * e + 1]);
    *reinterpret_cast<uint4*>(dst + 8 * v) = o;
  }
}

// Selects arr[i] with compile-time indices (no local copy of the argument block).
template <typename T>
__device__ __forceinline__ T pick(const T (&arr)[kMaxTp], int i) {
  T v = arr[0];
#pragma unroll
  for (int k = 1; k < kMaxTp; ++k)
    if (i == k) v = arr[k];
  return v;
}

// Mode 3: GEMM + tensor-parallel all-reduce in one launch, over peer memory.
// Every rank runs the same persistent schedule; tile t is reduced by rank
// tile_owner(t).  A rank that does not own t stores its bf16 partial tile into
// the owner's staging slot (NVLink stores, 512 contiguous bytes per warp
// instruction); after a barrier over the epilogue threads one thread
// release-stores (system scope) the partial flag.  The owner
// acquire-waits for the world-1 partial flags, adds the partials to its fp32
// accumulator, rounds once to bf16 and writes the result rows (4 rows x 128
// contiguous bytes per instruction, through a swizzled shared-memory slab)
// into every rank's C, then release-stores each peer's final flag.  Before
// the launch ends every CTA acquire-waits for the final flags of the tiles it
// pushed, so C is complete on every rank when the kernel retires.  Per rank
// the NVLink bytes are 2 (world-1)/world of C, the ring all-reduce volume,
// and they move while the tensor cores compute the next tiles.  Flags hold
// the launch's epoch, so nothing is reset between launches; a peer that
// stops answering ends every wait after peer_timeout_ns with
// kStatusPeerTimeout in *err.  Staging and C are reused by the next launch
// safely: a rank's launch ends only after every owner consumed its partials,
// and an owner writes into a rank's C only after that rank pushed its own
// partial of the tile, i.e. entered the same launch.
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmArgs p) {
  using namespace sm100;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * (A_BYTES + B_BYTES));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;      // [0,2): accumulator full; [2]: abort drain
  uint64_t* tempty = tfull + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  uint8_t* epi_smem = smem + STAGES * (A_BYTES + B_BYTES) + 256;  // mode 3 only
  __shared__ int s_abort;
  const uint64_t wait_ns = p.act == 3 ? p.peer_timeout_ns + kWaitTimeoutNs : kWaitTimeoutNs;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(&tfull[2], 1);
    s_abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc<kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (p.M + BM - 1) / BM, num_n = (p.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;
  const int my_tiles = (tiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t issued_mask = 0, issued_parity = 0;  // per stage: load issued / its phase parity
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int tile = cta_tile(j, my_tiles, p.act, p.world, p.rank);
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, wait_ns)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, kb * BK, mb * BM, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES, &tmB, kb * BK, nb * BN, &full[stage]);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // Abort: wait (bounded) until every issued copy has landed so that no
        // TMA write targets this CTA's shared memory after it exits.
        s_abort = 1;
        for (int i = 0; i < STAGES; ++i)
          if (issued_mask & (1u << i)) mbar_wait(&full[i], (issued_parity >> i) & 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int j = 0; j < my_tiles && ok; ++j) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, p.err, wait_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, wait_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(b0 + kk * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      if (!ok) {
        // Abort: make sure every issued MMA has retired before TMEM is freed.
        s_abort = 1;
        umma_commit(&tfull[2]);
        mbar_wait(&tfull[2], 0, nullptr);
      }
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter = warp % 4.
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const int et = threadIdx.x - 64;  // 0..127
    int acc = 0;
    uint32_t acc_phase = 0;
    bool aborted = false;
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = cta_tile(j, my_tiles, p.act, p.world, p.rank);
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      // tcgen05.ld is warp-collective: leave the loop as a whole warp (as all
      // four warps in mode 3, whose named barriers need every epilogue warp).
      const bool ready = mbar_wait(&tfull[acc], acc_phase, p.err, wait_ns);
      if (!(p.act == 3 ? epi_bar_and(ready) : __all_sync(0xffffffffu, ready))) {
        aborted = true;
        break;
      }
      tc_fence_after();
      const int row = mb * BM + row_in_tile;
      const bool row_ok = row < p.M;
      if (p.act == 3) {
        const int owner = tile_owner(tile, gridDim.x, p.world);
        const uint32_t trow = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
        if (owner != p.rank) {
          // partial tile -> owner's staging, [32-column chunk][16-byte piece][row]
          const int slot = (p.rank - owner - 1 + p.world) % p.world;
          bf16* stg = pick(p.stage_peer, owner) + (int64_t(slot) * p.max_tiles + tile) * (BM * BN);
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(trow + c * 32, r);
            tmem_wait_ld();
            if (row_ok) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 o;
                __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  oh[e] = __floats2bfloat162_rn(__uint_as_float(r[v * 8 + 2 * e]),
                                                __uint_as_float(r[v * 8 + 2 * e + 1]));
                *reinterpret_cast<uint4*>(stg + (int64_t(c * 4 + v) * BM + row_in_tile) * 8) = o;
              }
            }
          }
          // the barrier orders every epilogue thread's stores before thread
          // 0's system-scope release (release is cumulative)
          epi_bar();
          if (et == 0) st_release_sys_u32(pick(p.flag_peer, owner) + slot * p.max_tiles + tile, p.epoch);
        } else {
          uint32_t* my_flags = pick(p.flag_peer, p.rank);
          bool got = true;
          if (et < p.world - 1) got = wait_flag_geq(my_flags + et * p.max_tiles + tile, p.epoch, p.peer_timeout_ns);
          if (!epi_bar_and(got)) {
            if (et == 0) atomicCAS(p.err, 0u, uint32_t(kStatusPeerTimeout));
            aborted = true;
            break;
          }
          const bf16* stg = pick(p.stage_peer, p.rank) + int64_t(tile) * (BM * BN);
          const int64_t slot_stride = int64_t(p.max_tiles) * (BM * BN);
          uint4* slab = reinterpret_cast<uint4*>(epi_smem + (warp - 2) * (kEpiBytes / 4));
#pragma unroll 1
          for (int h = 0; h < BN / 64; ++h) {
            uint32_t r0[32], r1[32];
            tmem_ld32(trow + h * 64, r0);
            tmem_ld32(trow + h * 64 + 32, r1);
            tmem_wait_ld();
            float f[64];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              f[e] = __uint_as_float(r0[e]);
              f[32 + e] = __uint_as_float(r1[e]);
            }
            if (row_ok) {
#pragma unroll
              for (int s2 = 0; s2 < kMaxTp - 1; ++s2) {
                if (s2 >= p.world - 1) break;
                const bf16* src = stg + s2 * slot_stride;
#pragma unroll
                for (int q = 0; q < 8; ++q) {  // chunk 2h + q/4, piece q%4
                  const uint4 x = __ldcg(reinterpret_cast<const uint4*>(
                      src + (int64_t((2 * h + q / 4) * 4 + q % 4) * BM + row_in_tile) * 8));
                  const __nv_bfloat162* xh = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float2 y = __bfloat1622float2(xh[e]);
                    f[q * 8 + 2 * e] += y.x;
                    f[q * 8 + 2 * e + 1] += y.y;
                  }
                }
              }
            }
            // this thread's 64 columns -> row `lane` of the slab, pieces XOR-swizzled
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              uint4 o;
              __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
              for (int e = 0; e < 4; ++e) oh[e] = __floats2bfloat162_rn(f[q * 8 + 2 * e], f[q * 8 + 2 * e + 1]);
              slab[lane * 8 + (q ^ (lane & 7))] = o;
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = i * 4 + (lane >> 3), piece = lane & 7;
              const uint4 val = slab[rr * 8 + (piece ^ (rr & 7))];
              const int grow = mb * BM + quarter * 32 + rr;
              if (grow < p.M) {
                const int64_t off = int64_t(grow) * p.ldc + nb * BN + h * 64 + piece * 8;
#pragma unroll
                for (int d = 0; d < kMaxTp; ++d) {
                  if (d >= p.world) break;
                  *reinterpret_cast<uint4*>(p.out_peer[d] + off) = val;
                }
              }
            }
            __syncwarp();
          }
          epi_bar();
          if (et < p.world && et != p.rank)
            st_release_sys_u32(pick(p.flag_peer, et) + (p.world - 1) * p.max_tiles + tile, p.epoch);
        }
      } else if (p.act == 2) {
        // Two heads per tile.  Values are rounded to bf16 before the rotation
        // (the same arithmetic as the stand-alone rope kernel, so prefill and
        // decode agree bit for bit).
        const int pos = row_ok ? p.positions[row] : 0;
        const float* cs = p.cos_sin + int64_t(pos) * 128;
#pragma unroll 1
        for (int hl = 0; hl < BN / 128; ++hl) {
          const int hh = nb * (BN / 128) + hl;
          if (hh * 128 >= p.N) break;
          const uint32_t tb = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + hl * 128);
          bf16* crow = p.C + int64_t(row) * p.ldc + hh * 128;
          const bool rotary = hh < p.hq + p.hkv;
          const bool is_k = hh >= p.hq && hh < p.hq + p.hkv;
          bf16* extra = nullptr;
          if (is_k && p.k_dst) extra = p.k_dst + int64_t(row) * p.dst_tok_stride + int64_t(hh - p.hq) * p.dst_head_stride;
          if (!rotary && p.v_dst)
            extra = p.v_dst + int64_t(row) * p.dst_tok_stride + int64_t(hh - p.hq - p.hkv) * p.dst_head_stride;
#pragma unroll 1
          for (int cc = 0; cc < 2; ++cc) {
            uint32_t r1[32], r2[32];
            tmem_ld32(tb + cc * 32, r1);
            tmem_ld32(tb + 64 + cc * 32, r2);
            tmem_wait_ld();
            if (!row_ok) continue;
            float x1[32], x2[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int d = cc * 32 + e;
              float a1 = __uint_as_float(r1[e]), a2 = __uint_as_float(r2[e]);
              if (p.bias) {
                a1 += __bfloat162float(p.bias[hh * 128 + d]);
                a2 += __bfloat162float(p.bias[hh * 128 + 64 + d]);
              }
              x1[e] = __bfloat162float(__float2bfloat16_rn(a1));
              x2[e] = __bfloat162float(__float2bfloat16_rn(a2));
            }
            if (rotary) {
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const int d = cc * 32 + e;
                const float c = cs[d], sn = cs[64 + d];
                const float o1 = x1[e] * c - x2[e] * sn, o2 = x2[e] * c + x1[e] * sn;
                x1[e] = o1;
                x2[e] = o2;
              }
            }
            store32_bf16(crow + cc * 32, x1);
            store32_bf16(crow + 64 + cc * 32, x2);
            if (extra) {
              store32_bf16(extra + cc * 32, x1);
              store32_bf16(extra + 64 + cc * 32, x2);
            }
          }
        }
      } else if (p.act) {
        // gate in accumulator columns [0, 128), up in [128, 256) of the same
        // 128 output features; output columns nb*128 + [0, 128).
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
          uint32_t g[32], u[32];
          const uint32_t t0 = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + c * 32);
          tmem_ld32(t0, g);
          tmem_ld32(t0 + BN / 2, u);
          tmem_wait_ld();
          const int col0 = nb * (BN / 2) + c * 32;
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = col0 + v * 8;
              if (col >= p.N / 2) break;
              uint4 o;
              __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float g0 = __uint_as_float(g[v * 8 + 2 * e]), g1 = __uint_as_float(g[v * 8 + 2 * e + 1]);
                const float u0 = __uint_as_float(u[v * 8 + 2 * e]), u1 = __uint_as_float(u[v * 8 + 2 * e + 1]);
                // silu(g) = g / (1 + e^-g); the exponent argument is capped so the
                // divisor stays finite and the fast division applies
                const float d0 = 1.0f + __expf(fminf(-g0, 80.0f)), d1 = 1.0f + __expf(fminf(-g1, 80.0f));
                oh[e] = __floats2bfloat162_rn(__fdividef(g0, d0) * u0, __fdividef(g1, d1) * u1);
              }
              *reinterpret_cast<uint4*>(p.C + int64_t(row) * p.ldc + col) = o;
            }
          }
        }
      } else {
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN + c * 32), r);
        tmem_wait_ld();
        const int col0 = nb * BN + c * 32;
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int col = col0 + v * 8;
            if (col >= p.N) break;
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(r[v * 8 + e]);
            if (p.bias) {
              const uint4 bb = *reinterpret_cast<const uint4*>(p.bias + col);
              const __nv_bfloat162* bh = reinterpret_cast<const __nv_bfloat162*>(&bb);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 x = __bfloat1622float2(bh[e]);
                f[2 * e] += x.x;
                f[2 * e + 1] += x.y;
              }
            }
            if (p.R) {
              const uint4 rr = *reinterpret_cast<const uint4*>(p.R + int64_t(row) * p.ldr + col);
              const __nv_bfloat162* rh = reinterpret_cast<const __nv_bfloat162*>(&rr);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 x = __bfloat1622float2(rh[e]);
                f[2 * e] += x.x;
                f[2 * e + 1] += x.y;
              }
            }
            uint4 o;
            __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) oh[e] = __floats2bfloat162_rn(f[2 * e], f[2 * e + 1]);
            *reinterpret_cast<uint4*>(p.C + int64_t(row) * p.ldc + col) = o;
          }
        }
      }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (p.act == 3 && !aborted) {
      // C is complete on this rank once every tile this CTA pushed came back
      const uint32_t* finals = pick(p.flag_peer, p.rank) + (p.world - 1) * p.max_tiles;
      bool got = true;
      for (int t = blockIdx.x + et * gridDim.x; t < tiles && got; t += 128 * gridDim.x)
        if (tile_owner(t, gridDim.x, p.world) != p.rank) got = wait_flag_geq(finals + t, p.epoch, p.peer_timeout_ns);
      if (!epi_bar_and(got) && et == 0) atomicCAS(p.err, 0u, uint32_t(kStatusPeerTimeout));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<kTmemCols>(tmem_base);
  }
}

using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn get_encode_fn() {
  static EncodeFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    KVS_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    KVS_CHECK_ARG(q == cudaDriverEntryPointSuccess && ptr != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

}  // namespace

CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  KVS_CHECK_ARG((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  KVS_CHECK_ARG(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KVS_CHECK_ARG(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    KVS_CUDA_CHECK(cudaGetDevice(&dev));
    KVS_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

namespace {
void launch_gemm(const torch::Tensor& a, const torch::Tensor& b, GemmArgs& p) {
  const int M = p.M, N = p.N, K = p.K;
  const CUtensorMap ta = make_tmap_2d_bf16(a.data_ptr(), K, M, uint64_t(a.stride(0)) * 2, BK, BM);
  const CUtensorMap tb = make_tmap_2d_bf16(b.data_ptr(), K, N, uint64_t(b.stride(0)) * 2, BK, BN);
  static bool attr_set = false;
  if (!attr_set) {
    KVS_CUDA_CHECK(cudaFuncSetAttribute(gemm_bf16_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SMEM_BYTES + kEpiBytes));
    attr_set = true;
  }
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  gemm_bf16_tn_kernel<<<grid, kThreads, SMEM_BYTES + (p.act == 3 ? kEpiBytes : 0), st>>>(ta, tb, p);
  KVS_CUDA_CHECK(cudaGetLastError());
}
}  // namespace

void gemm_qkv_rope_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, c10::optional<torch::Tensor> bias,
                        torch::Tensor cos_sin, torch::Tensor positions, int64_t hq, int64_t hkv,
                        c10::optional<torch::Tensor> k_dst, c10::optional<torch::Tensor> v_dst, torch::Tensor err) {
  KVS_CHECK_ARG(a.is_cuda() && b.is_cuda() && c.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                    b.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16,
                "gemm_qkv_rope: bf16 CUDA operands");
  KVS_CHECK_ARG(a.dim() == 2 && b.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                    c.stride(1) == 1,
                "gemm_qkv_rope: 2-D row-major operands");
  const int M = int(a.size(0)), K = int(a.size(1)), N = int(b.size(0));
  KVS_CHECK_ARG(b.size(1) == K && c.size(0) == M && c.size(1) == N && N == (hq + 2 * hkv) * 128,
                "gemm_qkv_rope: b [(hq+2hkv)*128, K], c [M, N]");
  KVS_CHECK_ARG(K % 8 == 0 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && c.stride(0) % 8 == 0,
                "gemm_qkv_rope: K and leading dims must be multiples of 8");
  KVS_CHECK_ARG(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() && cos_sin.size(1) == 128,
                "gemm_qkv_rope: cos_sin [max_pos, 128] fp32");
  KVS_CHECK_ARG(positions.scalar_type() == at::kInt && positions.numel() >= M, "gemm_qkv_rope: int32 positions");
  if (M == 0) return;
  GemmArgs p{};
  p.C = reinterpret_cast<bf16*>(c.data_ptr());
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = c.stride(0);
  p.act = 2;
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  if (bias.has_value()) {
    KVS_CHECK_ARG(bias->numel() == N && bias->is_contiguous() && bias->scalar_type() == at::kBFloat16,
                  "gemm_qkv_rope: bias must be contiguous bf16 [N]");
    p.bias = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  p.cos_sin = cos_sin.data_ptr<float>();
  p.positions = positions.data_ptr<int32_t>();
  p.hq = int(hq);
  p.hkv = int(hkv);
  if (k_dst.has_value() || v_dst.has_value()) {
    KVS_CHECK_ARG(k_dst.has_value() && v_dst.has_value() && k_dst->dim() == 3 && k_dst->strides() == v_dst->strides() &&
                      k_dst->stride(2) == 1 && k_dst->size(0) >= M && k_dst->stride(0) % 8 == 0 &&
                      k_dst->stride(1) % 8 == 0,
                  "gemm_qkv_rope: k_dst/v_dst [>=M, hkv, 128] with equal strides");
    p.k_dst = reinterpret_cast<bf16*>(k_dst->data_ptr());
    p.v_dst = reinterpret_cast<bf16*>(v_dst->data_ptr());
    p.dst_tok_stride = k_dst->stride(0);
    p.dst_head_stride = k_dst->stride(1);
  }
  launch_gemm(a, b, p);
}

void gemm_allreduce_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, std::vector<int64_t> out_ptrs,
                         std::vector<int64_t> stage_ptrs, std::vector<int64_t> flag_ptrs, int64_t rank,
                         int64_t max_tiles, int64_t epoch, int64_t timeout_ns, torch::Tensor err) {
  KVS_CHECK_ARG(a.is_cuda() && b.is_cuda() && c.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                    b.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16,
                "gemm_allreduce: bf16 CUDA operands");
  KVS_CHECK_ARG(a.dim() == 2 && b.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                    c.is_contiguous(),
                "gemm_allreduce: row-major a, b and contiguous c");
  const int M = int(a.size(0)), K = int(a.size(1)), N = int(b.size(0));
  const int world = int(out_ptrs.size());
  KVS_CHECK_ARG(b.size(1) == K && c.size(0) == M && c.size(1) == N, "gemm_allreduce: shape mismatch");
  KVS_CHECK_ARG(K % 8 == 0 && N % BN == 0 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0,
                "gemm_allreduce: K % 8 == 0 and N % 256 == 0");
  KVS_CHECK_ARG(world >= 1 && world <= kMaxTp && int(stage_ptrs.size()) == world &&
                    int(flag_ptrs.size()) == world && rank >= 0 && rank < world,
                "gemm_allreduce: 1..8 ranks with one output, staging and flag pointer each");
  KVS_CHECK_ARG(out_ptrs[rank] == reinterpret_cast<int64_t>(c.data_ptr()), "gemm_allreduce: c must be out_ptrs[rank]");
  const int64_t tiles = int64_t((M + BM - 1) / BM) * (N / BN);
  KVS_CHECK_ARG(tiles <= max_tiles, "gemm_allreduce: more tiles than the workspace holds");
  for (int r = 0; r < world; ++r)
    KVS_CHECK_ARG(out_ptrs[r] % 16 == 0 && stage_ptrs[r] % 16 == 0 && flag_ptrs[r] % 4 == 0,
                  "gemm_allreduce: misaligned peer buffer");
  if (M == 0) return;
  GemmArgs p{};
  p.C = reinterpret_cast<bf16*>(c.data_ptr());
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = N;
  p.act = 3;
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  p.world = world;
  p.rank = int(rank);
  p.epoch = uint32_t(epoch);
  p.peer_timeout_ns = uint64_t(timeout_ns);
  p.max_tiles = int(max_tiles);
  for (int r = 0; r < world; ++r) {
    p.out_peer[r] = reinterpret_cast<bf16*>(out_ptrs[r]);
    p.stage_peer[r] = reinterpret_cast<bf16*>(stage_ptrs[r]);
    p.flag_peer[r] = reinterpret_cast<uint32_t*>(flag_ptrs[r]);
  }
  launch_gemm(a, b, p);
}

void gemm_silu_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, torch::Tensor err) {
  KVS_CHECK_ARG(a.is_cuda() && b.is_cuda() && c.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                    b.scalar_type() == at::kBFloat16 && c.scalar_type() == at::kBFloat16,
                "gemm_silu: bf16 CUDA operands");
  KVS_CHECK_ARG(a.dim() == 2 && b.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                    c.stride(1) == 1,
                "gemm_silu: 2-D row-major operands");
  const int M = int(a.size(0)), K = int(a.size(1)), N = int(b.size(0));
  KVS_CHECK_ARG(b.size(1) == K && c.size(0) == M && 2 * c.size(1) == N && N % BN == 0,
                "gemm_silu: b [2I, K] (gate/up interleaved in 128-row blocks), c [M, I], I % 128 == 0");
  KVS_CHECK_ARG(K % 8 == 0 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && c.stride(0) % 8 == 0,
                "gemm_silu: K and leading dims must be multiples of 8");
  if (M == 0) return;
  GemmArgs p{};
  p.C = reinterpret_cast<bf16*>(c.data_ptr());
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = c.stride(0);
  p.act = 1;
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  launch_gemm(a, b, p);
}

void gemm_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor c, c10::optional<torch::Tensor> residual,
               c10::optional<torch::Tensor> bias, torch::Tensor err) {
  KVS_CHECK_ARG(a.is_cuda() && b.is_cuda() && c.is_cuda(), "gemm: CUDA tensors");
  KVS_CHECK_ARG(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 &&
                    c.scalar_type() == at::kBFloat16,
                "gemm: bf16 operands");
  KVS_CHECK_ARG(a.dim() == 2 && b.dim() == 2 && c.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 &&
                    c.stride(1) == 1,
                "gemm: 2-D row-major operands");
  const int M = int(a.size(0)), K = int(a.size(1)), N = int(b.size(0));
  KVS_CHECK_ARG(b.size(1) == K && c.size(0) == M && c.size(1) == N, "gemm: shape mismatch");
  KVS_CHECK_ARG(K % 8 == 0 && N % 8 == 0 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && c.stride(0) % 8 == 0,
                "gemm: K, N and leading dims must be multiples of 8");
  if (M == 0 || N == 0) return;
  GemmArgs p{};
  p.C = reinterpret_cast<bf16*>(c.data_ptr());
  p.M = M;
  p.N = N;
  p.K = K;
  p.ldc = c.stride(0);
  p.R = nullptr;
  p.ldr = 0;
  if (residual.has_value()) {
    KVS_CHECK_ARG(residual->sizes() == c.sizes() && residual->stride(1) == 1 && residual->stride(0) % 8 == 0,
                  "gemm: residual shape");
    p.R = reinterpret_cast<const bf16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  p.bias = nullptr;
  if (bias.has_value()) {
    KVS_CHECK_ARG(bias->numel() == N && bias->is_contiguous() && bias->scalar_type() == at::kBFloat16,
                  "gemm: bias must be contiguous bf16 [N]");
    p.bias = reinterpret_cast<const bf16*>(bias->data_ptr());
  }
  p.err = reinterpret_cast<uint32_t*>(err.data_ptr<int32_t>());
  launch_gemm(a, b, p);
}

}  // namespace kvs
