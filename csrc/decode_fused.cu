// Decode-step kernels that fuse a projection with the collective after it.
//
// * gemv_allreduce: a row-parallel projection (attention output, MLP down)
//   of a decode step (M <= 8 tokens) and the tensor-parallel all-reduce of its
//   [M, N] result in ONE launch.  Each CTA computes 16 output rows from this
//   rank's K shard and stores every fp32 partial into every TP rank's staging
//   memory over NVLink as a 64-bit "LL" word (high half: the launch's flag
//   value, low half: the partial; plain peer stores, no TMA and no
//   multicast).  It then polls its own staging, bounded by %globaltimer,
//   until the words of all ranks carry the flag, and sums ranks 0..world-1
//   in that fixed order — every rank writes bitwise the same bf16 result.
//   A 64-bit aligned store is single-copy atomic, so no fence and no
//   separate flag word are needed; the transfer of one CTA's rows overlaps
//   the weight streaming of the others; there is no separate NCCL call.
// * gemv_argmax: the decode step's LM-head projection fused with greedy
//   sampling: per-CTA argmax of its 16 logits, a last-CTA reduction over the
//   CTAs, and — with tensor parallelism over the vocabulary — an exchange of
//   each rank's (value, index) with every peer as two LL words.  The logits
//   never go to memory.
// * decode_epoch_bump: advances the step epoch that tags the words (one
//   thread, the last kernel of a decode step; a CUDA graph replays the step
//   with frozen arguments, so the epoch lives in device memory).
//
// Flag values are epoch * num_sites + site + 1 (strictly increasing over a
// run).  Staging is double-buffered by the parity of the launch site: a
// peer can only write the next site of the same parity after this rank has
// published the site in between, which it does only after it has read the
// current one.  All CTAs of a gemv_allreduce launch must be co-resident (the
// host checks the occupancy), so a poll never depends on an unscheduled CTA.
// The GEMVs are PDL launches: their weight prefetch overlaps the tail of the
// previous kernel of the step.
//
// The reference has no decode engine (vLLM serves decode, with NCCL
// all-reduces after its row-parallel layers); these kernels belong to the
// standalone engine of this framework.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"
#include "gemv_core.cuh"
#include "ops.h"

namespace kvs {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxTok = 8;

struct PeerTable {
  uint64_t stage[kMaxRanks];   // byte address of each rank's LL staging region (peer-mapped)
};

__device__ __forceinline__ void report(uint32_t* status, uint32_t code) {
  if (status) atomicCAS(status, uint32_t(kStatusOk), code);
}

constexpr int kMaxChunks = 8;   // 16-row chunks per CTA (grid = N / (16 * chunks) must fit at once)

// Staging of rank `src`'s partial rows in rank `dst`'s region: LL words
// [parity][src][token][stage_ld] (one 64-bit word per fp32 partial).
__device__ __forceinline__ uint64_t* stage_word(uint64_t base, int parity, int world, int src, int m,
                                                int64_t stage_ld, int64_t col) {
  return reinterpret_cast<uint64_t*>(base) + ((int64_t(parity) * world + src) * kMaxTok + m) * stage_ld + col;
}

template <int M>
__global__ void __launch_bounds__(kGemvThreads) gemv_allreduce_kernel(
    const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w, int64_t ldw, bf16* __restrict__ y,
    int64_t ldy, int N, int K, int chunks, PeerTable peers, int rank, int world, int site, int num_sites,
    const int32_t* __restrict__ epoch_ptr, int64_t stage_ld, uint64_t timeout_ns, uint32_t* __restrict__ status) {
  extern __shared__ uint4 xs_raw[];  // [M][K] bf16
  __shared__ __align__(16) float part[kMaxChunks][M][kGemvRowsPerCta];
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col0 = int64_t(blockIdx.x) * chunks * kGemvRowsPerCta;   // N % (16 * chunks) == 0
  GemvWarp<M> g;
  g.prefetch(w, ldw, int(col0) + warp * kGemvRows, N, K, lane);
  pdl_wait();   // x, the epoch and the staging words of the previous site are the predecessor's
  gemv_stage_x<M>(x, ldx, xs_raw, K);
  __syncthreads();
  for (int c = 0; c < chunks; ++c) {
    const int row0 = int(col0) + c * kGemvRowsPerCta + warp * kGemvRows;
    float acc[kGemvRows][M];
    if (c > 0) g.have = false;
    g.run(w, ldw, reinterpret_cast<const bf16*>(xs_raw), row0, N, K, lane, acc);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) part[c][m][warp * kGemvRows + r] = acc[r][m];
    }
  }
  __syncthreads();
  const int parity = site & 1;
  const uint32_t val = uint32_t(*epoch_ptr) * uint32_t(num_sites) + uint32_t(site) + 1u;
  const int rows = chunks * kGemvRowsPerCta;
  // push: every partial, tagged with `val`, into slot [parity][rank] of every
  // rank (itself included) — one single-copy-atomic 64-bit store each
  for (int t = threadIdx.x; t < world * M * rows; t += blockDim.x) {
    const int r = t / (M * rows), rem = t % (M * rows);
    const int m = rem / rows, i = rem % rows;
    st_ll(stage_word(peers.stage[r], parity, world, rank, m, stage_ld, col0 + i),
          __float_as_uint(part[i / kGemvRowsPerCta][m][i % kGemvRowsPerCta]), val);
  }
  // pull: poll this rank's own staging until every rank's word of the row
  // carries `val`, then sum in rank order 0..world-1 (bitwise equal on all ranks)
  const uint64_t deadline = globaltimer_ns() + timeout_ns;
  bool ok = true;
  for (int t = threadIdx.x; t < M * rows; t += blockDim.x) {
    const int m = t / rows, i = t % rows;
    float s = 0.f;
    for (int r = 0; r < world && ok; ++r)
      s += __uint_as_float(poll_ll(stage_word(peers.stage[rank], parity, world, r, m, stage_ld, col0 + i), val,
                                   deadline, ok));
    y[int64_t(m) * ldy + col0 + i] = rn(s);
  }
  if (!ok) report(status, kStatusPeerTimeout);
}

struct ArgmaxSlot {
  float val;
  int32_t idx;
};

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

template <int M>
__global__ void __launch_bounds__(kGemvThreads) gemv_argmax_kernel(
    const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ w, int64_t ldw, int N, int K,
    int64_t vocab_begin, float* __restrict__ part_val, int32_t* __restrict__ part_idx,
    uint32_t* __restrict__ counter, int32_t* __restrict__ out, PeerTable peers, int rank, int world, int site,
    int num_sites, const int32_t* __restrict__ epoch_ptr, uint64_t timeout_ns, uint32_t* __restrict__ status) {
  extern __shared__ uint4 xs_raw[];
  __shared__ float sv[M][kGemvRowsPerCta];
  __shared__ int si[M][kGemvRowsPerCta];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = blockIdx.x * kGemvRowsPerCta + warp * kGemvRows;
  pdl_trigger();
  GemvWarp<M> g;
  g.prefetch(w, ldw, row0, N, K, lane);
  pdl_wait();
  gemv_stage_x<M>(x, ldx, xs_raw, K);
  __syncthreads();
  float acc[kGemvRows][M];
  if (row0 < N) g.run(w, ldw, reinterpret_cast<const bf16*>(xs_raw), row0, N, K, lane, acc);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const bool ok = row0 + r < N;
        // the logits are bf16 in the unfused path: compare the rounded values
        sv[m][warp * kGemvRows + r] = ok ? rnf(acc[r][m]) : -INFINITY;
        si[m][warp * kGemvRows + r] = ok ? row0 + r : 0x7fffffff;
      }
  }
  __syncthreads();
  if (threadIdx.x < M) {
    const int m = threadIdx.x;
    float bv = sv[m][0];
    int bi = si[m][0];
    for (int i = 1; i < kGemvRowsPerCta; ++i)
      if (better(sv[m][i], si[m][i], bv, bi)) { bv = sv[m][i]; bi = si[m][i]; }
    part_val[int64_t(m) * gridDim.x + blockIdx.x] = bv;
    part_idx[int64_t(m) * gridDim.x + blockIdx.x] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // last CTA: one warp per token reduces the per-CTA candidates
  __shared__ ArgmaxSlot best[M];
  for (int m = warp; m < M; m += kGemvThreads / 32) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < int(gridDim.x); c += 32) {
      const float v = __ldcg(part_val + int64_t(m) * gridDim.x + c);
      const int i = __ldcg(part_idx + int64_t(m) * gridDim.x + c);
      if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) best[m] = ArgmaxSlot{bv, int32_t(bi + vocab_begin)};
  }
  __syncthreads();
  if (world > 1) {
    const int parity = site & 1;
    const uint32_t val = uint32_t(*epoch_ptr) * uint32_t(num_sites) + uint32_t(site) + 1u;
    // candidate of this rank -> LL words [parity][rank][token][value, index] of every rank
    if (threadIdx.x < world * M) {
      const int r = threadIdx.x / M, m = threadIdx.x % M;
      uint64_t* dst = reinterpret_cast<uint64_t*>(peers.stage[r]) + ((int64_t(parity) * world + rank) * kMaxTok + m) * 2;
      st_ll(dst, __float_as_uint(best[m].val), val);
      st_ll(dst + 1, uint32_t(best[m].idx), val);
    }
    if (threadIdx.x < M) {
      const int m = threadIdx.x;
      const uint64_t deadline = globaltimer_ns() + timeout_ns;
      bool ok = true;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int r = 0; r < world && ok; ++r) {
        const uint64_t* src = reinterpret_cast<const uint64_t*>(peers.stage[rank]) +
                              ((int64_t(parity) * world + r) * kMaxTok + m) * 2;
        const float v = __uint_as_float(poll_ll(src, val, deadline, ok));
        const int i = int(poll_ll(src + 1, val, deadline, ok));
        if (ok && better(v, i, bv, bi)) { bv = v; bi = i; }
      }
      if (!ok) report(status, kStatusPeerTimeout);
      out[m] = bi;
    }
  } else if (threadIdx.x < M) {
    out[threadIdx.x] = best[threadIdx.x].idx;
  }
  if (threadIdx.x == 0) *counter = 0u;   // the next launch is stream-ordered after this one
}

__global__ void decode_epoch_bump_kernel(int32_t* epoch) {
  pdl_trigger();
  if (threadIdx.x == 0 && blockIdx.x == 0) *epoch += 1;
}

PeerTable make_table(const std::vector<int64_t>& stage, int world) {
  KVS_CHECK_ARG(world >= 1 && world <= kMaxRanks && int(stage.size()) == world,
                "decode collective: one staging address per rank (1..8 ranks)");
  PeerTable t{};
  for (int r = 0; r < world; ++r) {
    KVS_CHECK_ARG(stage[r] && stage[r] % 16 == 0, "decode collective: staging must be 16-byte aligned");
    t.stage[r] = uint64_t(stage[r]);
  }
  return t;
}

// CTAs of `kern` (kGemvThreads threads, `smem` bytes of dynamic shared
// memory) that fit on the GPU at once (cached per kernel and size).
template <typename Kern>
int resident_capacity(Kern kern, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void*, size_t>, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kern), smem);
  const auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  KVS_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  int per_sm = 0, dev = 0, sms = 0;
  KVS_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGemvThreads, smem));
  KVS_CUDA_CHECK(cudaGetDevice(&dev));
  KVS_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return cache[key] = per_sm * sms;
}

void check_gemv_args(const torch::Tensor& x, const torch::Tensor& w, int& M, int& K, int& N) {
  KVS_CHECK_ARG(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
                "decode gemv: CUDA bf16 operands");
  KVS_CHECK_ARG(x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1,
                "decode gemv: row-major 2-D operands");
  M = int(x.size(0));
  K = int(x.size(1));
  N = int(w.size(0));
  KVS_CHECK_ARG(w.size(1) == K && M >= 1 && M <= kMaxTok, "decode gemv: x [M<=8, K], w [N, K]");
  KVS_CHECK_ARG(K % 8 == 0 && w.stride(0) % 8 == 0 && x.stride(0) % 8 == 0, "decode gemv: K multiple of 8");
  KVS_CHECK_ARG(size_t(M) * K * 2 <= 200 * 1024, "decode gemv: x does not fit in shared memory");
}

}  // namespace

void gemv_allreduce_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor y, std::vector<int64_t> stage_ptrs,
                         int64_t rank, int64_t site, int64_t num_sites, torch::Tensor epoch, int64_t stage_ld,
                         int64_t timeout_ns, torch::Tensor status) {
  int M, K, N;
  check_gemv_args(x, w, M, K, N);
  const int world = int(stage_ptrs.size());
  const PeerTable peers = make_table(stage_ptrs, world);
  KVS_CHECK_ARG(y.is_cuda() && y.scalar_type() == at::kBFloat16 && y.dim() == 2 && y.size(0) == M &&
                    y.size(1) == N && y.stride(1) == 1,
                "gemv_allreduce: y [M, N] bf16");
  KVS_CHECK_ARG(N % kGemvRowsPerCta == 0 && N <= stage_ld && stage_ld % 2 == 0,
                "gemv_allreduce: N must be a multiple of 16 within the staging width");
  KVS_CHECK_ARG(rank >= 0 && rank < world && site >= 0 && site < num_sites, "gemv_allreduce: rank/site");
  KVS_CHECK_ARG(epoch.is_cuda() && epoch.scalar_type() == at::kInt && status.is_cuda() &&
                    status.scalar_type() == at::kInt,
                "gemv_allreduce: epoch / status int32 device tensors");
  const size_t smem = size_t(M) * K * 2;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto wp = reinterpret_cast<const bf16*>(w.data_ptr());
  auto yp = reinterpret_cast<bf16*>(y.data_ptr());
  auto ep = reinterpret_cast<const int32_t*>(epoch.data_ptr());
  auto sp = reinterpret_cast<uint32_t*>(status.data_ptr());
// The fewest 16-row chunks per CTA that keep the whole grid resident (the
// peer polls need every CTA running): large K at M = 8 leaves one CTA per SM.
#define KVS_GAR_CASE(MM)                                                                                        \
  case MM: {                                                                                                    \
    const int cap = resident_capacity(gemv_allreduce_kernel<MM>, smem);                                        \
    int chunks = 1;                                                                                             \
    while (chunks < kMaxChunks && N / (kGemvRowsPerCta * chunks) > cap && N % (kGemvRowsPerCta * chunks * 2) == 0) \
      chunks *= 2;                                                                                              \
    const int grid = N / (kGemvRowsPerCta * chunks);                                                            \
    KVS_CHECK_ARG(N % (kGemvRowsPerCta * chunks) == 0 && grid <= cap,                                           \
                  "gemv_allreduce: the grid does not fit on the GPU at once (peer waits need co-resident CTAs)"); \
    launch_pdl(gemv_allreduce_kernel<MM>, dim3(grid), dim3(kGemvThreads), smem, st, xp, x.stride(0), wp,          \
               w.stride(0), yp, y.stride(0), N, K, chunks, peers, int(rank), world, int(site), int(num_sites), ep, \
               stage_ld, uint64_t(timeout_ns), sp);                                                             \
    break;                                                                                                      \
  }
  switch (M) {
    KVS_GAR_CASE(1)
    KVS_GAR_CASE(2)
    KVS_GAR_CASE(3)
    KVS_GAR_CASE(4)
    KVS_GAR_CASE(5)
    KVS_GAR_CASE(6)
    KVS_GAR_CASE(7)
    KVS_GAR_CASE(8)
  }
#undef KVS_GAR_CASE
  KVS_CUDA_CHECK(cudaGetLastError());
}

void gemv_argmax_bf16(torch::Tensor x, torch::Tensor w, torch::Tensor out, torch::Tensor part_val,
                      torch::Tensor part_idx, torch::Tensor counter, int64_t vocab_begin,
                      std::vector<int64_t> slot_ptrs, int64_t rank, int64_t site,
                      int64_t num_sites, torch::Tensor epoch, int64_t timeout_ns, torch::Tensor status) {
  int M, K, N;
  check_gemv_args(x, w, M, K, N);
  const int grid = int(ceil_div(N, kGemvRowsPerCta));
  KVS_CHECK_ARG(out.is_cuda() && out.scalar_type() == at::kInt && out.numel() >= M, "gemv_argmax: out int32 [M]");
  KVS_CHECK_ARG(part_val.scalar_type() == at::kFloat && part_idx.scalar_type() == at::kInt &&
                    part_val.numel() >= int64_t(M) * grid && part_idx.numel() >= int64_t(M) * grid,
                "gemv_argmax: partial buffers [M * ceil(N / 16)]");
  KVS_CHECK_ARG(counter.scalar_type() == at::kInt && counter.numel() >= 1, "gemv_argmax: counter int32");
  const int world = slot_ptrs.empty() ? 1 : int(slot_ptrs.size());
  PeerTable peers{};
  if (world > 1) peers = make_table(slot_ptrs, world);
  KVS_CHECK_ARG(rank >= 0 && rank < world, "gemv_argmax: rank");
  const size_t smem = size_t(M) * K * 2;
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  auto xp = reinterpret_cast<const bf16*>(x.data_ptr());
  auto wp = reinterpret_cast<const bf16*>(w.data_ptr());
  const int32_t* ep = world > 1 ? reinterpret_cast<const int32_t*>(epoch.data_ptr()) : nullptr;
  auto sp = reinterpret_cast<uint32_t*>(status.data_ptr());
  auto pv = reinterpret_cast<float*>(part_val.data_ptr());
  auto pi = reinterpret_cast<int32_t*>(part_idx.data_ptr());
  auto cp = reinterpret_cast<uint32_t*>(counter.data_ptr());
  auto op = reinterpret_cast<int32_t*>(out.data_ptr());
#define KVS_GAM_CASE(MM)                                                                                       \
  case MM: {                                                                                                   \
    static bool set = false;                                                                                   \
    if (!set) {                                                                                                \
      KVS_CUDA_CHECK(cudaFuncSetAttribute(gemv_argmax_kernel<MM>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                          200 * 1024));                                                        \
      set = true;                                                                                              \
    }                                                                                                          \
    launch_pdl(gemv_argmax_kernel<MM>, dim3(grid), dim3(kGemvThreads), smem, st, xp, x.stride(0), wp,         \
               w.stride(0), N, K, int64_t(vocab_begin), pv, pi, cp, op, peers, int(rank), world, int(site),    \
               int(num_sites), ep, uint64_t(timeout_ns), sp);                                                  \
    break;                                                                                                     \
  }
  switch (M) {
    KVS_GAM_CASE(1)
    KVS_GAM_CASE(2)
    KVS_GAM_CASE(3)
    KVS_GAM_CASE(4)
    KVS_GAM_CASE(5)
    KVS_GAM_CASE(6)
    KVS_GAM_CASE(7)
    KVS_GAM_CASE(8)
  }
#undef KVS_GAM_CASE
  KVS_CUDA_CHECK(cudaGetLastError());
}

void decode_epoch_bump(torch::Tensor epoch) {
  KVS_CHECK_ARG(epoch.is_cuda() && epoch.scalar_type() == at::kInt, "decode_epoch_bump: int32 device tensor");
  decode_epoch_bump_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<int32_t*>(epoch.data_ptr()));
  KVS_CUDA_CHECK(cudaGetLastError());
}

}  // namespace kvs
