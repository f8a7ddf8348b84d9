// Shared device/host helpers for the kvserve_b200 sm_100a kernels.
//
// Everything here is written for Blackwell (sm_100a): 32-lane warps,
// 148 SMs, up to 227 KB of shared memory per CTA, tcgen05 / TMEM / TMA.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <stdexcept>
#include <string>

namespace kvs {

using bf16 = __nv_bfloat16;

constexpr int kWarp = 32;
constexpr int kNumSMs = 148;

#define KVS_CUDA_CHECK(expr)                                                  \
  do {                                                                        \
    cudaError_t _e = (expr);                                                  \
    if (_e != cudaSuccess) {                                                  \
      throw std::runtime_error(std::string("CUDA error: ") +                  \
                               cudaGetErrorString(_e) + " at " + __FILE__ +   \
                               ":" + std::to_string(__LINE__));               \
    }                                                                         \
  } while (0)

#define KVS_CHECK_ARG(cond, msg)                                   \
  do {                                                             \
    if (!(cond)) throw std::invalid_argument(std::string(msg));    \
  } while (0)

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

__device__ __forceinline__ float to_f32(bf16 v) { return __bfloat162float(v); }
// Round-to-nearest-even float -> bf16 (the cvt.rn.bf16.f32 instruction).
__device__ __forceinline__ bf16 rn(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float rnf(float v) { return to_f32(rn(v)); }

// ---------------------------------------------------------------------------
// Ordered-integer encoding of floats so that min/max reductions across CTAs
// can use integer atomics (monotone map: a < b  <=>  enc(a) < enc(b)).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t float_to_ordered(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// ---------------------------------------------------------------------------
// Memory-ordering helpers for peer (NVLink) signalling.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t atom_add_release_sys_u32(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.release.sys.global.u32 %0, [%1], %2;"
               : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu_u32(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;"
               : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for a 32-bit flag to reach at least `target` (wrap-safe
// comparison).  Returns true on success, false when `timeout_ns` elapsed.
// Never traps and never spins forever.
__device__ __forceinline__ bool wait_flag_geq(const uint32_t* flag, uint32_t target,
                                              uint64_t timeout_ns) {
  const uint64_t start = globaltimer_ns();
  uint32_t sleep_ns = 32;
  while (true) {
    const uint32_t v = ld_acquire_sys_u32(flag);
    if (static_cast<int32_t>(v - target) >= 0) return true;
    if (globaltimer_ns() - start > timeout_ns) return false;
    __nanosleep(sleep_ns);
    if (sleep_ns < 1024) sleep_ns <<= 1;
  }
}

// Low-latency ("LL") peer words: a 64-bit word whose high half is a flag and
// whose low half is a 32-bit payload.  A naturally aligned 64-bit access is
// single-copy atomic, so a reader that sees the expected flag also sees the
// payload written with it: no fence and no separate flag word are needed.
__device__ __forceinline__ void st_ll(uint64_t* p, uint32_t payload, uint32_t flag) {
  const uint64_t v = (uint64_t(flag) << 32) | payload;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Bounded poll of an LL word until its flag reaches `flag` (wrap-safe);
// returns the payload, or sets `ok` false after `deadline_ns` (globaltimer).
__device__ __forceinline__ uint32_t poll_ll(const uint64_t* p, uint32_t flag, uint64_t deadline_ns, bool& ok) {
  for (int it = 0;; ++it) {
    const uint64_t v = ld_ll(p);
    if (static_cast<int32_t>(uint32_t(v >> 32) - flag) >= 0) return uint32_t(v);
    if ((it & 63) == 63 && globaltimer_ns() > deadline_ns) {
      ok = false;
      return 0u;
    }
  }
}

// Hand-off trace stamps (%globaltimer ns), four per layer: encode start,
// frame published, ingest start (first CTA past the layer's flag), ingest
// end.  Starts are stored as ~t with atomicMax (the earliest CTA wins), ends
// as t with atomicMax; a zeroed buffer means "not stamped".  Null = off.
__device__ __forceinline__ void trace_start(uint64_t* tr) {
  if (tr != nullptr) atomicMax(reinterpret_cast<unsigned long long*>(tr), ~(unsigned long long)globaltimer_ns());
}
__device__ __forceinline__ void trace_end(uint64_t* tr) {
  if (tr != nullptr) atomicMax(reinterpret_cast<unsigned long long*>(tr), (unsigned long long)globaltimer_ns());
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL).  A kernel launched with the PDL
// attribute may start while its predecessor in the stream is still running;
// it must call pdl_wait() before it reads anything the predecessor wrote
// (griddepcontrol.wait returns once the predecessor grid has completed and
// its memory is visible).  pdl_trigger() lets the dependent launch early; a
// dependent launched without the attribute still waits for completion, so
// triggering is always safe.  Decode-step kernels trigger at entry and the
// weight-streaming GEMVs are PDL launches that prefetch their weights before
// waiting, which hides the launch gap between consecutive kernels.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// KVSERVE_PDL=0 turns the PDL attribute off (A/B measurements).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  KVS_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}

// Status codes written by kernels into a device status word.
enum Status : uint32_t {
  kStatusOk = 0,
  kStatusTimeout = 1,
  kStatusBadHeader = 2,
  kStatusBadSymbol = 3,
  kStatusBadSize = 4,
  kStatusPeerTimeout = 5,  // a tensor-parallel peer's tile or flag did not arrive in time
};

}  // namespace kvs
