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
