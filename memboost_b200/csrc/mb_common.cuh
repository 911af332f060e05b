// Shared helpers for the memboost_b200 sm_100a kernels and their C-ABI
// wrappers: error reporting, launch checks and small device utilities.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <string>

#include "memboost_b200.h"

namespace mb {

constexpr int kGroup1 = 16;   // 1st-order group width (columns)
constexpr int kGroup2 = 256;  // 2nd-order group length (flattened scales)

// Records `msg` as the calling thread's last error and returns `st`.
mb_status set_error(mb_status st, const std::string& msg);
void clear_error();

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ inline int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

#define MB_CUDA_TRY(expr)                                                             \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    if (_e != cudaSuccess)                                                            \
      return ::mb::set_error(MB_ERR_CUDA, std::string("CUDA error: ") +               \
                                              cudaGetErrorString(_e) + " at " #expr); \
  } while (0)

#define MB_LAUNCH_CHECK(name)                                                            \
  do {                                                                                   \
    cudaError_t _e = cudaGetLastError();                                                 \
    if (_e != cudaSuccess)                                                               \
      return ::mb::set_error(MB_ERR_CUDA, std::string("CUDA error: ") +                  \
                                              cudaGetErrorString(_e) + " launching " name); \
  } while (0)

// Raises `func`'s dynamic shared-memory limit to `bytes` once per device
// (the attribute belongs to the device context); `done` is one bit per
// device ordinal, owned by the caller (one per kernel instantiation).
template <typename F>
inline cudaError_t set_smem_limit_once(F* func, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// Resident blocks per SM of `func` (threads, dynamic shared memory) on the
// current device, queried once per device and kept in `cache` (one slot per
// device; 0 = not yet known).  Also raises the dynamic shared-memory limit.
template <typename F>
inline cudaError_t blocks_per_sm_once(F* func, int threads, int smem, std::atomic<int>* cache,
                                      int ncache, int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < ncache) {
    const int v = cache[dev].load(std::memory_order_acquire);
    if (v > 0) {
      *out = v;
      return cudaSuccess;
    }
  }
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, func, threads, smem);
  if (e != cudaSuccess) return e;
  per_sm = per_sm > 0 ? per_sm : 1;
  if (dev < ncache) cache[dev].store(per_sm, std::memory_order_release);
  *out = per_sm;
  return cudaSuccess;
}

#define MB_REQUIRE(cond, msg)                                                  \
  do {                                                                         \
    if (!(cond)) return ::mb::set_error(MB_ERR_INVALID_ARGUMENT, (msg));       \
  } while (0)

// ---- device helpers ----

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// float -> int32 with the semantics of a C cast compiled for the GPU
// (cvt.rzi.s32.f32: truncate, saturate, NaN -> 0).
__device__ __forceinline__ int f2i_rz(float x) { return __float2int_rz(x); }

}  // namespace mb

namespace mb {

// ---- packed fp32 pairs (sm_100 f32x2 arithmetic, round-to-nearest) ----
// A pair lives in one 64-bit register: element 0 in the low half.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// w * w of an fp16 value as an fp32 (exact: the product has <= 22 bits)
__device__ __forceinline__ float f16_square(uint16_t h) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %1, %2;" : "=f"(d) : "h"(h), "f"(0.0f));
  return d;
}

}  // namespace mb
