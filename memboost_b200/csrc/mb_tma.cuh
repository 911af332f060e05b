// TMA (cp.async.bulk.tensor) and mbarrier helpers for sm_100a, plus the
// host-side tensor-map encoder.  Loads here never use cluster multicast.
//
// Every wait on an mbarrier is bounded by wall time (globaltimer): a wait
// that runs out returns false, and callers record an error status instead of
// spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

namespace mb {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to hint_ns while the phase is
// incomplete (the thread resumes as soon as it completes), instead of
// returning at once: waiting warps leave the issue slots to working ones.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// 2-D tiled TMA load of the box at (x = innermost coordinate, y) into shared
// memory, completing on `bar` (transaction bytes).  x * element size must be
// a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// L2 eviction-priority policies (createpolicy) for the cache-hinted copies
// below: lines loaded or stored under evict_last stay over normal and
// evict_first lines; evict_first lines are the first to go.
__device__ __forceinline__ uint64_t l2_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tma_load_2d with an L2 eviction policy for the loaded lines.
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 2-D tiled TMA store of the box at (x, y) from shared memory (bulk-group
// completion).  The writes to `src` must be made visible to the async proxy
// first (fence_proxy_async_smem by every writing thread, then a barrier).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x,
                                             int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}

// tma_store_2d with an L2 eviction policy for the written lines.
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, const void* src, int x,
                                                  int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint"
      " [%0, {%2, %3}], [%1], %4;" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N of this thread's committed bulk groups still read
// their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until at most N of this thread's committed bulk groups are pending.
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Programmatic dependent launch: wait for the preceding grid's memory.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Programmatic dependent launch: the next grid in the stream may begin
// launching (it still waits for this grid's completion in
// grid_dependency_wait before reading what this grid writes).
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- host ----

// cuTensorMapEncodeTiled from the driver, without linking libcuda.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Row-major [rows, cols] fp16 matrix, box [box_rows, box_cols], no swizzle,
// out-of-bounds elements read as zero.  Returns false if the driver rejects
// it (base must be 16-byte aligned and cols * 2 a multiple of 16).
bool make_tensor_map_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                            uint32_t box_rows, uint32_t box_cols);

// Row-major [rows, cols] matrix of a 16-bit type (fp16 or bf16), box
// [box_rows, box_cols] with the 128-byte swizzle (box_cols * 2 must be 128),
// out-of-bounds elements read as zero.
bool make_tensor_map_2d_16bit_sw128(CUtensorMap* map, const void* base, bool bf16, uint64_t rows,
                                    uint64_t cols, uint32_t box_rows, uint32_t box_cols);

// Row-major [rows, cols] matrix of 1-, 2- or 4-byte elements (elem_bytes),
// box [box_rows, box_cols], swizzle 0 (none), 32, 64 or 128 (bytes).  For TMA
// stores: elements outside the matrix are not written.  False if the driver
// rejects it (base 16-byte aligned, cols * elem_bytes a multiple of 16,
// box_cols * elem_bytes a multiple of 16 and at most the swizzle span).
bool make_tensor_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows,
                        uint64_t cols, uint32_t box_rows, uint32_t box_cols, int swizzle);

}  // namespace mb
