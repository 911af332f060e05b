// Hessian of the GPTQ calibration on sm_100a: H = alpha * X^T X, or
// H += alpha * X^T X -- the accumulation of models/llama.py:523-528 (forward
// hook: H_acc.add_(x.T @ x)) and the normalisation of llama.py:547-551
// (H.div_(total_tokens)), as a tcgen05 tensor-core GEMM.
//
// X [N tokens, K features] fp16 or bf16 is read by TMA in 32-token stages
// with the 128-byte swizzle; both GEMM operands are the same feature-major
// tiles ("MN-major" in UMMA terms) and the fp32 accumulators live in TMEM.
// One CTA owns a 256 x 256 tile of H as two 128 x 256 accumulators (all 512
// TMEM columns).  H is symmetric: only tiles on or below the diagonal are
// computed, each off-diagonal tile is also written transposed, and a diagonal
// tile loads X once for both operands.
#include <atomic>
#include <cmath>
#include <cstring>

#include "mb_common.cuh"
#include "mb_tma.cuh"

namespace mb {
namespace {

// ---------------------------------------------------------------------------
// Hessian: tcgen05 GEMM
// ---------------------------------------------------------------------------
constexpr int kHT = 256;                     // output tile edge (features)
constexpr int kHBK = 32;                     // tokens per pipeline stage
constexpr int kHStages = 6;
constexpr int kHBox = kHBK * 128;            // one TMA box: 32 tokens x 64 features x 2 B
constexpr int kHTile = (kHT / 64) * kHBox;   // one operand: 32 tokens x 256 features (16 KB)
constexpr int kHStage = 2 * kHTile;          // A and B
constexpr int kHSmem = kHStages * kHStage + 1024;  // + alignment slack
constexpr int kHTmemCols = 2 * kHT;          // two 128 x 256 fp32 accumulators
// Tokens per launch: bounds one CTA's main loop (and so the epilogue's wait
// on it) to a few tens of milliseconds; larger inputs take several launches.
constexpr int64_t kHMaxTokens = 1 << 20;

constexpr uint32_t kStatusHessianTimeout = 1u;

// UMMA shared-memory descriptor of a feature-major ("MN-major") operand
// written by TMA with the 128-byte swizzle: 64 features (128 B) per swizzle
// row, 8 tokens per 1024-byte swizzle atom.  LBO = distance between
// consecutive 64-feature boxes, SBO = distance between 8-token groups.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(((uint32_t)kHBox >> 4) & 0x3FFFu) << 16;  // LBO
  d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;            // SBO
  d |= (uint64_t)1 << 46;                                   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                                   // 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A/B fp16 (0) or bf16
// (1), both operands MN-major, M = 128, N = 256.
__host__ __device__ constexpr uint32_t hessian_idesc(uint32_t fmt) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (1u << 16) |
         ((uint32_t)(kHT >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Grid: one CTA per 256 x 256 tile (bi, bj) with bi >= bj, 128 threads.
// Warp 0 lane 0 issues the TMA loads, warp 1 lane 0 the MMAs; afterwards all
// four warps drain TMEM (warp w owns TMEM lanes 32w .. 32w + 31, i.e. rows
// 32w + lane of both accumulators).
__global__ void __launch_bounds__(128, 1)
    hessian_kernel(const __grid_constant__ CUtensorMap tmx, int64_t N, int64_t K, float alpha,
                   int accumulate, float* __restrict__ H, uint32_t* __restrict__ status,
                   uint32_t idesc) {
  extern __shared__ uint8_t hsm_raw[];
  uint8_t* hsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(hsm_raw) + 1023) &
                                            ~(uintptr_t)1023);
  __shared__ uint64_t full_bar[kHStages], empty_bar[kHStages], done_bar;
  __shared__ uint32_t tmem_slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tile (bi, bj), bi >= bj, from the linear lower-triangle index
  const int64_t t = blockIdx.x;
  int64_t bi = (int64_t)((sqrt(8.0 * (double)t + 1.0) - 1.0) * 0.5);
  while (bi * (bi + 1) / 2 > t) --bi;
  while ((bi + 1) * (bi + 2) / 2 <= t) ++bi;
  const int64_t bj = t - bi * (bi + 1) / 2;
  const int i0 = (int)(bi * kHT), j0 = (int)(bj * kHT);
  const bool diag = bi == bj;
  const int64_t nk = ceil_div(N, kHBK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kHStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&tmem_slot)),
                 "r"(kHTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  bool ok = true;

  if (warp == 0 && lane == 0) {
    // TMA producer
    const uint32_t tx = diag ? (uint32_t)kHTile : (uint32_t)kHStage;
    int64_t issued = 0;
    for (int64_t k = 0; k < nk; ++k) {
      const int s = (int)(k % kHStages);
      if (k >= kHStages && !mbar_wait(&empty_bar[s], (uint32_t)((k / kHStages - 1) & 1))) {
        ok = false;
        break;
      }
      uint8_t* a = hsm + (size_t)s * kHStage;
      const int y = (int)(k * kHBK);
      mbar_arrive_expect_tx(&full_bar[s], tx);
#pragma unroll
      for (int c = 0; c < kHT / 64; ++c)
        tma_load_2d(a + c * kHBox, &tmx, &full_bar[s], i0 + 64 * c, y);
      if (!diag) {
#pragma unroll
        for (int c = 0; c < kHT / 64; ++c)
          tma_load_2d(a + kHTile + c * kHBox, &tmx, &full_bar[s], j0 + 64 * c, y);
      }
      ++issued;
    }
    // every load this thread issued has landed before the CTA can exit
    for (int64_t k = issued > kHStages ? issued - kHStages : 0; k < issued; ++k)
      if (!mbar_wait(&full_bar[k % kHStages], (uint32_t)((k / kHStages) & 1))) ok = false;
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: per stage and 16-token step, D0 += A[0:128]^T B, D1 += A[128:256]^T B
    for (int64_t k = 0; k < nk; ++k) {
      const int s = (int)(k % kHStages);
      if (!mbar_wait(&full_bar[s], (uint32_t)((k / kHStages) & 1))) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a = smem_u32(hsm + (size_t)s * kHStage);
      const uint32_t b = diag ? a : a + kHTile;
#pragma unroll
      for (int kk = 0; kk < kHBK / 16; ++kk) {
        const uint32_t acc = (k > 0 || kk > 0) ? 1u : 0u;
        const uint64_t db = umma_desc_mn_sw128(b + kk * 2048);
        umma_f16(tmem, umma_desc_mn_sw128(a + kk * 2048), db, idesc, acc);
        umma_f16(tmem + kHT, umma_desc_mn_sw128(a + 2 * kHBox + kk * 2048), db, idesc, acc);
      }
      umma_commit(&empty_bar[s]);  // the stage is free once these MMAs complete
    }
    umma_commit(&done_bar);
  }
  __syncwarp();

  if (!mbar_wait(&done_bar, 0)) ok = false;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    const int64_t i = i0 + half * 128 + warp * 32 + lane;
#pragma unroll 1
    for (int cc = 0; cc < kHT / 16; ++cc) {
      uint32_t v[16];
      tmem_ld16(tmem + lane_base + (uint32_t)(half * kHT + cc * 16), v);
      const int64_t jb = j0 + cc * 16;
      if (i < K) {
        float* p = H + i * K + jb;
        if (jb + 16 <= K) {
#pragma unroll
          for (int e = 0; e < 16; e += 4) {
            float4 o = make_float4(__fmul_rn(alpha, __uint_as_float(v[e])),
                                   __fmul_rn(alpha, __uint_as_float(v[e + 1])),
                                   __fmul_rn(alpha, __uint_as_float(v[e + 2])),
                                   __fmul_rn(alpha, __uint_as_float(v[e + 3])));
            if (accumulate) {
              const float4 h = *reinterpret_cast<const float4*>(p + e);
              o.x = __fadd_rn(h.x, o.x);
              o.y = __fadd_rn(h.y, o.y);
              o.z = __fadd_rn(h.z, o.z);
              o.w = __fadd_rn(h.w, o.w);
            }
            *reinterpret_cast<float4*>(p + e) = o;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (jb + e < K) {
              const float val = __fmul_rn(alpha, __uint_as_float(v[e]));
              p[e] = accumulate ? __fadd_rn(p[e], val) : val;
            }
          }
        }
      }
      if (!diag) {
        // transposed copy: for each column j the warp writes 32 consecutive H[j][i]
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int64_t j = jb + e;
          if (i < K && j < K) {
            const float val = __fmul_rn(alpha, __uint_as_float(v[e]));
            float* q = H + j * K + i;
            *q = accumulate ? __fadd_rn(*q, val) : val;
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kHTmemCols));
  if (!ok && status) atomicOr(status, kStatusHessianTimeout);
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" mb_status mb_hessian(const void* X, int64_t N, int64_t K, int x_is_bf16, float alpha,
                                int accumulate, float* H, uint32_t* status_device,
                                mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(X != nullptr && H != nullptr, "null pointer");
  MB_REQUIRE(N > 0 && K > 0, "X must be a non-empty [N, K] matrix");
  MB_REQUIRE(K % 8 == 0, "K must be a multiple of 8 (16-byte rows for TMA)");
  MB_REQUIRE(K <= 65536, "K too large");
  MB_REQUIRE((reinterpret_cast<uintptr_t>(X) & 15u) == 0, "X must be 16-byte aligned");
  MB_REQUIRE((reinterpret_cast<uintptr_t>(H) & 15u) == 0, "H must be 16-byte aligned");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  static std::atomic<uint64_t> attr_done{0};
  MB_CUDA_TRY(set_smem_limit_once(hessian_kernel, kHSmem, attr_done));
  const int64_t kb = ceil_div(K, kHT);
  const int64_t tiles = kb * (kb + 1) / 2;
  const uint32_t idesc = hessian_idesc(x_is_bf16 ? 1u : 0u);
  const size_t row_bytes = (size_t)K * 2;
  for (int64_t n0 = 0; n0 < N; n0 += kHMaxTokens) {
    const int64_t n = min64(kHMaxTokens, N - n0);
    CUtensorMap tm;
    std::memset(&tm, 0, sizeof(tm));
    if (!make_tensor_map_2d_16bit_sw128(&tm,
                                        static_cast<const uint8_t*>(X) + (size_t)n0 * row_bytes,
                                        x_is_bf16 != 0, (uint64_t)n, (uint64_t)K, kHBK, 64))
      return set_error(MB_ERR_CUDA, "cuTensorMapEncodeTiled rejected X");
    hessian_kernel<<<(unsigned)tiles, 128, kHSmem, stream>>>(
        tm, n, K, alpha, (accumulate || n0 > 0) ? 1 : 0, H, status_device, idesc);
    MB_LAUNCH_CHECK("hessian_kernel");
  }
  return MB_OK;
}
