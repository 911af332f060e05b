// Quantized GEMV on sm_100a (no counterpart in the reference, which has no
// matmul over its format): y[r] = sum_c W[r, c] x[c] in fp32, where W is the
// reference dequantization of the codes (core/quantize.cu:386-444: per
// element fp16(float(scale) * ((float)q - (float)zero)), the subtraction and
// the product rounded separately) with every CSR outlier's exact fp16 value
// in place of its code's.  The packed words are read directly, never
// expanded to fp16 in memory: 0.44 bytes a weight for a 2-bit group (code
// word, scale, zero) against 2 for an fp16 matrix.
//
// One warp per row, lanes over the row's 16-column groups; then the row's
// outliers replace their codes' contributions (exact value minus decoded
// value, times x); a warp sum gives y[r].
#include "mb_common.cuh"

namespace mb {
namespace {

// Weight i (0..15) of a group: code from the packed word(s), then the
// reference's rounding.
__device__ __forceinline__ float decode_one(uint32_t wa, uint32_t wb, bool four, float scale,
                                            float zf, int i) {
  const uint32_t q = four ? (((i < 8 ? wa : wb) >> (4 * (i & 7))) & 0xFu) : ((wa >> (2 * i)) & 0x3u);
  return __half2float(__float2half_rn(__fmul_rn(scale, __fsub_rn((float)q, zf))));
}

__device__ __forceinline__ void load_group(const int32_t* __restrict__ packed2,
                                           const int32_t* __restrict__ packed4, bool four,
                                           int64_t si, uint32_t& wa, uint32_t& wb) {
  if (four) {
    const int2 w = reinterpret_cast<const int2*>(packed4)[si];
    wa = (uint32_t)w.x;
    wb = (uint32_t)w.y;
  } else {
    wa = (uint32_t)packed2[si];
    wb = 0u;
  }
}

__global__ void __launch_bounds__(256)
    qgemv_kernel(const int32_t* __restrict__ packed2, const int32_t* __restrict__ packed4,
                 const __half* __restrict__ scales1, const int8_t* __restrict__ zeros1,
                 const uint8_t* __restrict__ gp, const int32_t* __restrict__ row_ptrs,
                 const int32_t* __restrict__ cols, const __half* __restrict__ vals, int64_t nnz,
                 int64_t M, int64_t K, int ng, const __half* __restrict__ x, bool x_vec,
                 float* __restrict__ y) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= M) return;  // whole warps: blockDim is a multiple of 32
  float acc = 0.0f;
  for (int g = lane; g < ng; g += 32) {
    const int64_t si = r * ng + g;
    const bool four = gp[g] != 0;
    uint32_t wa, wb;
    load_group(packed2, packed4, four, si, wa, wb);
    const float scale = __half2float(scales1[si]);
    const float zf = (float)(int)zeros1[si];
    const int64_t c0 = (int64_t)g * kGroup1;
    const int gs = (int)min64(kGroup1, K - c0);
    float xv[16];
    if (x_vec && gs == kGroup1) {
      const uint4 a = reinterpret_cast<const uint4*>(x + c0)[0];
      const uint4 b = reinterpret_cast<const uint4*>(x + c0)[1];
      const uint32_t h[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        xv[2 * k] = __half2float(__ushort_as_half((uint16_t)(h[k] & 0xFFFFu)));
        xv[2 * k + 1] = __half2float(__ushort_as_half((uint16_t)(h[k] >> 16)));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) xv[i] = i < gs ? __half2float(x[c0 + i]) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < gs) acc = fmaf(decode_one(wa, wb, four, scale, zf, i), xv[i], acc);
  }
  // the row's outliers: their exact values in place of the decoded ones
  const int64_t j0 = max64(0, row_ptrs[r]), j1 = min64(nnz, row_ptrs[r + 1]);
  for (int64_t j = j0 + lane; j < j1; j += 32) {
    const int64_t col = cols[j];
    if (col < 0 || col >= K) continue;
    const int g = (int)(col >> 4), i = (int)(col & 15);
    const int64_t si = r * ng + g;
    const bool four = gp[g] != 0;
    uint32_t wa, wb;
    load_group(packed2, packed4, four, si, wa, wb);
    const float wq = decode_one(wa, wb, four, __half2float(scales1[si]),
                                (float)(int)zeros1[si], i);
    acc = fmaf(__half2float(vals[j]) - wq, __half2float(x[col]), acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) y[r] = acc;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" mb_status mb_qgemv(const int32_t* packed_2bit, const int32_t* packed_4bit,
                              const void* scales_1st_fp16, const int8_t* zeros_1st,
                              const uint8_t* group_precision, const int32_t* outlier_row_ptrs,
                              const int32_t* outlier_col_indices, const void* outlier_values_fp16,
                              int64_t nnz, int64_t M, int64_t K, const void* x_fp16, float* y,
                              mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(packed_2bit && packed_4bit && scales_1st_fp16 && zeros_1st && group_precision &&
                 outlier_row_ptrs && x_fp16 && y,
             "qgemv pointers must not be null");
  MB_REQUIRE(M > 0 && K > 0, "M and K must be positive");
  MB_REQUIRE(nnz >= 0, "nnz must not be negative");
  MB_REQUIRE(nnz == 0 || (outlier_col_indices && outlier_values_fp16),
             "outlier CSR pointers must not be null when nnz > 0");
  MB_REQUIRE((reinterpret_cast<uintptr_t>(packed_4bit) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(packed_2bit) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_1st_fp16) & 1u) == 0 &&
                 (reinterpret_cast<uintptr_t>(x_fp16) & 1u) == 0 &&
                 (reinterpret_cast<uintptr_t>(y) & 3u) == 0,
             "misaligned packed_4bit / packed_2bit / scales_1st / x / y pointer");
  const int64_t ng = ceil_div(K, kGroup1);
  const bool x_vec = (reinterpret_cast<uintptr_t>(x_fp16) & 15u) == 0;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  qgemv_kernel<<<(unsigned)ceil_div(M * 32, 256), 256, 0, stream>>>(
      packed_2bit, packed_4bit, static_cast<const __half*>(scales_1st_fp16), zeros_1st,
      group_precision, outlier_row_ptrs, outlier_col_indices,
      static_cast<const __half*>(outlier_values_fp16), nnz, M, K, (int)ng,
      static_cast<const __half*>(x_fp16), x_vec, y);
  MB_LAUNCH_CHECK("qgemv_kernel");
  return MB_OK;
}
