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
//
// The weights are decoded two at a time in fp16 with the reference's result:
// q - zero is an integer of at most 143 in magnitude (exact in fp16, formed
// as (1024 + q) - (1024 + zero) from bit patterns), and scale * (q - zero)
// has at most 19 significant bits, so it is exact in fp32 and the
// reference's fp32 product rounded to fp16 equals one fp16 multiply.  Each
// product w * x is exact in fp32 and added with a single rounding
// (fma.rn.f32.f16), as fmaf on the converted values would.
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

// acc += lo(w) * lo(x) + hi(w) * hi(x) (two fp32 FMAs, fp16 operands)
__device__ __forceinline__ void fma2_f16(uint32_t w, uint32_t x, float& acc) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\t"
      "mov.b32 {wl, wh}, %1;\n\tmov.b32 {xl, xh}, %2;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\tfma.rn.f32.f16 %0, wh, xh, %0;\n\t}"
      : "+f"(acc)
      : "r"(w), "r"(x));
}

// Weights 2k and 2k + 1 of a group as fp16 pairs: codes from the packed
// word(s) as 1024 + q, minus 1024 + zero (zh2), times the scale (sh2).
__device__ __forceinline__ uint32_t decode_pair(uint32_t wa, uint32_t wb, bool four, int k,
                                                __half2 zh2, __half2 sh2) {
  uint32_t t, c;
  if (four) {
    t = (k < 4 ? wa : wb) >> (8 * (k & 3));
    c = (t & 0xFu) | ((t << 12) & 0xF0000u);
  } else {
    t = wa >> (4 * k);
    c = (t & 0x3u) | ((t << 14) & 0x30000u);
  }
  const uint32_t h = 0x64006400u | c;
  const __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&h), zh2);
  const __half2 w = __hmul2(d, sh2);
  return *reinterpret_cast<const uint32_t*>(&w);
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
    const __half sc = scales1[si];
    const __half2 sh2 = __halves2half2(sc, sc);
    const __half zh = __int2half_rn(1024 + (int)zeros1[si]);  // exact: 896 .. 1151
    const __half2 zh2 = __halves2half2(zh, zh);
    const int64_t c0 = (int64_t)g * kGroup1;
    const int gs = (int)min64(kGroup1, K - c0);
    uint32_t xw[8];
    if (x_vec && gs == kGroup1) {
      const uint4 a = reinterpret_cast<const uint4*>(x + c0)[0];
      const uint4 b = reinterpret_cast<const uint4*>(x + c0)[1];
      xw[0] = a.x; xw[1] = a.y; xw[2] = a.z; xw[3] = a.w;
      xw[4] = b.x; xw[5] = b.y; xw[6] = b.z; xw[7] = b.w;
    } else {  // a partial group or an unaligned x: x = 0 past K
      const uint16_t* xs = reinterpret_cast<const uint16_t*>(x) + c0;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        xw[k] = (2 * k < gs ? (uint32_t)xs[2 * k] : 0u) |
                (2 * k + 1 < gs ? (uint32_t)xs[2 * k + 1] << 16 : 0u);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t w = decode_pair(wa, wb, four, k, zh2, sh2);
      // weights past K: 0 (a non-finite weight times x = 0 would give NaN)
      if (2 * k >= gs) w &= 0xFFFF0000u;
      if (2 * k + 1 >= gs) w &= 0x0000FFFFu;
      fma2_f16(w, xw[k], acc);
    }
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
