// memboost dequantize on sm_100a -- replaces dequantize_weights_kernel
// (core/quantize.cu:386-444) and dequantize_op (core/torch_ops.cu:267-301).
//
// One thread per (row, 16-column group): one or two packed words in, 32 bytes
// of fp16 out as two 16-byte stores.  Per element, the reference's
//   out = __float2half(float(scale) * ((float)q - (float)zero))
// with the subtraction and the product rounded separately (no outlier
// add-back, 2nd-order fields unused -- as in the reference).
//
// mb_dequantize_2nd (no counterpart in the reference, which computes
// scales_1st_quant / scales_2nd / zeros_2nd in core/quantize.cu:245-280 but
// never reads them back) rebuilds every group's scale from its 4-bit
// 2nd-order code by the same rule one level up,
//   s = fp16(float(scales_2nd[c]) * ((float)q2 - (float)zeros_2nd[c])),
//   q2 = scales_1st_quant[r, g], c = (r ng + g) / 256,
// decodes the weights with s in place of scales_1st, and can write the CSR
// outliers back (their exact fp16 values) -- the weights a consumer of the
// compact format (codes, 4-bit scale codes, per-chunk scales) sees.
#include "mb_common.cuh"

namespace mb {
namespace {

// kSecond: the scale from the 2nd-order code (sq, scales2, zeros2) instead of
// scales1.
template <bool kSecond>
__global__ void __launch_bounds__(128)
    dequantize_kernel(const int32_t* __restrict__ packed2, const int32_t* __restrict__ packed4,
                      const __half* __restrict__ scales1, const int8_t* __restrict__ zeros1,
                      const uint8_t* __restrict__ sq, const __half* __restrict__ scales2,
                      const int8_t* __restrict__ zeros2, const uint8_t* __restrict__ gp,
                      int64_t M, int64_t K, int ng, bool out_aligned, __half* __restrict__ out) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ng) return;
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, K - c0);
  const bool vec = out_aligned && (gs == kGroup1) && ((K & 7) == 0);
  const bool four = gp[g] != 0;
  for (int64_t r = blockIdx.y; r < M; r += gridDim.y) {
    const int64_t si = r * ng + g;
    float scale;
    if (kSecond) {
      const int64_t c = si / kGroup2;
      const float s = __fmul_rn(__half2float(scales2[c]),
                                __fsub_rn((float)sq[si], (float)(int)zeros2[c]));
      scale = __half2float(__float2half_rn(s));
    } else {
      scale = __half2float(scales1[si]);
    }
    const float zf = (float)(int)zeros1[si];
    uint32_t wa, wb = 0;
    if (four) {
      const int2 w = reinterpret_cast<const int2*>(packed4)[si];
      wa = (uint32_t)w.x;
      wb = (uint32_t)w.y;
    } else {
      wa = (uint32_t)packed2[si];
    }
    uint32_t h[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      uint32_t pair = 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * k + e;
        uint32_t q;
        if (!four)
          q = (wa >> (2 * i)) & 0x3u;
        else
          q = ((i < 8 ? wa : wb) >> (4 * (i & 7))) & 0xFu;
        const float v = __fmul_rn(scale, __fsub_rn((float)q, zf));
        pair |= (uint32_t)__half_as_ushort(__float2half_rn(v)) << (16 * e);
      }
      h[k] = pair;
    }
    __half* o = out + r * K + c0;
    if (vec) {
      reinterpret_cast<uint4*>(o)[0] = make_uint4(h[0], h[1], h[2], h[3]);
      reinterpret_cast<uint4*>(o)[1] = make_uint4(h[4], h[5], h[6], h[7]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < gs) o[i] = __ushort_as_half((uint16_t)(h[i >> 1] >> (16 * (i & 1))));
    }
  }
}

// out[r, col] = value for every CSR outlier, one warp per row; entries past
// nnz and columns outside [0, K) are skipped.
__global__ void __launch_bounds__(256)
    outlier_writeback_kernel(const int32_t* __restrict__ row_ptrs,
                             const int32_t* __restrict__ cols, const __half* __restrict__ vals,
                             int64_t nnz, int64_t M, int64_t K, __half* __restrict__ out) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= M) return;
  const int64_t j0 = max64(0, row_ptrs[r]), j1 = min64(nnz, row_ptrs[r + 1]);
  for (int64_t j = j0 + lane; j < j1; j += 32) {
    const int64_t col = cols[j];
    if (col >= 0 && col < K) out[r * K + col] = vals[j];
  }
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" mb_status mb_dequantize(const int32_t* packed_2bit, const int32_t* packed_4bit,
                                   const void* scales_1st_fp16, const int8_t* zeros_1st,
                                   const uint8_t* group_precision, int64_t M, int64_t K,
                                   void* out_fp16, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(packed_2bit && packed_4bit && scales_1st_fp16 && zeros_1st && group_precision &&
                 out_fp16,
             "dequantize pointers must not be null");
  MB_REQUIRE(M > 0 && K > 0, "M and K must be positive");
  const int64_t ng = ceil_div(K, kGroup1);
  MB_REQUIRE((reinterpret_cast<uintptr_t>(packed_4bit) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(packed_2bit) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_1st_fp16) & 1u) == 0,
             "misaligned packed_4bit / packed_2bit / scales_1st pointer");
  const bool out_aligned = (reinterpret_cast<uintptr_t>(out_fp16) & 15u) == 0;
  MB_REQUIRE((reinterpret_cast<uintptr_t>(out_fp16) & 1u) == 0, "misaligned output pointer");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  dim3 grid((unsigned)ceil_div(ng, 128), (unsigned)std::min<int64_t>(M, 65535));
  dequantize_kernel<false><<<grid, 128, 0, stream>>>(
      packed_2bit, packed_4bit, static_cast<const __half*>(scales_1st_fp16), zeros_1st, nullptr,
      nullptr, nullptr, group_precision, M, K, (int)ng, out_aligned,
      static_cast<__half*>(out_fp16));
  MB_LAUNCH_CHECK("dequantize_kernel");
  return MB_OK;
}

extern "C" mb_status mb_dequantize_2nd(const int32_t* packed_2bit, const int32_t* packed_4bit,
                                       const uint8_t* scales_1st_quant,
                                       const void* scales_2nd_fp16, const int8_t* zeros_2nd,
                                       const int8_t* zeros_1st, const uint8_t* group_precision,
                                       const int32_t* outlier_row_ptrs,
                                       const int32_t* outlier_col_indices,
                                       const void* outlier_values_fp16, int64_t nnz, int64_t M,
                                       int64_t K, void* out_fp16, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(packed_2bit && packed_4bit && scales_1st_quant && scales_2nd_fp16 && zeros_2nd &&
                 zeros_1st && group_precision && out_fp16,
             "dequantize pointers must not be null");
  MB_REQUIRE(M > 0 && K > 0, "M and K must be positive");
  MB_REQUIRE(nnz >= 0, "nnz must not be negative");
  MB_REQUIRE(nnz == 0 || (outlier_row_ptrs && outlier_col_indices && outlier_values_fp16),
             "outlier CSR pointers must not be null when nnz > 0");
  const int64_t ng = ceil_div(K, kGroup1);
  MB_REQUIRE((reinterpret_cast<uintptr_t>(packed_4bit) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(packed_2bit) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_2nd_fp16) & 1u) == 0,
             "misaligned packed_4bit / packed_2bit / scales_2nd pointer");
  const bool out_aligned = (reinterpret_cast<uintptr_t>(out_fp16) & 15u) == 0;
  MB_REQUIRE((reinterpret_cast<uintptr_t>(out_fp16) & 1u) == 0, "misaligned output pointer");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  dim3 grid((unsigned)ceil_div(ng, 128), (unsigned)std::min<int64_t>(M, 65535));
  dequantize_kernel<true><<<grid, 128, 0, stream>>>(
      packed_2bit, packed_4bit, nullptr, zeros_1st, scales_1st_quant,
      static_cast<const __half*>(scales_2nd_fp16), zeros_2nd, group_precision, M, K, (int)ng,
      out_aligned, static_cast<__half*>(out_fp16));
  MB_LAUNCH_CHECK("dequantize_kernel<2nd>");
  if (nnz > 0) {
    outlier_writeback_kernel<<<(unsigned)ceil_div(M * 32, 256), 256, 0, stream>>>(
        outlier_row_ptrs, outlier_col_indices, static_cast<const __half*>(outlier_values_fp16),
        nnz, M, K, static_cast<__half*>(out_fp16));
    MB_LAUNCH_CHECK("outlier_writeback_kernel");
  }
  return MB_OK;
}
