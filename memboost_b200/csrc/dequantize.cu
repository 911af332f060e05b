// memboost dequantize on sm_100a -- replaces dequantize_weights_kernel
// (core/quantize.cu:386-444) and dequantize_op (core/torch_ops.cu:267-301).
//
// One thread per (row, 16-column group): one or two packed words in, 32 bytes
// of fp16 out as two 16-byte stores.  Per element, the reference's
//   out = __float2half(float(scale) * ((float)q - (float)zero))
// with the subtraction and the product rounded separately (no outlier
// add-back, 2nd-order fields unused -- as in the reference).
#include "mb_common.cuh"

namespace mb {
namespace {

__global__ void __launch_bounds__(128)
    dequantize_kernel(const int32_t* __restrict__ packed2, const int32_t* __restrict__ packed4,
                      const __half* __restrict__ scales1, const int8_t* __restrict__ zeros1,
                      const uint8_t* __restrict__ gp, int64_t M, int64_t K, int ng,
                      bool out_aligned, __half* __restrict__ out) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ng) return;
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, K - c0);
  const bool vec = out_aligned && (gs == kGroup1) && ((K & 7) == 0);
  const bool four = gp[g] != 0;
  for (int64_t r = blockIdx.y; r < M; r += gridDim.y) {
    const int64_t si = r * ng + g;
    const float scale = __half2float(scales1[si]);
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
  dequantize_kernel<<<grid, 128, 0, stream>>>(packed_2bit, packed_4bit,
                                              static_cast<const __half*>(scales_1st_fp16),
                                              zeros_1st, group_precision, M, K, (int)ng,
                                              out_aligned, static_cast<__half*>(out_fp16));
  MB_LAUNCH_CHECK("dequantize_kernel");
  return MB_OK;
}
