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
#include <algorithm>
#include <atomic>

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

// The row's outliers: each exact value replaces its code's contribution,
// acc += (value - decoded) * x (the fp32 subtraction rounds; a non-finite
// decoded weight gives a non-finite result, as it does without outliers).
__device__ __forceinline__ float outlier_terms(const int32_t* __restrict__ packed2,
                                               const int32_t* __restrict__ packed4,
                                               const __half* __restrict__ scales1,
                                               const int8_t* __restrict__ zeros1,
                                               const uint8_t* __restrict__ gp,
                                               const int32_t* __restrict__ row_ptrs,
                                               const int32_t* __restrict__ cols,
                                               const __half* __restrict__ vals, int64_t nnz,
                                               int64_t r, int64_t K, int ng,
                                               const __half* __restrict__ x, int lane) {
  float acc = 0.0f;
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
  return acc;
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
  acc += outlier_terms(packed2, packed4, scales1, zeros1, gp, row_ptrs, cols, vals, nnz, r, K,
                       ng, x, lane);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) y[r] = acc;
}

// Vector form (K = 16 ng, ng a multiple of 8, 16-byte aligned rows): lane l
// takes the 8 consecutive groups 8 l .. 8 l + 7 of each 256-group span of a
// row, so its code words (32 bytes), scales (16) and zeros (8) are three
// vector loads; 4-bit groups load their two words (8 bytes) under a
// predicate, and the decode selects per group without branching.  x sits in
// shared memory with 16 bytes of padding after every 128 columns, so the
// lanes' 256-byte spans start in different banks.  Warps stride over the
// rows; a CTA stages x and group_precision once.
constexpr int kQvSpan = 128;                        // columns per lane per 256-group span
constexpr int kQvPitch = kQvSpan * 2 + 16;          // bytes per padded 128-column block

__device__ __forceinline__ uint32_t decode_pair_sel(uint32_t w2, uint32_t w4a, uint32_t w4b,
                                                    bool four, int k, __half2 zh2,
                                                    __half2 sh2) {
  const uint32_t t4 = (k < 4 ? w4a : w4b) >> (8 * (k & 3));
  const uint32_t c4 = (t4 & 0xFu) | ((t4 << 12) & 0xF0000u);
  const uint32_t t2 = w2 >> (4 * k);
  const uint32_t c2 = (t2 & 0x3u) | ((t2 << 14) & 0x30000u);
  const uint32_t h = 0x64006400u | (four ? c4 : c2);
  const __half2 d = __hsub2(*reinterpret_cast<const __half2*>(&h), zh2);
  const __half2 w = __hmul2(d, sh2);
  return *reinterpret_cast<const uint32_t*>(&w);
}

__global__ void __launch_bounds__(256)
    qgemv_vec_kernel(const int32_t* __restrict__ packed2, const int32_t* __restrict__ packed4,
                     const __half* __restrict__ scales1, const int8_t* __restrict__ zeros1,
                     const uint8_t* __restrict__ gp, const int32_t* __restrict__ row_ptrs,
                     const int32_t* __restrict__ cols, const __half* __restrict__ vals,
                     int64_t nnz, int64_t M, int64_t K, int ng, const __half* __restrict__ x,
                     float* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t qsm[];
  uint8_t* xs = qsm;                                     // padded x
  uint8_t* gps = qsm + (size_t)(K / kQvSpan) * kQvPitch;  // group_precision
  const int tid = threadIdx.x, lane = tid & 31;
  for (int64_t c = tid; c < K / 8; c += blockDim.x)  // 16-byte chunks of x
    *reinterpret_cast<uint4*>(xs + (c >> 4) * kQvPitch + (c & 15) * 16) =
        reinterpret_cast<const uint4*>(x)[c];
  for (int g = tid; g < ng; g += blockDim.x) gps[g] = gp[g];
  __syncthreads();
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + tid) >> 5; r < M; r += nw) {
    float acc = 0.0f;
    for (int g0 = 8 * lane; g0 < ng; g0 += 256) {
      const int64_t si = r * ng + g0;
      const uint4 pa = reinterpret_cast<const uint4*>(packed2 + si)[0];
      const uint4 pb = reinterpret_cast<const uint4*>(packed2 + si)[1];
      const uint4 sc = *reinterpret_cast<const uint4*>(scales1 + si);
      const uint2 zr = *reinterpret_cast<const uint2*>(zeros1 + si);
      const uint2 pr = *reinterpret_cast<const uint2*>(gps + g0);
      const uint32_t w2[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
      const uint32_t sw[4] = {sc.x, sc.y, sc.z, sc.w};
      uint32_t w4a[8], w4b[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool four = ((q < 4 ? pr.x : pr.y) >> (8 * (q & 3))) & 0xFFu;
        uint2 v = make_uint2(0u, 0u);
        if (four) v = reinterpret_cast<const uint2*>(packed4)[si + q];
        w4a[q] = v.x;
        w4b[q] = v.y;
      }
      const uint8_t* xq = xs + (g0 >> 3) * kQvPitch;  // this lane's 128 columns
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const bool four = ((q < 4 ? pr.x : pr.y) >> (8 * (q & 3))) & 0xFFu;
        const uint32_t sbits = (sw[q >> 1] >> (16 * (q & 1))) & 0xFFFFu;
        const uint32_t ss = sbits * 0x00010001u;
        const __half2 sh2 = *reinterpret_cast<const __half2*>(&ss);
        const int z = (int)(int8_t)(((q < 4 ? zr.x : zr.y) >> (8 * (q & 3))) & 0xFFu);
        const uint32_t zb = (uint32_t)__half_as_ushort(__int2half_rn(1024 + z));  // exact
        const uint32_t zz = zb * 0x00010001u;
        const __half2 zh2 = *reinterpret_cast<const __half2*>(&zz);
        const uint4 xa = *reinterpret_cast<const uint4*>(xq + q * 32);
        const uint4 xb = *reinterpret_cast<const uint4*>(xq + q * 32 + 16);
        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int k = 0; k < 8; ++k)
          fma2_f16(decode_pair_sel(w2[q], w4a[q], w4b[q], four, k, zh2, sh2), xw[k], acc);
      }
    }
    acc += outlier_terms(packed2, packed4, scales1, zeros1, gps, row_ptrs, cols, vals, nnz, r, K,
                         ng, x, lane);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) y[r] = acc;
  }
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
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const size_t vsmem = (size_t)(K / kQvSpan) * kQvPitch + (size_t)ng;
  if (K == ng * kGroup1 && ng % 8 == 0 && x_vec && al16(packed_2bit) && al16(packed_4bit) &&
      al16(scales_1st_fp16) && (reinterpret_cast<uintptr_t>(zeros_1st) & 7u) == 0 &&
      vsmem <= 200 * 1024) {
    static std::atomic<uint64_t> attr_done{0};
    MB_CUDA_TRY(set_smem_limit_once(qgemv_vec_kernel, 200 * 1024, attr_done));
    int sms = 148, dev = 0;
    MB_CUDA_TRY(cudaGetDevice(&dev));
    MB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(M, 8), (int64_t)sms * 4));
    qgemv_vec_kernel<<<(unsigned)grid, 256, vsmem, stream>>>(
        packed_2bit, packed_4bit, static_cast<const __half*>(scales_1st_fp16), zeros_1st,
        group_precision, outlier_row_ptrs, outlier_col_indices,
        static_cast<const __half*>(outlier_values_fp16), nnz, M, K, (int)ng,
        static_cast<const __half*>(x_fp16), y);
    MB_LAUNCH_CHECK("qgemv_vec_kernel");
    return MB_OK;
  }
  qgemv_kernel<<<(unsigned)ceil_div(M * 32, 256), 256, 0, stream>>>(
      packed_2bit, packed_4bit, static_cast<const __half*>(scales_1st_fp16), zeros_1st,
      group_precision, outlier_row_ptrs, outlier_col_indices,
      static_cast<const __half*>(outlier_values_fp16), nnz, M, K, (int)ng,
      static_cast<const __half*>(x_fp16), x_vec, y);
  MB_LAUNCH_CHECK("qgemv_kernel");
  return MB_OK;
}
