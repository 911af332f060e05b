// memboost pack / unpack on sm_100a -- replaces the host loops of
// pack_2bit_op / unpack_2bit_op / pack_4bit_op / unpack_4bit_op
// (core/torch_ops.cu:20-102).  Layout: element j of word i at bits
// [2j, 2j+2) (2-bit, 16 per word) or [4j, 4j+4) (4-bit, 8 per word); only the
// low 2 (4) bits of each input byte are kept.  One thread per packed word.
#include "mb_common.cuh"

namespace mb {
namespace {

template <int kBits>
__global__ void pack_kernel(const uint8_t* __restrict__ v, int64_t n_words,
                            int32_t* __restrict__ out) {
  constexpr int kPer = 32 / kBits;
  constexpr uint32_t kMask = (1u << kBits) - 1u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) word |= ((uint32_t)v[i * kPer + j] & kMask) << (j * kBits);
    out[i] = (int32_t)word;
  }
}

template <int kBits>
__global__ void unpack_kernel(const int32_t* __restrict__ p, int64_t n_words, int64_t n_out,
                              uint8_t* __restrict__ out) {
  constexpr int kPer = 32 / kBits;
  constexpr uint32_t kMask = (1u << kBits) - 1u;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_words;
       i += (int64_t)gridDim.x * blockDim.x) {
    if (i * kPer >= n_out) continue;
    const uint32_t word = (uint32_t)p[i];
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (i * kPer + j < n_out) out[i * kPer + j] = (uint8_t)((word >> (j * kBits)) & kMask);
  }
}

unsigned grid_for(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), 148 * 32)); }

template <int kBits>
mb_status pack_impl(const uint8_t* values, int64_t n_values, int32_t* packed, mb_stream_t s) {
  clear_error();
  constexpr int kPer = 32 / kBits;
  MB_REQUIRE(n_values >= 0 && n_values % kPer == 0,
             kBits == 2 ? "length must be multiple of 16" : "length must be multiple of 8");
  const int64_t n_words = n_values / kPer;
  if (n_words == 0) return MB_OK;
  MB_REQUIRE(values && packed, "null pointer");
  pack_kernel<kBits><<<grid_for(n_words), 256, 0, reinterpret_cast<cudaStream_t>(s)>>>(
      values, n_words, packed);
  MB_LAUNCH_CHECK("pack_kernel");
  return MB_OK;
}

template <int kBits>
mb_status unpack_impl(const int32_t* packed, int64_t n_words, int64_t num_elements,
                      uint8_t* values, mb_stream_t s) {
  clear_error();
  constexpr int kPer = 32 / kBits;
  MB_REQUIRE(num_elements <= n_words * kPer, "num_elements too large");
  MB_REQUIRE(num_elements >= 0 && n_words >= 0, "negative size");
  if (num_elements == 0) return MB_OK;
  MB_REQUIRE(values && packed, "null pointer");
  unpack_kernel<kBits><<<grid_for(n_words), 256, 0, reinterpret_cast<cudaStream_t>(s)>>>(
      packed, n_words, num_elements, values);
  MB_LAUNCH_CHECK("unpack_kernel");
  return MB_OK;
}

}  // namespace
}  // namespace mb

extern "C" mb_status mb_pack_2bit(const uint8_t* values, int64_t n_values, int32_t* packed,
                                  mb_stream_t stream) {
  return mb::pack_impl<2>(values, n_values, packed, stream);
}
extern "C" mb_status mb_unpack_2bit(const int32_t* packed, int64_t n_words, int64_t num_elements,
                                    uint8_t* values, mb_stream_t stream) {
  return mb::unpack_impl<2>(packed, n_words, num_elements, values, stream);
}
extern "C" mb_status mb_pack_4bit(const uint8_t* values, int64_t n_values, int32_t* packed,
                                  mb_stream_t stream) {
  return mb::pack_impl<4>(values, n_values, packed, stream);
}
extern "C" mb_status mb_unpack_4bit(const int32_t* packed, int64_t n_words, int64_t num_elements,
                                    uint8_t* values, mb_stream_t stream) {
  return mb::unpack_impl<4>(packed, n_words, num_elements, values, stream);
}
