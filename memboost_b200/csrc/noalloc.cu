// Quantize without any device allocation by this library or by the caller.
//
// Some callers cannot hand the library a workspace: a C or C++ host that
// links only this library (no torch caching allocator) and runs where
// every byte of device memory is owned by its own fixed arena, or a latency
// path that must never reach cudaMalloc / cudaFree (both can synchronise
// the whole device).  For them, mb_quantize_noalloc keeps its scratch in one
// statically sized device array that exists, once per GPU, for as long as
// the library is loaded.
//
// Rules that follow from that single shared array:
//   * the scratch holds at most MB_NOALLOC_SCRATCH_BYTES; larger matrices are
//     rejected (use mb_quantize with a caller workspace for those),
//   * every call reuses the array and it keeps the previous call's contents;
//     the pipeline clears what must start at zero on every call,
//   * two calls whose GPU work overlaps (different streams, different host
//     threads) race on the array and corrupt each other's results -- order
//     them on one stream or synchronise between them,
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress with that device current); make that first call
//     before any stream capture.
#include <mutex>

#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kMaxDevices = 64;

// The scratch array.  In host code this name is only a stand-in: its device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MB_NOALLOC_SCRATCH_BYTES];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
mb_status scratch_address(void** out) {
  int dev = 0;
  MB_CUDA_TRY(cudaGetDevice(&dev));
  MB_REQUIRE(dev >= 0 && dev < kMaxDevices, "device ordinal too large for the static scratch table");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    MB_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return MB_OK;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" mb_status mb_quantize_noalloc(
    const void* weights_fp16, int64_t M, int64_t K, double ratio_4bit, const float* hessian_diag,
    int64_t hessian_numel, int32_t* packed_2bit, int32_t* packed_4bit, void* scales_1st_fp16,
    int8_t* zeros_1st, void* scales_2nd_fp16, int8_t* zeros_2nd, uint8_t* scales_1st_quant,
    uint8_t* group_precision, int32_t* outlier_row_ptrs, int32_t* nnz_device,
    void* outlier_values_fp16, int32_t* outlier_col_indices, int64_t outlier_capacity,
    int64_t* nnz_host, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(M > 0 && K > 0, "weights must be a non-empty 2D [M, K] matrix");
  MB_REQUIRE(nnz_host != nullptr, "nnz_host must not be null");
  const size_t need = mb_quantize_workspace_size(M, K);
  if (need > (size_t)MB_NOALLOC_SCRATCH_BYTES)
    return set_error(MB_ERR_INVALID_ARGUMENT,
                     "matrix too large for mb_quantize_noalloc: it needs " +
                         std::to_string(need) + " bytes of scratch, the static array holds " +
                         std::to_string((size_t)MB_NOALLOC_SCRATCH_BYTES) +
                         "; use mb_quantize with a caller workspace");
  void* ws = nullptr;
  if (mb_status st = scratch_address(&ws)) return st;
  if (mb_status st = mb_quantize(weights_fp16, M, K, ratio_4bit, hessian_diag, hessian_numel,
                                 packed_2bit, packed_4bit, scales_1st_fp16, zeros_1st,
                                 scales_2nd_fp16, zeros_2nd, scales_1st_quant, group_precision,
                                 outlier_row_ptrs, nnz_device, ws, MB_NOALLOC_SCRATCH_BYTES,
                                 stream_))
    return st;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  int32_t nnz = 0;
  MB_CUDA_TRY(cudaMemcpyAsync(&nnz, nnz_device, sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
  MB_CUDA_TRY(cudaStreamSynchronize(stream));
  *nnz_host = nnz;
  if (nnz == 0) return MB_OK;
  if (nnz > outlier_capacity)
    return set_error(MB_ERR_INVALID_ARGUMENT,
                     "outlier capacity too small: " + std::to_string(nnz) +
                         " outliers, capacity " + std::to_string(outlier_capacity) +
                         " (every output except the CSR values and columns is valid)");
  return mb_quantize_extract_outliers(weights_fp16, M, K, outlier_row_ptrs, outlier_values_fp16,
                                      outlier_col_indices, ws, MB_NOALLOC_SCRATCH_BYTES, stream_);
}
