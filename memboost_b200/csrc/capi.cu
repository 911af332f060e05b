// Error reporting and version of the memboost_b200 C ABI.
#include <string>

#include "mb_common.cuh"

namespace mb {
namespace {
thread_local std::string g_last_error;
}

mb_status set_error(mb_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

void clear_error() { g_last_error.clear(); }

}  // namespace mb

extern "C" const char* mb_last_error(void) { return mb::g_last_error.c_str(); }

extern "C" const char* mb_version(void) { return "memboost_b200 0.1.0 sm_100a"; }

// ---- tensor maps (declared in mb_tma.cuh) ----
#include "mb_tma.cuh"

namespace mb {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool make_tensor_map_2d_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                            uint32_t box_rows, uint32_t box_cols) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tensor_map_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows,
                        uint64_t cols, uint32_t box_rows, uint32_t box_cols, int swizzle) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * elem_bytes) % 16 != 0)
    return false;
  if ((box_cols * elem_bytes) % 16 != 0) return false;
  CUtensorMapDataType dt;
  switch (elem_bytes) {
    case 1: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case 2: dt = CU_TENSOR_MAP_DATA_TYPE_UINT16; break;
    case 4: dt = CU_TENSOR_MAP_DATA_TYPE_INT32; break;
    default: return false;
  }
  CUtensorMapSwizzle sw;
  switch (swizzle) {
    case 0: sw = CU_TENSOR_MAP_SWIZZLE_NONE; break;
    case 32: sw = CU_TENSOR_MAP_SWIZZLE_32B; break;
    case 64: sw = CU_TENSOR_MAP_SWIZZLE_64B; break;
    case 128: sw = CU_TENSOR_MAP_SWIZZLE_128B; break;
    default: return false;
  }
  if (swizzle != 0 && box_cols * (uint32_t)elem_bytes > (uint32_t)swizzle) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tensor_map_2d_16bit_sw128(CUtensorMap* map, const void* base, bool bf16, uint64_t rows,
                                    uint64_t cols, uint32_t box_rows, uint32_t box_cols) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0) return false;
  if (box_cols * 2 != 128) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace mb
