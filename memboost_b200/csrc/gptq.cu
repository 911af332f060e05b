// GPTQ blockwise quantization on sm_100a: gptq_quantize of the reference
// (models/llama.py:234-294).  Per-group parameters come from the original W;
// then for every (row, 128-column block) the sequential column-by-column
// rounding with the intra-block error update runs in the reference's fp32
// operation order, so Q is bit-identical to the reference's.
#include <atomic>
#include <cmath>

#include "mb_common.cuh"

namespace mb {
namespace {

// ---------------------------------------------------------------------------
// GPTQ block update
// ---------------------------------------------------------------------------
struct __align__(32) GptqGroup {
  float gmin;    // min of the group's original weights (torch min: NaN propagates)
  float sc;      // (gmax - gmin) / (L - 1) in double, stored as fp32; 0 unless gmax > gmin
  float rsc;     // fp32 1 / sc (the divisor PyTorch's CUDA scalar division multiplies by)
  float zero_f;  // round_half_even(-gmin / sc) in double, as the fp32 operand of the subtraction
  float lmax;    // L - 1
  float pad[3];
};

// Per-group parameters -- llama.py:252-263: min/max of W[:, 16g:16g+16]
// (.item() -> Python float), the scale in Python double arithmetic stored into
// an fp32 tensor, and zero = round(-gmin / sc) (llama.py:279) in double.
__global__ void __launch_bounds__(256)
    gptq_group_kernel(const float* __restrict__ W, int64_t M, int64_t K,
                      const uint8_t* __restrict__ gp, GptqGroup* __restrict__ out) {
  const int g = blockIdx.x;
  float mn = INFINITY, mx = -INFINITY;
  bool nan = false;
  for (int64_t idx = threadIdx.x; idx < M * kGroup1; idx += blockDim.x) {
    const int64_t r = idx >> 4;
    const float v = W[r * K + (int64_t)g * kGroup1 + (idx & 15)];
    nan |= isnan(v);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  mn = warp_min(mn);
  mx = warp_max(mx);
  nan = __any_sync(0xffffffffu, nan);
  __shared__ float smn[8], smx[8];
  __shared__ int snan[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    smn[warp] = mn;
    smx[warp] = mx;
    snan[warp] = nan;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
      mn = fminf(mn, smn[w]);
      mx = fmaxf(mx, smx[w]);
      nan |= snan[w] != 0;
    }
    if (nan) mn = mx = __int_as_float(0x7fc00000);
    const int L = gp[g] ? 16 : 4;
    float sc = 0.0f;
    if (mx > mn)
      sc = __double2float_rn(__ddiv_rn(__dsub_rn((double)mx, (double)mn), (double)(L - 1)));
    GptqGroup G;
    G.gmin = mn;
    G.sc = sc;
    G.rsc = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    G.zero_f = sc > 0.0f ? __double2float_rn(rint(__ddiv_rn(-(double)mn, (double)sc))) : 0.0f;
    G.lmax = (float)(L - 1);
    G.pad[0] = G.pad[1] = G.pad[2] = 0.0f;
    out[g] = G;
  }
}

constexpr int kGB = 128;  // GPTQ block size (llama.py:238 default, used at :345, :353)

// Column J of a block, then columns J+1 .. kGB-1 (template recursion keeps
// every index compile-time, so the block's weights stay in registers).
//   kRecip: (w - gmin) / sc evaluated as (w - gmin) * fp32(1 / sc), which is
//   how PyTorch divides a CUDA tensor by a Python scalar; otherwise the IEEE
//   quotient (CPU tensors).
template <int J, bool kRecip>
struct GptqColumn {
  static __device__ __forceinline__ void run(float (&w)[kGB], const float* hs,
                                             const GptqGroup* gsh) {
    if constexpr (J < kGB) {
      const GptqGroup& G = gsh[J / kGroup1];
      const float x = w[J];
      float q;
      if (G.sc > 0.0f) {
        // q_int = ((w - gmin) / sc).round().clamp(0, L - 1); q = sc * (q_int - zero)
        const float d = __fsub_rn(x, G.gmin);
        float qi = rintf(kRecip ? __fmul_rn(d, G.rsc) : __fdiv_rn(d, G.sc));
        if (!isnan(qi)) qi = fminf(fmaxf(qi, 0.0f), G.lmax);
        q = __fmul_rn(G.sc, __fsub_rn(qi, G.zero_f));
      } else {
        q = G.gmin;
      }
      // Err = (w - q) / Hinv_cho[col, col]; W_block[:, j+1:] -= Err * Hinv_cho[col, j+1:]
      const float err = __fdiv_rn(__fsub_rn(x, q), hs[J * kGB + J]);
      w[J] = q;
#pragma unroll
      for (int c = J + 1; c < kGB; ++c) w[c] = __fsub_rn(w[c], __fmul_rn(err, hs[J * kGB + c]));
      GptqColumn<J + 1, kRecip>::run(w, hs, gsh);
    }
  }
};

// One thread per (row, block): the block's weights stay in registers; the
// Hinv_cho block sits in shared memory and every read of it is a broadcast.
// Blocks only read the original W (the reference clones Q's block columns
// before any of them is written), so all blocks run in parallel.  A partial
// last block (n < 128 columns) runs padded: the padding never feeds the real
// columns (updates only flow to later columns) and is not stored.
template <bool kRecip>
__global__ void __launch_bounds__(128)
    gptq_block_kernel(const float* __restrict__ W, int64_t M, int64_t K,
                      const float* __restrict__ Hc, const GptqGroup* __restrict__ groups,
                      float* __restrict__ Q, int64_t row0) {
  extern __shared__ float hs[];  // [kGB][kGB]: Hinv_cho[bs + j, bs + c]
  __shared__ GptqGroup gsh[kGB / kGroup1];
  const int64_t bs = (int64_t)blockIdx.x * kGB;
  const int n = (int)min64(kGB, K - bs);
  for (int idx = threadIdx.x; idx < kGB * kGB; idx += blockDim.x) {
    const int j = idx / kGB, c = idx % kGB;
    hs[idx] = (j < n && c < n) ? Hc[(bs + j) * K + bs + c] : (j == c ? 1.0f : 0.0f);
  }
  if (threadIdx.x < kGB / kGroup1) {
    const int64_t g = bs / kGroup1 + threadIdx.x;
    gsh[threadIdx.x] = (threadIdx.x * kGroup1 < n)
                           ? groups[g]
                           : GptqGroup{0.0f, 0.0f, 0.0f, 0.0f, 3.0f, {0.0f, 0.0f, 0.0f}};
  }
  __syncthreads();
  // rows [row0, M) of W; Q holds them from its first row
  const int64_t row = row0 + (int64_t)blockIdx.y * blockDim.x + threadIdx.x;
  if (row >= M) return;
  const float* wr = W + row * K + bs;
  float* qr = Q + (row - row0) * K + bs;
  float w[kGB];
  if (n == kGB) {
#pragma unroll
    for (int c = 0; c < kGB; c += 4) {
      const float4 v = *reinterpret_cast<const float4*>(wr + c);
      w[c] = v.x;
      w[c + 1] = v.y;
      w[c + 2] = v.z;
      w[c + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int c = 0; c < kGB; ++c) w[c] = c < n ? wr[c] : 0.0f;
  }
  GptqColumn<0, kRecip>::run(w, hs, gsh);
  if (n == kGB) {
#pragma unroll
    for (int c = 0; c < kGB; c += 4)
      *reinterpret_cast<float4*>(qr + c) = make_float4(w[c], w[c + 1], w[c + 2], w[c + 3]);
  } else {
#pragma unroll
    for (int c = 0; c < kGB; ++c)
      if (c < n) qr[c] = w[c];
  }
}

template <bool kRecip>
mb_status launch_block(const float* W, int64_t row0, int64_t row1, int64_t K, const float* Hc,
                       const GptqGroup* groups, float* Q, cudaStream_t stream) {
  constexpr size_t smem = sizeof(float) * kGB * kGB;
  static std::atomic<uint64_t> attr_done{0};
  MB_CUDA_TRY(set_smem_limit_once(gptq_block_kernel<kRecip>, (int)smem, attr_done));
  gptq_block_kernel<kRecip><<<dim3((unsigned)ceil_div(K, kGB), (unsigned)ceil_div(row1 - row0, 128)),
                              128, smem, stream>>>(W, row1, K, Hc, groups, Q, row0);
  MB_LAUNCH_CHECK("gptq_block_kernel");
  return MB_OK;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" size_t mb_gptq_workspace_size(int64_t M, int64_t K) {
  (void)M;
  if (K <= 0) return 0;
  return align_up(sizeof(GptqGroup) * (size_t)ceil_div(K, kGroup1), 256);
}

extern "C" mb_status mb_gptq_quantize_rows(const float* W, int64_t M, int64_t K, int64_t row0,
                                           int64_t row1, const float* hinv_cho,
                                           const uint8_t* group_precision, int blocksize,
                                           int scalar_division, float* Q_rows, void* workspace,
                                           size_t workspace_bytes, mb_stream_t stream_);

extern "C" mb_status mb_gptq_quantize(const float* W, int64_t M, int64_t K, const float* hinv_cho,
                                      const uint8_t* group_precision, int blocksize,
                                      int scalar_division, float* Q, void* workspace,
                                      size_t workspace_bytes, mb_stream_t stream_) {
  return mb_gptq_quantize_rows(W, M, K, 0, M, hinv_cho, group_precision, blocksize,
                               scalar_division, Q, workspace, workspace_bytes, stream_);
}

extern "C" mb_status mb_gptq_quantize_rows(const float* W, int64_t M, int64_t K, int64_t row0,
                                           int64_t row1, const float* hinv_cho,
                                           const uint8_t* group_precision, int blocksize,
                                           int scalar_division, float* Q, void* workspace,
                                           size_t workspace_bytes, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(row0 >= 0 && row0 < row1 && row1 <= M, "row range must be inside [0, M)");
  MB_REQUIRE(W && hinv_cho && group_precision && Q, "null pointer");
  MB_REQUIRE(M > 0 && K > 0, "W must be a non-empty [M, K] matrix");
  MB_REQUIRE(K % kGroup1 == 0, "K must be a multiple of 16 (whole column groups)");
  MB_REQUIRE(blocksize == kGB, "blocksize must be 128");
  MB_REQUIRE(scalar_division == MB_GPTQ_DIV_TRUE || scalar_division == MB_GPTQ_DIV_RECIPROCAL,
             "unknown scalar_division mode");
  MB_REQUIRE(row1 - row0 <= 65535LL * 128, "too many rows");
  MB_REQUIRE(((reinterpret_cast<uintptr_t>(W) | reinterpret_cast<uintptr_t>(Q)) & 15u) == 0,
             "W and Q must be 16-byte aligned");
  MB_REQUIRE(W != Q, "Q must not alias W");
  MB_REQUIRE(workspace && workspace_bytes >= mb_gptq_workspace_size(M, K),
             "gptq workspace too small");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  GptqGroup* groups = static_cast<GptqGroup*>(workspace);
  const int64_t ng = K / kGroup1;
  gptq_group_kernel<<<(unsigned)ng, 256, 0, stream>>>(W, M, K, group_precision, groups);
  MB_LAUNCH_CHECK("gptq_group_kernel");
  return scalar_division == MB_GPTQ_DIV_RECIPROCAL
             ? launch_block<true>(W, row0, row1, K, hinv_cho, groups, Q, stream)
             : launch_block<false>(W, row0, row1, K, hinv_cho, groups, Q, stream);
}
