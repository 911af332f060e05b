// memboost quantize on sm_100a.
//
// Replaces the reference's six-kernel pipeline with host round trips
// (core/torch_ops.cu:105-264 driving core/quantize.cu:72-321) by a
// stream-ordered device pipeline with no host synchronisation:
//
//   stats      one CTA per 16-column group streams the group's rows once and
//              produces min/max (quantize.cu:103-128) and, when a hessian is
//              given, the group sensitivity (quantize.cu:72-98) -- the
//              reference's serial fp32 sum reproduced bit for bit by an exact
//              block-parallel scan (see sens_stage below).
//   select     device top-k of the sensitivities (torch_ops.cu:149-179).
//   params     per-group scale / zero / threshold tables
//              (quantize.cu:153-176).
//   second     2nd-order quantisation of the 1st-order scales
//              (quantize.cu:245-281).
//   encode     one pass over W writing both packed arrays, scales, zeros and
//              2nd-order codes, and counting outliers per row
//              (quantize.cu:132-242, 284-299) -- no [M, K] outlier mask.
//   rowscan    exclusive scan of the per-row outlier counts into
//              outlier_row_ptrs and nnz (torch_ops.cu:219-229).
//   extract    (second entry point) CSR values/columns in ascending column
//              order (quantize.cu:301-321).
//
// Arithmetic that decides an output bit is done with the same fp32
// operations as the reference, written with explicit rounding intrinsics so
// the compiler cannot contract or reorder them.
#include <algorithm>
#include <cmath>

#include "mb_common.cuh"

namespace mb {
namespace {

constexpr int kFlagRegular = 1;  // group takes the threshold path; cannot hold outliers

// Per 1st-order group parameters (identical for every row of the group, as in
// the reference where scale/zero depend only on the group's column range).
struct __align__(16) GroupParams {
  float gmin, gmax, scale, thr;
  int zero, levels, flags, scale_h;  // scale_h: fp16 bit pattern of scales_1st
  uint16_t thresh[16];               // fp16 patterns T_1..T_{L-1}; 0x7C00 = never
};
static_assert(sizeof(GroupParams) == 64, "GroupParams must stay 64 bytes");

struct Workspace {
  float* gmin;
  float* gmax;
  float* sens;
  GroupParams* params;
  float2* chunk2;      // per 2nd-order chunk: (min, fp32 scale)
  int32_t* row_counts; // per row outlier counts
  uint32_t* status;    // [0] flags (bit 0: selection tie)
};

size_t workspace_layout(int64_t M, int64_t K, char* base, Workspace* ws) {
  const int64_t ng = ceil_div(K, kGroup1);
  const int64_t ng2 = ceil_div(M * ng, kGroup2);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return base ? base + o : nullptr;
  };
  char* p_gmin = take(sizeof(float) * ng);
  char* p_gmax = take(sizeof(float) * ng);
  char* p_sens = take(sizeof(float) * ng);
  char* p_par = take(sizeof(GroupParams) * ng);
  char* p_ch = take(sizeof(float2) * ng2);
  char* p_rc = take(sizeof(int32_t) * M);
  char* p_st = take(sizeof(uint32_t) * 8);
  if (ws) {
    ws->gmin = reinterpret_cast<float*>(p_gmin);
    ws->gmax = reinterpret_cast<float*>(p_gmax);
    ws->sens = reinterpret_cast<float*>(p_sens);
    ws->params = reinterpret_cast<GroupParams*>(p_par);
    ws->chunk2 = reinterpret_cast<float2*>(p_ch);
    ws->row_counts = reinterpret_cast<int32_t*>(p_rc);
    ws->status = reinterpret_cast<uint32_t*>(p_st);
  }
  return off;
}

// ---------------------------------------------------------------------------
// Row loads.  A group's 16 fp16 values of one row are 32 contiguous bytes;
// when K % 8 == 0 they are two aligned 16-byte vectors.
// ---------------------------------------------------------------------------
struct Row16 {
  uint4 lo, hi;  // 16 fp16 values, element i in half i
};

__device__ __forceinline__ Row16 load_row16(const __half* __restrict__ W, int64_t r, int64_t K,
                                            int64_t c0, int gs, bool vec) {
  Row16 v;
  const __half* p = W + r * K + c0;
  if (vec) {
    v.lo = __ldg(reinterpret_cast<const uint4*>(p));
    v.hi = __ldg(reinterpret_cast<const uint4*>(p) + 1);
  } else {
    uint16_t h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i)
      h[i] = (i < gs) ? __half_as_ushort(__ldg(p + i)) : (uint16_t)0;
    v.lo = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                      h[6] | (h[7] << 16));
    v.hi = make_uint4(h[8] | (h[9] << 16), h[10] | (h[11] << 16), h[12] | (h[13] << 16),
                      h[14] | (h[15] << 16));
  }
  return v;
}

__device__ __forceinline__ float row_elem(const Row16& v, int i) {
  const uint32_t w = (i < 8) ? (&v.lo.x)[(i & 7) >> 1] : (&v.hi.x)[(i & 7) >> 1];
  const uint16_t h = (i & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFF);
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t row_bits(const Row16& v, int i) {
  const uint32_t w = (i < 8) ? (&v.lo.x)[(i & 7) >> 1] : (&v.hi.x)[(i & 7) >> 1];
  return (i & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFF);
}

// ---------------------------------------------------------------------------
// stats: min/max and exact serial-order sensitivity per group.
//
// The reference sums a group's M*16 terms t = (h > 1e-8 ? w*w/h : w*w) one
// after another in fp32 (quantize.cu:87-95).  The sum S is non-decreasing
// (every term is >= 0).  While S stays inside one binade [2^e, 2^(e+1)) every
// fp32 value there is a multiple of q = 2^(e-23), so
//     fl(S + t) = S + rint(t / q) * q
// exactly, unless t / q is a tie (fraction exactly .5, where the result
// depends on the parity of S / q) or the exact S + t leaves the binade.
// The block therefore adds whole runs of terms as integers: each thread
// rounds its 16 terms to multiples of q, a block-wide prefix sum gives every
// thread's running total, and the first thread whose run contains a tie or
// would cross 2^(e+1) adds its terms one by one in fp32 (exactly the
// reference's operations) before the scan restarts after it with the new
// binade.  Threads before it are committed with one exact fp32 add.  Every
// committed value equals the reference's serial sum, so the result is
// bit-identical; only the number of rounds depends on the data.
// ---------------------------------------------------------------------------
template <int NW>
struct ScanSmem {
  float wtot[NW];
  int wfirst[NW];
  float S;
};

template <int NW>
__device__ __forceinline__ void sens_stage(float& S, const float (&t)[16],
                                           ScanSmem<NW>& sm) {
  constexpr int kRows = NW * 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int from = 0;
  while (from < kRows) {
    const bool mine = tid >= from;
    if (isfinite(S) && S >= 0x1p-103f) {
      const uint32_t E = (__float_as_uint(S) >> 23) & 0xFFu;  // >= 24 here
      const float inv_q = __uint_as_float((277u - E) << 23);   // 2^(23-e)
      const float q = __uint_as_float((E - 23u) << 23);        // 2^(e-23)
      const float m = __fmul_rn(S, inv_q);                     // S / q, in [2^23, 2^24)
      const float limit = __fsub_rn(16777216.0f, m);           // room left in the binade
      float loc = 0.0f, dmax = 0.0f;
      if (mine) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = __fmul_rn(t[i], inv_q);
          const float k = rintf(a);
          loc = __fadd_rn(loc, k);
          dmax = fmaxf(dmax, fabsf(__fsub_rn(a, k)));
        }
      }
      // inclusive scan within the warp
      float incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl = __fadd_rn(incl, y);
      }
      // exclusive prefix from the previous lane's inclusive value (never
      // incl - loc: when this thread's own run is huge that difference is
      // inexact, while every value before the first special thread is exact)
      float excl = __shfl_up_sync(0xffffffffu, incl, 1);
      if (lane == 0) excl = 0.0f;
      if (lane == 31) sm.wtot[warp] = incl;
      __syncthreads();
      float off = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w)
        if (w < warp) off = __fadd_rn(off, sm.wtot[w]);
      incl = __fadd_rn(incl, off);
      excl = __fadd_rn(excl, off);
      const bool special = mine && (dmax == 0.5f || !(incl < limit));
      const unsigned bal = __ballot_sync(0xffffffffu, special);
      if (lane == 0) sm.wfirst[warp] = bal ? warp * 32 + __ffs(bal) - 1 : kRows;
      __syncthreads();
      int ls = kRows;
#pragma unroll
      for (int w = 0; w < NW; ++w) ls = min(ls, sm.wfirst[w]);
      if (ls == kRows) {
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) tot = __fadd_rn(tot, sm.wtot[w]);
        S = __fadd_rn(S, __fmul_rn(tot, q));
        from = kRows;
      } else {
        if (tid == ls) {
          float s = __fadd_rn(S, __fmul_rn(excl, q));
#pragma unroll
          for (int i = 0; i < 16; ++i) s = __fadd_rn(s, t[i]);
          sm.S = s;
        }
        __syncthreads();
        S = sm.S;
        from = ls + 1;
      }
      __syncthreads();  // smem reuse by the next round
    } else if (S == 0.0f) {
      // fl(0 + t) = t: runs of zero terms commit nothing; the first thread
      // holding a non-zero (or NaN) term goes serial.
      bool nz = false;
      if (mine) {
#pragma unroll
        for (int i = 0; i < 16; ++i) nz |= (t[i] != 0.0f);
      }
      const unsigned bal = __ballot_sync(0xffffffffu, nz);
      if (lane == 0) sm.wfirst[warp] = bal ? warp * 32 + __ffs(bal) - 1 : kRows;
      __syncthreads();
      int ls = kRows;
#pragma unroll
      for (int w = 0; w < NW; ++w) ls = min(ls, sm.wfirst[w]);
      if (ls == kRows) {
        from = kRows;
      } else {
        if (tid == ls) {
          float s = S;
#pragma unroll
          for (int i = 0; i < 16; ++i) s = __fadd_rn(s, t[i]);
          sm.S = s;
        }
        __syncthreads();
        S = sm.S;
        from = ls + 1;
      }
      __syncthreads();
    } else if (!isfinite(S)) {
      // inf or NaN absorbs every later term the same way in any order.
      float loc = 0.0f;
      if (mine) {
#pragma unroll
        for (int i = 0; i < 16; ++i) loc = __fadd_rn(loc, t[i]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) loc = __fadd_rn(loc, __shfl_xor_sync(0xffffffffu, loc, o));
      if (lane == 0) sm.wtot[warp] = loc;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w) tot = __fadd_rn(tot, sm.wtot[w]);
      S = __fadd_rn(S, tot);
      from = kRows;
      __syncthreads();
    } else {
      // 0 < S < 2^-103: too small for the integer grid; one thread at a time.
      const int ls = from;
      if (tid == ls) {
        float s = S;
#pragma unroll
        for (int i = 0; i < 16; ++i) s = __fadd_rn(s, t[i]);
        sm.S = s;
      }
      __syncthreads();
      S = sm.S;
      from = ls + 1;
      __syncthreads();
    }
  }
}

template <int NW, bool kSens>
__global__ void __launch_bounds__(NW * 32)
    stats_kernel(const __half* __restrict__ W, int64_t M, int64_t K, bool w_aligned,
                 const float* __restrict__ hess, float* __restrict__ gmin_out,
                 float* __restrict__ gmax_out, float* __restrict__ sens_out) {
  constexpr int kRows = NW * 32;
  __shared__ ScanSmem<NW> sm;
  __shared__ float red[2][NW];
  const int g = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, K - c0);
  const bool vec = w_aligned && (gs == kGroup1) && ((K & 7) == 0);

  float hv[16];
  bool divide = false;
  if (kSens) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      hv[i] = (i < gs) ? __ldg(hess + c0 + i) : 1.0f;
      divide |= (hv[i] > 1e-8f) && (hv[i] != 1.0f);
    }
  }

  float mn = 1e10f, mx = -1e10f, S = 0.0f;
  Row16 nxt;
  if (tid < M) nxt = load_row16(W, tid, K, c0, gs, vec);
  for (int64_t base = 0; base < M; base += kRows) {
    const int64_t r = base + tid;
    const bool valid = r < M;
    const Row16 cur = nxt;
    if (r + kRows < M) nxt = load_row16(W, r + kRows, K, c0, gs, vec);
    float t[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float v = row_elem(cur, i);
      const bool ok = valid && (i < gs);
      if (ok) {
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
      if (kSens) {
        const float x = __fmul_rn(v, v);  // exact for fp16 inputs
        float s = x;
        if (divide && hv[i] > 1e-8f) s = __fdiv_rn(x, hv[i]);
        t[i] = ok ? s : 0.0f;
      }
    }
    if (kSens) sens_stage<NW>(S, t, sm);
  }

  mn = warp_min(mn);
  mx = warp_max(mx);
  const int lane = tid & 31, warp = tid >> 5;
  if (lane == 0) {
    red[0][warp] = mn;
    red[1][warp] = mx;
  }
  __syncthreads();
  if (tid == 0) {
    float a = red[0][0], b = red[1][0];
#pragma unroll
    for (int w = 1; w < NW; ++w) {
      a = fminf(a, red[0][w]);
      b = fmaxf(b, red[1][w]);
    }
    gmin_out[g] = a;
    gmax_out[g] = b;
    if (kSens) sens_out[g] = S;
  }
}

// ---------------------------------------------------------------------------
// select: the n4 largest sensitivities become 4-bit (torch_ops.cu:163-178).
// Rank of group i = #{j : s_j > s_i} + #{j < i : s_j == s_i}; group i is
// selected iff rank < n4.  Sensitivities are >= 0, so comparing their bit
// patterns as unsigned integers orders them like the reference's float
// comparison.  Equal keys straddling the boundary are flagged in status[0].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
    select_kernel(const float* __restrict__ sens, int ng, int n4, uint8_t* __restrict__ gp,
                  uint32_t* __restrict__ status) {
  extern __shared__ uint32_t keys[];
  for (int i = threadIdx.x; i < ng; i += blockDim.x) keys[i] = __float_as_uint(sens[i]);
  __syncthreads();
  __shared__ uint32_t boundary_key;
  __shared__ int have_boundary;
  if (threadIdx.x == 0) have_boundary = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < ng; i += blockDim.x) {
    const uint32_t ki = keys[i];
    int rank = 0;
    for (int j = 0; j < ng; ++j) {
      const uint32_t kj = keys[j];
      rank += (kj > ki) || (kj == ki && j < i);
    }
    gp[i] = rank < n4 ? 1 : 0;
    if (rank == n4 - 1) {
      boundary_key = ki;
      have_boundary = 1;
    }
  }
  __syncthreads();
  if (have_boundary && n4 < ng) {
    // tie across the boundary: some unselected group has the boundary key
    const uint32_t bk = boundary_key;
    for (int i = threadIdx.x; i < ng; i += blockDim.x)
      if (keys[i] == bk && gp[i] == 0) atomicOr(status, 1u);
  }
}

// ---------------------------------------------------------------------------
// params: scale / zero / threshold per group (quantize.cu:153-176).
//
// The reference's code of a value w is
//   q(w) = clamp((int)roundf((w - gmin) / scale), 0, L-1)
// which is non-decreasing in w.  For a group whose zero point is not clamped
// and whose scale is not clamped ("regular"), |w - scale*(q-zero)| is at most
// about one scale for every w in [gmin, gmax], below the outlier threshold
// (0.4*range = 1.2 scale for 2-bit, 0.15*range = 2.25 scale for 4-bit), so
// no outliers exist and q(w) is fully described by the L-1 smallest fp16
// values reaching each code.  Those thresholds are found here by binary
// search over the ordered fp16 values, evaluating the reference formula.
// Other groups use the formula per element in `encode`.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int code_of(float x, float gmin, float scale, int L) {
  const float a = __fdiv_rn(__fsub_rn(x, gmin), scale);
  const int q = f2i_rz(roundf(a));
  return max(0, min(L - 1, q));
}

__device__ __forceinline__ uint16_t ord_to_half_bits(int ord) {
  return ord >= 0 ? (uint16_t)ord : (uint16_t)(0x8000 | (-ord - 1));
}

__global__ void __launch_bounds__(256)
    params_kernel(const float* __restrict__ gmin_in, const float* __restrict__ gmax_in, int ng,
                  bool selected, uint8_t* __restrict__ gp, GroupParams* __restrict__ params) {
  const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (g >= ng) return;
  const float gmin = gmin_in[g], gmax = gmax_in[g];
  int prec = 0;
  if (selected) prec = gp[g];
  __syncwarp();
  if (!selected && lane == 0) gp[g] = 0;
  const int L = prec ? 16 : 4;
  const float range = __fsub_rn(gmax, gmin);
  const float scale_raw = __fdiv_rn(range, (float)(L - 1));
  float scale = scale_raw;
  if (scale < 1e-8f) scale = 1e-8f;
  const int zr = f2i_rz(roundf(__fdiv_rn(-gmin, scale)));
  const int zero = max(0, min(L - 1, zr));
  const float thr = prec == 0 ? __fmul_rn(0.4f, range) : __fmul_rn(0.15f, range);
  const bool regular = isfinite(gmin) && isfinite(gmax) && (scale_raw >= 1e-8f) && zr >= 0 &&
                       zr <= L - 1 && isfinite(thr);
  uint16_t T = 0x7C00;
  if (regular && lane < L - 1) {
    const int level = lane + 1;
    int lo = -31744, hi = 31744;  // finite fp16 values in order; hi = "none"
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;  // floor for negatives too (arithmetic shift)
      const float x = __half2float(__ushort_as_half(ord_to_half_bits(mid)));
      if (code_of(x, gmin, scale, L) >= level)
        hi = mid;
      else
        lo = mid + 1;
    }
    if (lo < 31744) T = ord_to_half_bits(lo);
  }
  GroupParams* p = params + g;
  if (lane < 16) p->thresh[lane] = T;
  if (lane == 0) {
    p->gmin = gmin;
    p->gmax = gmax;
    p->scale = scale;
    p->thr = thr;
    p->zero = zero;
    p->levels = L;
    p->flags = regular ? kFlagRegular : 0;
    p->scale_h = __half_as_ushort(__float2half_rn(scale));
  }
}

// 2nd-order: one warp per 256-long chunk of the flattened [M, ng] scales
// (quantize.cu:245-272).  scales_1st[r, g] depends only on g.
__global__ void __launch_bounds__(256)
    second_order_kernel(const GroupParams* __restrict__ params, int64_t M, int ng, int64_t ng2,
                        __half* __restrict__ scales2, int8_t* __restrict__ zeros2,
                        float2* __restrict__ chunk2) {
  const int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (c >= ng2) return;
  const int64_t total = M * (int64_t)ng;
  const int64_t s0 = c * kGroup2;
  const int64_t s1 = min64(s0 + kGroup2, total);
  float mn = 1e10f, mx = -1e10f;
  for (int64_t i = s0 + lane; i < s1; i += 32) {
    const int g = (int)(i % ng);
    const float s = __half2float(__ushort_as_half((uint16_t)params[g].scale_h));
    mn = fminf(mn, s);
    mx = fmaxf(mx, s);
  }
  mn = warp_min(mn);
  mx = warp_max(mx);
  if (lane == 0) {
    float sc2 = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    if (sc2 < 1e-10f) sc2 = 1e-10f;
    const int z2 = f2i_rz(roundf(__fdiv_rn(-mn, sc2)));
    scales2[c] = __float2half_rn(sc2);
    zeros2[c] = (int8_t)z2;  // low byte, as the reference's (int8_t) cast
    chunk2[c] = make_float2(mn, sc2);
  }
}

// ---------------------------------------------------------------------------
// encode: one thread per (row, group).  Writes every per-(row, group) output
// and counts outliers per row.  Both packed arrays are written in full
// (zeros where the group has the other precision), so no memset is needed.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

__global__ void __launch_bounds__(128)
    encode_kernel(const __half* __restrict__ W, int64_t M, int64_t K, bool w_aligned, int ng,
                  const GroupParams* __restrict__ params, const float2* __restrict__ chunk2,
                  int32_t* __restrict__ packed2, int32_t* __restrict__ packed4,
                  __half* __restrict__ scales1, int8_t* __restrict__ zeros1,
                  uint8_t* __restrict__ sq, int32_t* __restrict__ row_counts, int fma_mode) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= ng) return;
  const GroupParams p = params[g];
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, K - c0);
  const bool vec = w_aligned && (gs == kGroup1) && ((K & 7) == 0);
  const bool four = p.levels == 16;
  const __half sh = __ushort_as_half((uint16_t)p.scale_h);
  const float s1f = __half2float(sh);
  __half2 T2[15];
#pragma unroll
  for (int j = 0; j < 15; ++j) T2[j] = __half2half2(__ushort_as_half(p.thresh[j]));

  for (int64_t r = blockIdx.y; r < M; r += gridDim.y) {
    const Row16 v = load_row16(W, r, K, c0, gs, vec);
    uint32_t wa = 0, wb = 0;  // 2-bit word, or the two 4-bit words
    int cnt = 0;
    if (p.flags & kFlagRegular) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t pair = k < 4 ? (&v.lo.x)[k] : (&v.hi.x)[k - 4];
        const __half2 w2 = *reinterpret_cast<const __half2*>(&pair);
        __half2 acc = __float2half2_rn(1024.0f);
        if (!four) {
#pragma unroll
          for (int j = 0; j < 3; ++j) acc = __hadd2(acc, __hge2(w2, T2[j]));
        } else {
#pragma unroll
          for (int j = 0; j < 15; ++j) acc = __hadd2(acc, __hge2(w2, T2[j]));
        }
        // acc = 1024 + code in each half: 1024 has an ulp of 1, so the code
        // sits in the low mantissa bits.
        const uint32_t b = h2_bits(acc);
        const uint32_t qa = b & 0xFu, qb = (b >> 16) & 0xFu;
        const int i0 = 2 * k;  // element index of qa; qb is i0 + 1
        if (!four) {
          wa |= (qa << (2 * i0)) | (qb << (2 * i0 + 2));
        } else if (i0 < 8) {
          wa |= (qa << (4 * i0)) | (qb << (4 * i0 + 4));
        } else {
          wb |= (qa << (4 * (i0 - 8))) | (qb << (4 * (i0 - 8) + 4));
        }
      }
      // columns past K in a partial group hold code 0 in the reference
      if (gs < kGroup1) {
        if (!four) {
          wa &= (gs >= 16) ? 0xFFFFFFFFu : ((1u << (2 * gs)) - 1u);
        } else {
          const int ga = min(gs, 8), gb = max(gs - 8, 0);
          wa &= (ga >= 8) ? 0xFFFFFFFFu : ((1u << (4 * ga)) - 1u);
          wb &= (gb >= 8) ? 0xFFFFFFFFu : ((1u << (4 * gb)) - 1u);
        }
      }
    } else {
      const int L = p.levels;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i < gs) {
          const float x = row_elem(v, i);
          const int q = code_of(x, p.gmin, p.scale, L);
          const float qz = (float)(q - p.zero);
          float err;
          if (fma_mode)
            err = fabsf(__fmaf_rn(-p.scale, qz, x));
          else
            err = fabsf(__fsub_rn(x, __fmul_rn(p.scale, qz)));
          cnt += (err > p.thr);
          if (!four)
            wa |= (uint32_t)(q & 0x3) << (2 * i);
          else if (i < 8)
            wa |= (uint32_t)(q & 0xF) << (4 * i);
          else
            wb |= (uint32_t)(q & 0xF) << (4 * (i - 8));
        }
      }
    }
    const int64_t si = r * ng + g;
    packed2[si] = four ? 0 : (int32_t)wa;
    reinterpret_cast<int2*>(packed4)[si] = four ? make_int2((int)wa, (int)wb) : make_int2(0, 0);
    scales1[si] = sh;
    zeros1[si] = (int8_t)p.zero;
    const float2 ch = chunk2[si / kGroup2];
    const int q2 = f2i_rz(roundf(__fdiv_rn(__fsub_rn(s1f, ch.x), ch.y)));
    sq[si] = (uint8_t)max(0, min(15, q2));
    if (cnt) atomicAdd(row_counts + r, cnt);
  }
}

// Exclusive scan of row counts -> outlier_row_ptrs [M+1], nnz.
__global__ void __launch_bounds__(1024)
    rowscan_kernel(const int32_t* __restrict__ counts, int64_t M, int32_t* __restrict__ row_ptrs,
                   int32_t* __restrict__ nnz) {
  __shared__ long long part[1024];
  const int t = threadIdx.x;
  const int64_t per = ceil_div(M, (int64_t)blockDim.x);
  const int64_t r0 = min64(M, t * per), r1 = min64(M, r0 + per);
  long long s = 0;
  for (int64_t r = r0; r < r1; ++r) s += counts[r];
  part[t] = s;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const long long y = t >= o ? part[t - o] : 0;
    __syncthreads();
    part[t] += y;
    __syncthreads();
  }
  long long run = part[t] - s;  // exclusive
  if (t == 0) row_ptrs[0] = 0;
  for (int64_t r = r0; r < r1; ++r) {
    run += counts[r];
    row_ptrs[r + 1] = (int32_t)run;
  }
  if (t == blockDim.x - 1) *nnz = (int32_t)part[t];
}

// extract: one warp per row with outliers; only non-regular groups can hold
// them.  Lanes 0-15 take the group's 16 columns; the ballot order is the
// column order.
__global__ void __launch_bounds__(256)
    extract_kernel(const __half* __restrict__ W, int64_t M, int64_t K, int ng,
                   const GroupParams* __restrict__ params, const int32_t* __restrict__ row_ptrs,
                   __half* __restrict__ vals, int32_t* __restrict__ cols, int fma_mode) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= M) return;
  int32_t o = row_ptrs[r];
  const int32_t end = row_ptrs[r + 1];
  if (o == end) return;
  for (int g = 0; g < ng && o < end; ++g) {
    const GroupParams& p = params[g];
    if (p.flags & kFlagRegular) continue;
    const int64_t c = (int64_t)g * kGroup1 + lane;
    bool out = false;
    __half wv = __ushort_as_half(0);
    if (lane < kGroup1 && c < K) {
      wv = W[r * K + c];
      const float x = __half2float(wv);
      const int q = code_of(x, p.gmin, p.scale, p.levels);
      const float qz = (float)(q - p.zero);
      float err;
      if (fma_mode)
        err = fabsf(__fmaf_rn(-p.scale, qz, x));
      else
        err = fabsf(__fsub_rn(x, __fmul_rn(p.scale, qz)));
      out = err > p.thr;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, out);
    const int pos = o + __popc(bal & ((1u << lane) - 1u));
    if (out && pos < end) {
      vals[pos] = wv;
      cols[pos] = (int32_t)c;
    }
    o += __popc(bal);
  }
}

// Outlier test arithmetic of the reference kernel: 1 = the product
// scale*(q-zero) fused into the subtraction (one rounding), 0 = rounded
// product.  Fixed by the parity tests against the compiled reference.
constexpr int kOutlierFma = 1;

mb_status check_common(const void* weights, int64_t M, int64_t K) {
  MB_REQUIRE(weights != nullptr, "weights must not be null");
  MB_REQUIRE(M > 0 && K > 0, "weights must be a non-empty 2D [M, K] matrix");
  MB_REQUIRE(M * ceil_div(K, kGroup1) < (int64_t)INT32_MAX && M * K < (int64_t)INT32_MAX,
             "weights too large: M*K must be below 2^31 (int32 outlier indexing)");
  return MB_OK;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" size_t mb_quantize_workspace_size(int64_t M, int64_t K) {
  if (M <= 0 || K <= 0) return 0;
  return workspace_layout(M, K, nullptr, nullptr);
}

extern "C" mb_status mb_quantize(const void* weights_fp16, int64_t M, int64_t K,
                                 double ratio_4bit, const float* hessian_diag,
                                 int64_t hessian_numel, int32_t* packed_2bit,
                                 int32_t* packed_4bit, void* scales_1st_fp16, int8_t* zeros_1st,
                                 void* scales_2nd_fp16, int8_t* zeros_2nd,
                                 uint8_t* scales_1st_quant, uint8_t* group_precision,
                                 int32_t* outlier_row_ptrs, int32_t* nnz_device, void* workspace,
                                 size_t workspace_bytes, mb_stream_t stream_) {
  clear_error();
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (mb_status st = check_common(weights_fp16, M, K)) return st;
  MB_REQUIRE(packed_2bit && packed_4bit && scales_1st_fp16 && zeros_1st && scales_2nd_fp16 &&
                 zeros_2nd && scales_1st_quant && group_precision && outlier_row_ptrs &&
                 nnz_device,
             "output pointers must not be null");
  const int64_t ng = ceil_div(K, kGroup1);
  const int64_t ng2 = ceil_div(M * ng, kGroup2);
  const size_t need = workspace_layout(M, K, nullptr, nullptr);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(MB_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) +
                                           " bytes, got " + std::to_string(workspace_bytes));
  Workspace ws;
  workspace_layout(M, K, static_cast<char*>(workspace), &ws);
  const bool selecting = hessian_diag != nullptr && hessian_numel > 0 && ratio_4bit > 0.0;
  if (selecting)
    MB_REQUIRE(hessian_numel >= K, "hessian_diag must hold at least K values");
  int64_t n4 = 0;
  if (selecting) {
    n4 = (int64_t)(int)(ratio_4bit * (double)(int)ng);  // torch_ops.cu:172
    n4 = std::max<int64_t>(0, std::min<int64_t>(n4, ng));
  }
  const __half* W = static_cast<const __half*>(weights_fp16);
  const bool w_aligned = (reinterpret_cast<uintptr_t>(weights_fp16) & 15u) == 0;
  MB_REQUIRE((reinterpret_cast<uintptr_t>(packed_2bit) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(packed_4bit) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_1st_fp16) & 1u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_2nd_fp16) & 1u) == 0 &&
                 (reinterpret_cast<uintptr_t>(outlier_row_ptrs) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(nnz_device) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
             "misaligned output or workspace pointer (packed_4bit needs 8 bytes, "
             "int32/fp16 outputs natural alignment, workspace 256 bytes)");

  MB_CUDA_TRY(cudaMemsetAsync(ws.row_counts, 0, sizeof(int32_t) * M, stream));
  MB_CUDA_TRY(cudaMemsetAsync(ws.status, 0, sizeof(uint32_t) * 8, stream));

  // stats (+ sensitivity)
  const bool small_ng = ng < 2 * 148;
  if (selecting) {
    if (small_ng)
      stats_kernel<8, true><<<(unsigned)ng, 256, 0, stream>>>(W, M, K, w_aligned, hessian_diag, ws.gmin,
                                                               ws.gmax, ws.sens);
    else
      stats_kernel<4, true><<<(unsigned)ng, 128, 0, stream>>>(W, M, K, w_aligned, hessian_diag, ws.gmin,
                                                               ws.gmax, ws.sens);
  } else {
    if (small_ng)
      stats_kernel<8, false><<<(unsigned)ng, 256, 0, stream>>>(W, M, K, w_aligned, nullptr, ws.gmin,
                                                                ws.gmax, ws.sens);
    else
      stats_kernel<4, false><<<(unsigned)ng, 128, 0, stream>>>(W, M, K, w_aligned, nullptr, ws.gmin,
                                                                ws.gmax, ws.sens);
  }
  MB_LAUNCH_CHECK("stats_kernel");

  const bool use_sel = selecting && n4 > 0;
  if (use_sel) {
    const size_t smem = sizeof(uint32_t) * ng;
    MB_REQUIRE(smem <= 200 * 1024, "too many column groups for the device selection");
    if (smem > 48 * 1024)
      MB_CUDA_TRY(cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
    select_kernel<<<1, 1024, smem, stream>>>(ws.sens, (int)ng, (int)n4, group_precision,
                                             ws.status);
    MB_LAUNCH_CHECK("select_kernel");
  }
  params_kernel<<<(unsigned)ceil_div(ng * 32, 256), 256, 0, stream>>>(
      ws.gmin, ws.gmax, (int)ng, use_sel, group_precision, ws.params);
  MB_LAUNCH_CHECK("params_kernel");
  second_order_kernel<<<(unsigned)ceil_div(ng2 * 32, 256), 256, 0, stream>>>(
      ws.params, M, (int)ng, ng2, static_cast<__half*>(scales_2nd_fp16), zeros_2nd, ws.chunk2);
  MB_LAUNCH_CHECK("second_order_kernel");
  {
    dim3 grid((unsigned)ceil_div(ng, 128), (unsigned)std::min<int64_t>(M, 65535));
    encode_kernel<<<grid, 128, 0, stream>>>(W, M, K, w_aligned, (int)ng, ws.params, ws.chunk2, packed_2bit,
                                            packed_4bit, static_cast<__half*>(scales_1st_fp16),
                                            zeros_1st, scales_1st_quant, ws.row_counts,
                                            kOutlierFma);
    MB_LAUNCH_CHECK("encode_kernel");
  }
  rowscan_kernel<<<1, 1024, 0, stream>>>(ws.row_counts, M, outlier_row_ptrs, nnz_device);
  MB_LAUNCH_CHECK("rowscan_kernel");
  return MB_OK;
}

extern "C" mb_status mb_quantize_extract_outliers(const void* weights_fp16, int64_t M, int64_t K,
                                                  const int32_t* outlier_row_ptrs,
                                                  void* outlier_values_fp16,
                                                  int32_t* outlier_col_indices,
                                                  const void* workspace, size_t workspace_bytes,
                                                  mb_stream_t stream_) {
  clear_error();
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (mb_status st = check_common(weights_fp16, M, K)) return st;
  MB_REQUIRE(outlier_row_ptrs && outlier_values_fp16 && outlier_col_indices,
             "CSR pointers must not be null");
  const size_t need = workspace_layout(M, K, nullptr, nullptr);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(MB_ERR_WORKSPACE, "workspace too small");
  Workspace ws;
  workspace_layout(M, K, static_cast<char*>(const_cast<void*>(workspace)), &ws);
  const int64_t ng = ceil_div(K, kGroup1);
  extract_kernel<<<(unsigned)ceil_div(M * 32, 256), 256, 0, stream>>>(
      static_cast<const __half*>(weights_fp16), M, K, (int)ng, ws.params, outlier_row_ptrs,
      static_cast<__half*>(outlier_values_fp16), outlier_col_indices, kOutlierFma);
  MB_LAUNCH_CHECK("extract_kernel");
  return MB_OK;
}

extern "C" mb_status mb_quantize_flags(const void* workspace, size_t workspace_bytes,
                                       int64_t M, int64_t K, uint32_t* flags,
                                       mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(workspace && flags, "null argument");
  MB_REQUIRE(M > 0 && K > 0, "M and K must be positive");
  const size_t need = workspace_layout(M, K, nullptr, nullptr);
  if (workspace_bytes < need) return set_error(MB_ERR_WORKSPACE, "workspace too small");
  Workspace ws;
  workspace_layout(M, K, static_cast<char*>(const_cast<void*>(workspace)), &ws);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  MB_CUDA_TRY(cudaMemcpyAsync(flags, ws.status, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream));
  MB_CUDA_TRY(cudaStreamSynchronize(stream));
  return MB_OK;
}
