// memboost quantize on sm_100a.
//
// Replaces the reference's six-kernel pipeline with host round trips
// (core/torch_ops.cu:105-264 driving core/quantize.cu:72-321) by two
// stream-ordered kernels and no host synchronisation:
//
//   stats   one CTA per 16-column group streams the group's rows once from
//           HBM through a TMA ring buffer (quantize.cu:72-128):
//             * min / max of the group,
//             * the hessian-weighted sensitivity -- the reference's serial
//               fp32 sum reproduced bit for bit by an exact block scan
//               (sens_stage),
//             * scale / zero / code thresholds of the group for both 2-bit
//               and 4-bit precision (quantize.cu:153-176).
//           The last CTA to finish runs `finalize`: the top-k 4-bit
//           selection (torch_ops.cu:149-179) as a radix select, and the
//           2nd-order tables of the flattened scales (quantize.cu:245-281).
//   encode  reads W again (mostly from L2) and writes both packed arrays,
//           scales, zeros, 2nd-order codes, 2nd-order scales/zeros and
//           outlier row pointers (quantize.cu:132-242, 284-299; torch_ops.cu
//           :219-229).  No [M, K] outlier mask exists: only groups whose
//           parameters allow outliers are evaluated per element, and the
//           last CTA scans their per-row counts.
//   extract (second entry point) CSR values/columns in ascending column
//           order (quantize.cu:301-321).
//
// Arithmetic that decides an output bit uses the reference's fp32 operations,
// written with explicit rounding intrinsics so the compiler cannot contract
// or reorder them.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "mb_common.cuh"
#include "mb_tma.cuh"

namespace mb {
namespace {

constexpr int kFlagRegular = 1;  // threshold path valid; group cannot hold outliers
constexpr uint32_t kStatusTie = 1u;
constexpr uint32_t kStatusTimeout = 2u;
constexpr int kMaxStages = 8;

// Per-group parameters of one precision.  Every row of a group shares them
// (in the reference scale and zero depend only on the group's min/max).
struct __align__(16) GroupParams {
  float gmin, gmax, scale, thr;
  int zero, levels, flags, scale_h;  // scale_h: fp16 bit pattern of scales_1st
  uint16_t thresh[16];               // fp16 patterns T_1..T_{L-1}; 0x7C00 = never
};
static_assert(sizeof(GroupParams) == 64, "GroupParams must stay 64 bytes");

struct __align__(16) Header {
  uint32_t ticket_stats;   // stats CTAs finished
  uint32_t ticket_encode;  // encode CTAs finished
  uint32_t status;         // kStatus* bits
  uint32_t any_irregular;  // a group of its selected precision may hold outliers
  uint32_t n2;             // number of 2-bit groups (first entries of `order`)
  uint32_t pad[11];
};
static_assert(sizeof(Header) == 64, "Header must stay 64 bytes");

struct ChunkLayout {
  int64_t total;   // M * ng flattened scales
  int64_t nfull;   // full 256-long 2nd-order chunks
  int64_t ng2;     // all chunks (the last may be partial)
  int period;      // full chunks repeat with this period: ng / gcd(ng, 256)
  int ntab_full;   // distinct full chunks stored = min(nfull, period)
  int has_partial;
};

ChunkLayout chunk_layout(int64_t M, int64_t ng) {
  ChunkLayout c;
  c.total = M * ng;
  c.nfull = c.total / kGroup2;
  c.ng2 = ceil_div(c.total, kGroup2);
  int64_t a = ng, b = kGroup2;
  while (b) {
    const int64_t t = a % b;
    a = b;
    b = t;
  }
  c.period = (int)(ng / a);
  c.ntab_full = (int)std::min<int64_t>(c.nfull, c.period);
  c.has_partial = (c.total % kGroup2) != 0;
  return c;
}

struct Workspace {
  Header* hdr;
  float* gmin;
  float* gmax;
  float* sens;
  GroupParams* params;  // [2 * ng]: 2g = 2-bit, 2g + 1 = 4-bit
  float4* chunk_tab;    // [ntab_full + 1]: (min, fp32 scale2, fp16 bits of scale2, zero2)
  int32_t* row_counts;  // [M]
  uint8_t* prec;        // [ng] selected precision (copy of group_precision)
  int32_t* order;       // [ng] group indices, 2-bit groups first (ascending), then 4-bit
};

size_t workspace_layout(int64_t M, int64_t K, char* base, Workspace* ws) {
  const int64_t ng = ceil_div(K, kGroup1);
  const ChunkLayout cl = chunk_layout(M, ng);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off = align_up(off + bytes, 256);
    return base ? base + o : nullptr;
  };
  char* p_hdr = take(sizeof(Header));
  char* p_gmin = take(sizeof(float) * ng);
  char* p_gmax = take(sizeof(float) * ng);
  char* p_sens = take(sizeof(float) * ng);
  char* p_par = take(sizeof(GroupParams) * 2 * ng);
  char* p_ch = take(sizeof(float4) * (cl.ntab_full + 1));
  char* p_rc = take(sizeof(int32_t) * M);
  char* p_pr = take(ng);
  char* p_or = take(sizeof(int32_t) * ng);
  if (ws) {
    ws->hdr = reinterpret_cast<Header*>(p_hdr);
    ws->gmin = reinterpret_cast<float*>(p_gmin);
    ws->gmax = reinterpret_cast<float*>(p_gmax);
    ws->sens = reinterpret_cast<float*>(p_sens);
    ws->params = reinterpret_cast<GroupParams*>(p_par);
    ws->chunk_tab = reinterpret_cast<float4*>(p_ch);
    ws->row_counts = reinterpret_cast<int32_t*>(p_rc);
    ws->prec = reinterpret_cast<uint8_t*>(p_pr);
    ws->order = reinterpret_cast<int32_t*>(p_or);
  }
  return off;
}

// ---------------------------------------------------------------------------
// Row data.  A group's 16 fp16 values of one row are 32 contiguous bytes.
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
    uint32_t h[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = (i < gs) ? (uint32_t)__half_as_ushort(__ldg(p + i)) : 0u;
    v.lo = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                      h[6] | (h[7] << 16));
    v.hi = make_uint4(h[8] | (h[9] << 16), h[10] | (h[11] << 16), h[12] | (h[13] << 16),
                      h[14] | (h[15] << 16));
  }
  return v;
}

__device__ __forceinline__ uint32_t row_word(const Row16& v, int k) {
  return k < 4 ? (&v.lo.x)[k] : (&v.hi.x)[k - 4];
}

__device__ __forceinline__ float row_elem(const Row16& v, int i) {
  const uint32_t w = row_word(v, i >> 1);
  return __half2float(__ushort_as_half((uint16_t)((i & 1) ? (w >> 16) : (w & 0xFFFFu))));
}

__device__ __forceinline__ __half2 as_h2(uint32_t w) { return *reinterpret_cast<__half2*>(&w); }
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// ---------------------------------------------------------------------------
// Exact serial-order sensitivity.
//
// The reference sums a group's M*16 terms t = (h > 1e-8 ? w*w/h : w*w) one
// after another in fp32 (quantize.cu:87-95).  The sum S is non-decreasing
// (every term is >= 0).  While S stays inside one binade [2^e, 2^(e+1)) every
// fp32 value there is a multiple of q = 2^(e-23), so
//     fl(S + t) = S + rint(t / q) * q
// exactly, unless t / q is a tie (fraction exactly .5, where the result
// depends on the parity of S / q) or the exact S + t leaves the binade.
// The block adds whole runs of terms as integers: each thread rounds its 16
// terms to multiples of q, and if the block's total stays inside the binade
// and no run holds a tie, the stage commits at once.  Otherwise a prefix sum
// locates the first thread whose run holds a tie or would cross 2^(e+1);
// the threads before it are committed with one exact fp32 add, it adds its
// terms one by one in fp32 (exactly the reference's operations), and the
// scan restarts after it with the new binade.  Every committed value equals
// the reference's serial sum, so the result is bit-identical; only the
// number of rounds depends on the data.
// ---------------------------------------------------------------------------
template <int NW>
struct ScanSmem {
  float wtot[NW];
  float wsum[NW];
  int wfirst[NW];
  float S;
};

__device__ __forceinline__ float serial_add(float s, const uint64_t (&T2)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float t0, t1;
    f2_unpack(T2[k], t0, t1);
    s = __fadd_rn(__fadd_rn(s, t0), t1);
  }
  return s;
}

// One stage: the block's kRows threads each hold 16 consecutive terms of the
// serial order (thread order = serial order) as 8 packed pairs.
//
// Rounding a term to the grid uses the FMA pipe: for 0 <= a < 2^23,
// fl(a + 2^23) - 2^23 is a rounded to the nearest integer, ties to even (a
// >= 2^23 means t >= S / 2, a crossing, and the run is special anyway).  A
// tie (|a - k| = 0.5) is detected as fma(d, d, -0.25) >= 0; such a run
// reports an infinite length so it becomes the special thread.
template <int NW>
__device__ __forceinline__ void sens_stage(float& S, const uint64_t (&T2)[8], ScanSmem<NW>& sm) {
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
      float loc = 0.0f;
      if (mine) {
        const uint64_t iq2 = f2_pack(inv_q, inv_q);
        const uint64_t magic2 = f2_pack(8388608.0f, 8388608.0f);
        const uint64_t nq2 = f2_pack(-0.25f, -0.25f);
        uint64_t acc = f2_pack(0.0f, 0.0f);
        uint32_t sgn = 0xFFFFFFFFu;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint64_t a2 = f2_mul(T2[k], iq2);
          const uint64_t k2 = f2_sub(f2_add(a2, magic2), magic2);
          acc = f2_add(acc, k2);
          const uint64_t d2 = f2_sub(a2, k2);
          const uint64_t p2 = f2_fma(d2, d2, nq2);
          sgn &= (uint32_t)p2 & (uint32_t)(p2 >> 32);
        }
        float l0, l1;
        f2_unpack(acc, l0, l1);
        loc = __fadd_rn(l0, l1);
        if (!(sgn >> 31)) loc = INFINITY;  // a tie: this run goes serial
      }
      // fast path: the block's total
      float v = loc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) sm.wsum[warp] = v;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < NW; ++w) tot = __fadd_rn(tot, sm.wsum[w]);
      if (tot < limit) {
        S = __fadd_rn(S, __fmul_rn(tot, q));
        __syncthreads();  // wsum and the stage's shared data are free again
        break;
      }
      // a special thread exists: locate the first one
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
      const bool special = mine && !(incl < limit);
      const unsigned bal = __ballot_sync(0xffffffffu, special);
      if (lane == 0) sm.wfirst[warp] = bal ? warp * 32 + __ffs(bal) - 1 : kRows;
      __syncthreads();
      int ls = kRows;
#pragma unroll
      for (int w = 0; w < NW; ++w) ls = min(ls, sm.wfirst[w]);
      if (tid == ls) sm.S = serial_add(__fadd_rn(S, __fmul_rn(excl, q)), T2);
      __syncthreads();
      S = sm.S;
      from = ls + 1;
      __syncthreads();  // smem reuse by the next round
    } else if (S == 0.0f) {
      // fl(0 + t) = t: runs of zero terms commit nothing; the first thread
      // holding a non-zero (or NaN) term goes serial.
      bool nz = false;
      if (mine) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float t0, t1;
          f2_unpack(T2[k], t0, t1);
          nz |= (t0 != 0.0f) | (t1 != 0.0f);
        }
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
        if (tid == ls) sm.S = serial_add(S, T2);
        __syncthreads();
        S = sm.S;
        from = ls + 1;
      }
      __syncthreads();
    } else if (!isfinite(S)) {
      // inf or NaN absorbs every later term the same way in any order.
      float loc = 0.0f;
      if (mine) loc = serial_add(0.0f, T2);
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
      if (tid == ls) sm.S = serial_add(S, T2);
      __syncthreads();
      S = sm.S;
      from = ls + 1;
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Group parameters and code thresholds (quantize.cu:153-176).
//
// The reference's code of a value w is
//   q(w) = clamp((int)roundf((w - gmin) / scale), 0, L-1)
// which is non-decreasing in w.  For a group whose zero point and scale are
// not clamped ("regular"), |w - scale*(q-zero)| is at most about one scale
// for every w in [gmin, gmax], below the outlier threshold (0.4*range = 1.2
// scale for 2-bit, 0.15*range = 2.25 scale for 4-bit): no outliers exist and
// q(w) is described by the L-1 smallest fp16 values reaching each code.
// Each threshold is found by evaluating the reference formula next to its
// approximate position and walking fp16 values in order (binary search if
// the walk is long).  Other groups use the formula per element in `encode`.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int code_of(float x, float gmin, float scale, int L) {
  const float a = __fdiv_rn(__fsub_rn(x, gmin), scale);
  const int q = f2i_rz(roundf(a));
  return max(0, min(L - 1, q));
}

constexpr int kOrdMin = -31744, kOrdEnd = 31744;  // finite fp16 values in order: [min, end)

__device__ __forceinline__ uint16_t ord_to_half_bits(int ord) {
  return ord >= 0 ? (uint16_t)ord : (uint16_t)(0x8000 | (-ord - 1));
}
__device__ __forceinline__ int half_bits_to_ord(uint16_t b) {
  return (b & 0x8000) ? -(int)(b & 0x7FFF) - 1 : (int)b;
}
__device__ __forceinline__ float ord_val(int ord) {
  return __half2float(__ushort_as_half(ord_to_half_bits(ord)));
}

// Smallest finite fp16 (in value order) whose code is >= level; 0x7C00 if none.
__device__ uint16_t find_threshold(float gmin, float scale, int L, int level) {
  const float guess = __fadd_rn(gmin, __fmul_rn((float)level - 0.5f, scale));
  int o = half_bits_to_ord(__half_as_ushort(__float2half_rn(guess)));
  o = max(kOrdMin, min(kOrdEnd - 1, o));
  int lo, hi;  // answer in [lo, hi]; hi == kOrdEnd means none
  if (code_of(ord_val(o), gmin, scale, L) >= level) {
    // walk down while the previous value still reaches `level`
    int steps = 0;
    while (o > kOrdMin && steps < 64 && code_of(ord_val(o - 1), gmin, scale, L) >= level) {
      --o;
      ++steps;
    }
    if (o == kOrdMin || steps < 64) return ord_to_half_bits(o);
    lo = kOrdMin;
    hi = o;
  } else {
    int steps = 0;
    while (o < kOrdEnd - 1 && steps < 64 && code_of(ord_val(o + 1), gmin, scale, L) < level) {
      ++o;
      ++steps;
    }
    if (o == kOrdEnd - 1) return 0x7C00;
    if (steps < 64) return ord_to_half_bits(o + 1);
    lo = o + 1;
    hi = kOrdEnd;
  }
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;  // arithmetic shift: floor for negatives
    if (code_of(ord_val(mid), gmin, scale, L) >= level)
      hi = mid;
    else
      lo = mid + 1;
  }
  return lo < kOrdEnd ? ord_to_half_bits(lo) : (uint16_t)0x7C00;
}

__device__ void group_scalars(float gmin, float gmax, int L, GroupParams& p) {
  const float range = __fsub_rn(gmax, gmin);
  const float scale_raw = __fdiv_rn(range, (float)(L - 1));
  float scale = scale_raw;
  if (scale < 1e-8f) scale = 1e-8f;
  const int zr = f2i_rz(roundf(__fdiv_rn(-gmin, scale)));
  const float thr = L == 4 ? __fmul_rn(0.4f, range) : __fmul_rn(0.15f, range);
  const bool regular = isfinite(gmin) && isfinite(gmax) && (scale_raw >= 1e-8f) && zr >= 0 &&
                       zr <= L - 1 && isfinite(thr);
  p.gmin = gmin;
  p.gmax = gmax;
  p.scale = scale;
  p.thr = thr;
  p.zero = max(0, min(L - 1, zr));
  p.levels = L;
  p.flags = regular ? kFlagRegular : 0;
  p.scale_h = __half_as_ushort(__float2half_rn(scale));
}

// ---------------------------------------------------------------------------
// stats kernel
// ---------------------------------------------------------------------------
struct StatsArgs {
  const __half* W;
  int64_t M, K;
  int ng;
  int stages;  // TMA ring depth
  const float* hess;
  Workspace ws;
  uint8_t* gp;
  ChunkLayout cl;
  int n4;      // 4-bit groups to select
  int select;  // the selection runs (sensitivity needed)
  int w_aligned;
  size_t scratch_bytes;  // dynamic shared memory available to finalize
};

template <int NT>
__device__ void finalize(const StatsArgs& a, uint8_t* scratch);

template <int NW, bool kSens, bool kTma>
__global__ void __launch_bounds__(NW * 32, NW <= 4 ? 6 : (NW <= 8 ? 3 : 1))
    stats_kernel(const __grid_constant__ CUtensorMap tmap, const StatsArgs a) {
  constexpr int kRows = NW * 32;
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ uint64_t full_bar[kMaxStages];
  __shared__ ScanSmem<NW> sm;
  __shared__ float red[2][NW];
  __shared__ int s_flag;
  const int g = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t M = a.M, K = a.K;
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, K - c0);
  const int64_t nst = ceil_div(M, kRows);
  const int D = a.stages;

  if (kTma) {
    if (tid == 0) {
      for (int s = 0; s < D; ++s) mbar_init(&full_bar[s], 1);
      fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
      for (int s = 0; s < D && s < nst; ++s) {
        mbar_arrive_expect_tx(&full_bar[s], kRows * 32);
        tma_load_2d(dsm + (size_t)s * kRows * 32, &tmap, &full_bar[s], (int)c0, s * kRows);
      }
    }
  }

  // Divisor per column: the reference divides w*w by h when h > 1e-8.  For
  // h in [2^-60, 2^60] the correctly rounded quotient is
  //   q0 = x * r,  q1 = fma(fma(-q0, h, x), r, q0),  r = RN(1/h)
  // for every dividend x = w*w of an fp16 w (checked exhaustively for all
  // fp32 divisor significands by tests/test_division.py).  h <= 1e-8 (or NaN)
  // takes w*w unchanged: h = r = 1 makes the same three operations exact.
  __shared__ uint64_t sR2[8], sNH2[8];  // per column pair: RN(1/h) and -h
  bool slow_div = false, divide = false;
  if (kSens) {
    float hv[16], rv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float h = (i < gs) ? __ldg(a.hess + c0 + i) : 1.0f;
      if (h > 1e-8f) {
        hv[i] = h;
        rv[i] = __frcp_rn(h);
        slow_div |= !(h >= 0x1p-60f && h <= 0x1p60f);
        divide |= (h != 1.0f);
      } else {
        hv[i] = 1.0f;
        rv[i] = 1.0f;
      }
    }
    if (tid < 8) {
      sR2[tid] = f2_pack(rv[2 * tid], rv[2 * tid + 1]);
      sNH2[tid] = f2_pack(-hv[2 * tid], -hv[2 * tid + 1]);
    }
    __syncthreads();
  }

  __half2 hmn = __float2half2_rn(INFINITY), hmx = __float2half2_rn(-INFINITY);
  const __half2 hnan = as_h2(0x7E007E00u);
  float S = 0.0f;
  bool abort = false;
  int64_t s_abort = 0;
  const bool vec = a.w_aligned && (gs == kGroup1) && ((K & 7) == 0);
  Row16 nxt;
  if (!kTma && tid < M) nxt = load_row16(a.W, tid, K, c0, gs, vec);

  for (int64_t s = 0; s < nst; ++s) {
    const int64_t r = s * kRows + tid;
    const bool valid = r < M;
    Row16 cur;
    if (kTma) {
      const int slot = (int)(s % D);
      const bool ok = mbar_wait(&full_bar[slot], (uint32_t)((s / D) & 1));
      if (__syncthreads_or(!ok)) {
        abort = true;
        s_abort = s;
        break;
      }
      const uint4* src = reinterpret_cast<const uint4*>(dsm + (size_t)slot * kRows * 32) + 2 * tid;
      cur.lo = src[0];
      cur.hi = src[1];
    } else {
      cur = nxt;
      if (r + kRows < M) nxt = load_row16(a.W, r + kRows, K, c0, gs, vec);
      if (!valid) cur.lo = cur.hi = make_uint4(0, 0, 0, 0);
    }
    // min / max in fp16 (exact): elements outside the matrix become NaN,
    // which min/max ignore -- as fminf/fmaxf ignore NaN weights.
    const bool full = valid && gs == kGroup1;
    if (full) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const __half2 w2 = as_h2(row_word(cur, k));
        hmn = __hmin2(hmn, w2);
        hmx = __hmax2(hmx, w2);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        __half2 w2 = as_h2(row_word(cur, k));
        if (!valid || 2 * k >= gs) {
          w2 = hnan;
        } else if (2 * k + 1 >= gs) {
          w2 = __halves2half2(__low2half(w2), __high2half(hnan));
        }
        hmn = __hmin2(hmn, w2);
        hmx = __hmax2(hmx, w2);
      }
    }
    if (kSens) {
      // terms t = (h > 1e-8 ? w*w / h : w*w), packed in pairs
      uint64_t T2[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t w = row_word(cur, k);
        const uint64_t x2 =
            f2_pack(f16_square((uint16_t)(w & 0xFFFFu)), f16_square((uint16_t)(w >> 16)));
        T2[k] = x2;
        if (divide) {
          const uint64_t r2 = sR2[k];
          const uint64_t q0 = f2_mul(x2, r2);
          T2[k] = f2_fma(f2_fma(q0, sNH2[k], x2), r2, q0);
        }
      }
      if (slow_div) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t w = row_word(cur, k);
          float h0, h1;
          f2_unpack(sNH2[k], h0, h1);
          T2[k] = f2_pack(__fdiv_rn(f16_square((uint16_t)(w & 0xFFFFu)), -h0),
                          __fdiv_rn(f16_square((uint16_t)(w >> 16)), -h1));
        }
      }
      if (!full) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float t0, t1;
          f2_unpack(T2[k], t0, t1);
          if (!valid || 2 * k >= gs) t0 = 0.0f;
          if (!valid || 2 * k + 1 >= gs) t1 = 0.0f;
          T2[k] = f2_pack(t0, t1);
        }
      }
      sens_stage<NW>(S, T2, sm);  // ends with __syncthreads: the slot is free
    } else {
      __syncthreads();
    }
    if (kTma && tid == 0 && s + D < nst) {
      const int slot = (int)(s % D);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&full_bar[slot], kRows * 32);
      tma_load_2d(dsm + (size_t)slot * kRows * 32, &tmap, &full_bar[slot], (int)c0,
                  (int)((s + D) * kRows));
    }
  }
  if (abort) {
    // a TMA load never completed: record it, then wait (bounded) for the
    // loads still in flight (stages s_abort .. s_abort + D - 1) before the
    // block's shared memory is released
    if (tid == 0) {
      atomicOr(&a.ws.hdr->status, kStatusTimeout);
      for (int64_t k = s_abort; k < nst && k < s_abort + D; ++k)
        (void)mbar_wait(&full_bar[k % D], (uint32_t)((k / D) & 1));
    }
    __syncthreads();
  }

  // block min / max; the reference starts from +-1e10f and ignores NaN, which
  // equals clamping the exact min / max to +-1e10
  const __half hmin1 = __hmin(__low2half(hmn), __high2half(hmn));
  const __half hmax1 = __hmax(__low2half(hmx), __high2half(hmx));
  float mn = warp_min(__half2float(hmin1));
  float mx = warp_max(__half2float(hmax1));
  if (lane == 0) {
    red[0][warp] = mn;
    red[1][warp] = mx;
  }
  __syncthreads();
  mn = red[0][0];
  mx = red[1][0];
#pragma unroll
  for (int w = 1; w < NW; ++w) {
    mn = fminf(mn, red[0][w]);
    mx = fmaxf(mx, red[1][w]);
  }
  mn = fminf(1e10f, mn);
  mx = fmaxf(-1e10f, mx);
  if (tid == 0) {
    a.ws.gmin[g] = mn;
    a.ws.gmax[g] = mx;
    if (kSens) a.ws.sens[g] = S;
  }
  // parameters of this group for both precisions: threads 0-2 find the
  // 2-bit thresholds, threads 3-17 the 4-bit ones
  GroupParams* p2 = a.ws.params + 2 * g;
  GroupParams* p4 = p2 + 1;
  if (tid < 18) {
    const bool four = tid >= 3;
    const int L = four ? 16 : 4;
    const int level = four ? tid - 2 : tid + 1;
    GroupParams p;
    group_scalars(mn, mx, L, p);
    const uint16_t T =
        (p.flags & kFlagRegular) ? find_threshold(mn, p.scale, L, level) : (uint16_t)0x7C00;
    GroupParams* d = four ? p4 : p2;
    d->thresh[level - 1] = T;
    if (tid == 0 || tid == 3) {
      d->gmin = p.gmin;
      d->gmax = p.gmax;
      d->scale = p.scale;
      d->thr = p.thr;
      d->zero = p.zero;
      d->levels = p.levels;
      d->flags = p.flags;
      d->scale_h = p.scale_h;
    }
  } else if (tid < 32) {
    // unused threshold slots: 2-bit slots 3..15 and the 4-bit slot 15
    const int j = tid - 18;  // 0..13
    if (j < 13)
      p2->thresh[3 + j] = 0x7C00;
    else
      p4->thresh[15] = 0x7C00;
  }
  // zero this CTA's share of the per-row outlier counts
  {
    const int64_t r0 = M * g / gridDim.x, r1 = M * (g + 1) / gridDim.x;
    for (int64_t r = r0 + tid; r < r1; r += blockDim.x) a.ws.row_counts[r] = 0;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_flag = atomicAdd(&a.ws.hdr->ticket_stats, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  finalize<NW * 32>(a, dsm);
}

// ---------------------------------------------------------------------------
// finalize (last stats CTA): 4-bit selection and the 2nd-order tables.
//
// Selection -- the n4 largest sensitivities are 4-bit (torch_ops.cu:163-178).
// Sensitivities are >= 0, so their fp32 bit patterns order like the
// reference's float comparison.  A radix select (4 passes of 8 bits) finds
// the n4-th largest key T; groups above T are selected, and among groups
// equal to T the lowest indices fill the remaining slots.  If equal keys
// straddle the boundary the status records a tie (the reference's std::sort
// leaves that order unspecified).
// ---------------------------------------------------------------------------
template <int NT>
__device__ void finalize(const StatsArgs& a, uint8_t* scratch) {
  const int ng = a.ng;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NWARP = NT / 32;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_need;
  __shared__ uint32_t s_wsum[NWARP];
  __shared__ int s_irr;
  const uint32_t* keys = reinterpret_cast<const uint32_t*>(a.ws.sens);

  if (a.select && a.n4 > 0) {
    if (tid == 0) {
      s_prefix = 0;
      s_need = (uint32_t)a.n4;
    }
    uint32_t mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += NT) hist[i] = 0;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int i = tid; i < ng; i += NT) {
        const uint32_t k = __ldcg(keys + i);
        if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (warp == 0) {
        // suffix sums over bins, highest bin first; lane l owns bins 8l..8l+7
        uint32_t c[8], tot = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = hist[lane * 8 + j];
          tot += c[j];
        }
        uint32_t suf = tot;  // sum over lanes >= lane
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += y;
        }
        const uint32_t need = s_need;
        const uint32_t above = suf - tot;  // in lanes > lane
        const bool here = above < need && suf >= need;
        const unsigned bal = __ballot_sync(0xffffffffu, here);
        const int L = __ffs(bal) - 1;
        if (lane == L) {
          uint32_t acc = above;
          int b = 7;
          for (; b > 0; --b) {
            if (acc + c[b] >= need) break;
            acc += c[b];
          }
          s_prefix = prefix | ((uint32_t)(lane * 8 + b) << shift);
          s_need = need - acc;
        }
      }
      mask |= 0xFFu << shift;
      __syncthreads();
    }
    const uint32_t T = s_prefix, need_eq = s_need;
    // rank equal keys by index: contiguous index ranges per thread
    const int per = (ng + NT - 1) / NT;
    const int i0 = min(ng, tid * per), i1 = min(ng, i0 + per);
    uint32_t eq = 0;
    for (int i = i0; i < i1; ++i) eq += (__ldcg(keys + i) == T);
    uint32_t incl = eq;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    uint32_t off = 0, total_eq = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      if (w < warp) off += s_wsum[w];
      total_eq += s_wsum[w];
    }
    uint32_t rank = off + incl - eq;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = __ldcg(keys + i);
      uint8_t sel = k > T;
      if (k == T) {
        sel = rank < need_eq;
        ++rank;
      }
      a.gp[i] = sel;
      a.ws.prec[i] = sel;
    }
    if (tid == 0 && total_eq > need_eq) atomicOr(&a.ws.hdr->status, kStatusTie);
  } else {
    for (int i = tid; i < ng; i += NT) {
      a.gp[i] = 0;
      a.ws.prec[i] = 0;
    }
  }
  if (tid == 0) s_irr = 0;
  __syncthreads();

  // scales of the selected precision -> 2nd-order table (quantize.cu:245-272,
  // over the flattened [M, ng] scales; scales_1st[r, g] depends only on g, so
  // full chunks repeat with period ng / gcd(ng, 256))
  float* s1 = reinterpret_cast<float*>(scratch);
  const bool s1_in_smem = (size_t)ng * sizeof(float) <= a.scratch_bytes;
  int irr = 0;
  for (int g = tid; g < ng; g += NT) {
    const GroupParams& p = a.ws.params[2 * g + a.ws.prec[g]];
    if (s1_in_smem) s1[g] = __half2float(__ushort_as_half((uint16_t)p.scale_h));
    irr |= !(p.flags & kFlagRegular);
  }
  if (irr) atomicOr(&s_irr, 1);
  __syncthreads();
  auto scale_of = [&](int g) -> float {
    return s1_in_smem ? s1[g]
                      : __half2float(__ushort_as_half(
                            (uint16_t)a.ws.params[2 * g + a.ws.prec[g]].scale_h));
  };
  const ChunkLayout& cl = a.cl;
  const int nchunks = cl.ntab_full + cl.has_partial;
  for (int ci = warp; ci < nchunks; ci += NWARP) {
    const int64_t cidx = ci < cl.ntab_full ? ci : cl.nfull;  // the partial chunk is the last
    const int64_t s0 = cidx * kGroup2, s1e = min64(s0 + kGroup2, cl.total);
    float mn = 1e10f, mx = -1e10f;
    for (int64_t i = s0 + lane; i < s1e; i += 32) {
      const float v = scale_of((int)(i % ng));
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    mn = warp_min(mn);
    mx = warp_max(mx);
    if (lane == 0) {
      float sc2 = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
      if (sc2 < 1e-10f) sc2 = 1e-10f;
      const int z2 = f2i_rz(roundf(__fdiv_rn(-mn, sc2)));
      const int slot = ci < cl.ntab_full ? ci : cl.ntab_full;
      a.ws.chunk_tab[slot] =
          make_float4(mn, sc2, __int_as_float((int)__half_as_ushort(__float2half_rn(sc2))),
                      __int_as_float((int)(int8_t)z2));
    }
  }
  // group order for encode: 2-bit groups first, then 4-bit, each ascending,
  // so that a warp of encode threads shares one precision
  {
    const int per = (ng + NT - 1) / NT;
    const int i0 = min(ng, tid * per), i1 = min(ng, i0 + per);
    uint32_t n2 = 0;
    for (int i = i0; i < i1; ++i) n2 += (a.ws.prec[i] == 0);
    uint32_t incl = n2;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    __syncthreads();
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    uint32_t off = 0, total2 = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      if (w < warp) off += s_wsum[w];
      total2 += s_wsum[w];
    }
    uint32_t pos2 = off + incl - n2;            // 2-bit slots before my range
    uint32_t pos4 = total2 + (uint32_t)i0 - pos2;  // 4-bit slots before my range
    for (int i = i0; i < i1; ++i) {
      if (a.ws.prec[i] == 0)
        a.ws.order[pos2++] = i;
      else
        a.ws.order[pos4++] = i;
    }
    if (tid == 0) a.ws.hdr->n2 = total2;
  }
  if (tid == 0) {
    a.ws.hdr->any_irregular = s_irr;
    a.ws.hdr->ticket_stats = 0;
  }
}

// ---------------------------------------------------------------------------
// encode: one thread per (row, group), kEncRows rows per thread, loaded four
// rows at a time.
// ---------------------------------------------------------------------------
constexpr int kEncThreads = 64;
constexpr int kEncRows = 16;

struct EncodeArgs {
  const __half* W;
  int64_t M, K;
  int ng;
  int w_aligned;
  Workspace ws;
  ChunkLayout cl;
  int32_t* packed2;
  int32_t* packed4;
  __half* scales1;
  int8_t* zeros1;
  __half* scales2;
  int8_t* zeros2;
  uint8_t* sq;
  int32_t* row_ptrs;
  int32_t* nnz;
  int fma_mode;
};

__device__ __forceinline__ bool is_outlier(float x, float scale, int zero, float thr, int q,
                                           int fma_mode) {
  const float qz = (float)(q - zero);
  const float err = fma_mode ? fabsf(__fmaf_rn(-scale, qz, x))
                             : fabsf(__fsub_rn(x, __fmul_rn(scale, qz)));
  return err > thr;
}

__global__ void __launch_bounds__(kEncThreads, 16) encode_kernel(const EncodeArgs a) {
  grid_dependency_wait();  // stats (and its finalize) complete
  const int64_t M = a.M, K = a.K;
  const int ng = a.ng;
  const bool any_irr = *reinterpret_cast<volatile uint32_t*>(&a.ws.hdr->any_irregular) != 0;
  const int64_t gtid = ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gthreads = (int64_t)gridDim.x * gridDim.y * blockDim.x;

  // 2nd-order scales / zeros of every chunk, from the periodic table
  for (int64_t c = gtid; c < a.cl.ng2; c += gthreads) {
    const float4 e = a.ws.chunk_tab[c < a.cl.nfull ? (int)(c % a.cl.period) : a.cl.ntab_full];
    a.scales2[c] = __ushort_as_half((uint16_t)__float_as_int(e.z));
    a.zeros2[c] = (int8_t)__float_as_int(e.w);
  }
  if (!any_irr) {
    for (int64_t r = gtid; r <= M; r += gthreads) a.row_ptrs[r] = 0;
    if (gtid == 0) *a.nnz = 0;
  }

  // thread slot -> group: 2-bit groups first, so a warp shares one precision
  const int slot = blockIdx.x * kEncThreads + threadIdx.x;
  if (slot < ng) {
    const int g = a.ws.order[slot];
    const bool four = a.ws.prec[g] != 0;
    const GroupParams& pp = a.ws.params[2 * g + (four ? 1 : 0)];
    const float gmin = pp.gmin, scale = pp.scale, thr = pp.thr;
    const int zero = pp.zero, levels = pp.levels;
    const bool regular = (pp.flags & kFlagRegular) != 0;
    const __half sh = __ushort_as_half((uint16_t)pp.scale_h);
    const float s1f = __half2float(sh);
    const int64_t c0 = (int64_t)g * kGroup1;
    const int gs = (int)min64(kGroup1, K - c0);
    const bool vec = a.w_aligned && (gs == kGroup1) && ((K & 7) == 0);
    const uint4 tA = *reinterpret_cast<const uint4*>(&pp.thresh[0]);
    const uint4 tB = *reinterpret_cast<const uint4*>(&pp.thresh[8]);
    // threshold j as a broadcast half2
    auto T2 = [&](int j) -> __half2 {
      const uint32_t w = j < 8 ? (&tA.x)[j >> 1] : (&tB.x)[(j - 8) >> 1];
      const uint16_t h = (j & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFFu);
      return __half2half2(__ushort_as_half(h));
    };
    // columns past K in a partial group hold code 0 in the reference
    const uint32_t keep2 = gs >= 16 ? 0xFFFFFFFFu : ((1u << (2 * gs)) - 1u);
    const uint32_t keep4a = gs >= 8 ? 0xFFFFFFFFu : ((1u << (4 * gs)) - 1u);
    const uint32_t keep4b =
        gs >= 16 ? 0xFFFFFFFFu : (gs <= 8 ? 0u : ((1u << (4 * (gs - 8))) - 1u));
    const int64_t r0 = (int64_t)blockIdx.y * kEncRows;
    const int64_t r1 = min64(M, r0 + kEncRows);
    // position of (r, g) within one period of full 2nd-order chunks
    // (period * 256 = lcm(ng, 256) flat indices); its chunk is jt >> 8.
    // Advanced by ng per row.
    const int P256 = a.cl.period * kGroup2;
    int jt = (int)((r0 * ng + g) % P256);
    const int64_t full_end = a.cl.nfull * kGroup2;  // later flat indices: partial chunk
    for (int64_t rb = r0; rb < r1; rb += 2) {
      Row16 vb[2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
        if (rb + u < r1) vb[u] = load_row16(a.W, rb + u, K, c0, gs, vec);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int64_t r = rb + u;
        if (r >= r1) break;
        const Row16& v = vb[u];
        uint32_t wa = 0, wb = 0;
        int cnt = 0;
        if (regular) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const __half2 w2 = as_h2(row_word(v, k));
            __half2 acc = __float2half2_rn(1024.0f);
            if (!four) {
#pragma unroll
              for (int j = 0; j < 3; ++j) acc = __hadd2(acc, __hge2(w2, T2(j)));
            } else {
#pragma unroll
              for (int j = 0; j < 15; ++j) acc = __hadd2(acc, __hge2(w2, T2(j)));
            }
            // 1024 has an fp16 ulp of 1: the code sits in the low mantissa bits
            const uint32_t b = h2_bits(acc);
            if (!four) {
              wa |= ((b & 0x3u) | ((b >> 14) & 0xCu)) << (4 * k);
            } else {
              const uint32_t t = (b & 0xFu) | ((b >> 12) & 0xF0u);
              if (k < 4)
                wa |= t << (8 * k);
              else
                wb |= t << (8 * (k - 4));
            }
          }
          if (!four) {
            wa &= keep2;
          } else {
            wa &= keep4a;
            wb &= keep4b;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (i < gs) {
              const float x = row_elem(v, i);
              const int q = code_of(x, gmin, scale, levels);
              cnt += is_outlier(x, scale, zero, thr, q, a.fma_mode);
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
        a.packed2[si] = four ? 0 : (int32_t)wa;
        reinterpret_cast<int2*>(a.packed4)[si] =
            four ? make_int2((int)wa, (int)wb) : make_int2(0, 0);
        a.scales1[si] = sh;
        a.zeros1[si] = (int8_t)zero;
        // 2nd-order code (quantize.cu:274-280)
        const float4 ch = a.ws.chunk_tab[si < full_end ? (jt >> 8) : a.cl.ntab_full];
        const int q2 = f2i_rz(roundf(__fdiv_rn(__fsub_rn(s1f, ch.x), ch.y)));
        a.sq[si] = (uint8_t)max(0, min(15, q2));
        jt += ng;
        if (jt >= P256) jt -= P256;
        if (cnt) atomicAdd(a.ws.row_counts + r, cnt);
      }
    }
  }
  if (!any_irr) return;

  // the last CTA turns per-row counts into row pointers
  __shared__ int s_last;
  __shared__ long long part[kEncThreads];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0)
    s_last = atomicAdd(&a.ws.hdr->ticket_encode, 1u) == gridDim.x * gridDim.y - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int t = threadIdx.x;
  const int64_t per = ceil_div(M, (int64_t)kEncThreads);
  const int64_t q0 = min64(M, t * per), q1 = min64(M, q0 + per);
  long long s = 0;
  for (int64_t r = q0; r < q1; ++r) s += __ldcg(a.ws.row_counts + r);
  part[t] = s;
  __syncthreads();
  for (int o = 1; o < kEncThreads; o <<= 1) {
    const long long y = t >= o ? part[t - o] : 0;
    __syncthreads();
    part[t] += y;
    __syncthreads();
  }
  long long run = part[t] - s;
  if (t == 0) a.row_ptrs[0] = 0;
  for (int64_t r = q0; r < q1; ++r) {
    run += __ldcg(a.ws.row_counts + r);
    a.row_ptrs[r + 1] = (int32_t)run;
  }
  if (t == kEncThreads - 1) *a.nnz = (int32_t)part[t];
  if (t == 0) a.ws.hdr->ticket_encode = 0;
}

// extract: one warp per row with outliers; only non-regular groups can hold
// them.  Lanes 0-15 take the group's 16 columns; the ballot order is the
// column order.
__global__ void __launch_bounds__(256)
    extract_kernel(const __half* __restrict__ W, int64_t M, int64_t K, int ng,
                   const GroupParams* __restrict__ params, const uint8_t* __restrict__ prec,
                   const int32_t* __restrict__ row_ptrs, __half* __restrict__ vals,
                   int32_t* __restrict__ cols, int fma_mode) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= M) return;
  int32_t o = row_ptrs[r];
  const int32_t end = row_ptrs[r + 1];
  if (o == end) return;
  for (int g = 0; g < ng && o < end; ++g) {
    const GroupParams& p = params[2 * g + prec[g]];
    if (p.flags & kFlagRegular) continue;
    const int64_t c = (int64_t)g * kGroup1 + lane;
    bool out = false;
    __half wv = __ushort_as_half(0);
    if (lane < kGroup1 && c < K) {
      wv = W[r * K + c];
      const float x = __half2float(wv);
      out = is_outlier(x, p.scale, p.zero, p.thr, code_of(x, p.gmin, p.scale, p.levels),
                       fma_mode);
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

// Outlier-test arithmetic of the reference kernel: the product
// scale*(q-zero) fused into the subtraction (one rounding).  Established
// against the compiled reference by tests/test_gpu_parity.py.
constexpr int kOutlierFma = 1;

mb_status check_common(const void* weights, int64_t M, int64_t K) {
  MB_REQUIRE(weights != nullptr, "weights must not be null");
  MB_REQUIRE(M > 0 && K > 0, "weights must be a non-empty 2D [M, K] matrix");
  MB_REQUIRE(M * ceil_div(K, kGroup1) < (int64_t)INT32_MAX && M * K < (int64_t)INT32_MAX,
             "weights too large: M*K must be below 2^31 (int32 outlier indexing)");
  return MB_OK;
}

template <int NW, bool kSens, bool kTma>
mb_status launch_stats(const CUtensorMap& tmap, const StatsArgs& a, size_t smem,
                       cudaStream_t stream) {
  auto kern = stats_kernel<NW, kSens, kTma>;
  static std::atomic<uint64_t> attr_done{0};  // per instantiation, one bit per device
  MB_CUDA_TRY(set_smem_limit_once(kern, 96 * 1024, attr_done));
  kern<<<(unsigned)a.ng, NW * 32, smem, stream>>>(tmap, a);
  MB_LAUNCH_CHECK("stats_kernel");
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
  const size_t need = workspace_layout(M, K, nullptr, nullptr);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(MB_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) +
                                           " bytes, got " + std::to_string(workspace_bytes));
  MB_REQUIRE((reinterpret_cast<uintptr_t>(packed_2bit) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(packed_4bit) & 7u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_1st_fp16) & 1u) == 0 &&
                 (reinterpret_cast<uintptr_t>(scales_2nd_fp16) & 1u) == 0 &&
                 (reinterpret_cast<uintptr_t>(outlier_row_ptrs) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(nnz_device) & 3u) == 0 &&
                 (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
             "misaligned output or workspace pointer (packed_4bit needs 8 bytes, "
             "int32/fp16 outputs natural alignment, workspace 256 bytes)");
  MB_REQUIRE(ceil_div(M, kEncRows) <= 65535, "too many rows for the encode grid");
  Workspace ws;
  workspace_layout(M, K, static_cast<char*>(workspace), &ws);
  const bool selecting = hessian_diag != nullptr && hessian_numel > 0 && ratio_4bit > 0.0;
  if (selecting) MB_REQUIRE(hessian_numel >= K, "hessian_diag must hold at least K values");
  int64_t n4 = 0;
  if (selecting) {
    n4 = (int64_t)(int)(ratio_4bit * (double)(int)ng);  // torch_ops.cu:172
    n4 = std::max<int64_t>(0, std::min<int64_t>(n4, ng));
  }
  const bool sens = selecting && n4 > 0;
  const bool w_aligned = (reinterpret_cast<uintptr_t>(weights_fp16) & 15u) == 0;

  MB_CUDA_TRY(cudaMemsetAsync(ws.hdr, 0, sizeof(Header), stream));

  StatsArgs sa;
  sa.W = static_cast<const __half*>(weights_fp16);
  sa.M = M;
  sa.K = K;
  sa.ng = (int)ng;
  sa.hess = hessian_diag;
  sa.ws = ws;
  sa.gp = group_precision;
  sa.cl = chunk_layout(M, ng);
  sa.n4 = (int)n4;
  sa.select = sens;
  sa.w_aligned = w_aligned;

  // TMA needs a 16-byte aligned base and a row pitch that is a multiple of 16
  // bytes; other inputs take the direct-load variant of the same kernel.
  CUtensorMap tmap;
  std::memset(&tmap, 0, sizeof(tmap));
  const bool small_ng = ng < 2 * 148;
  const int NW = small_ng ? 8 : 4;
  const int rows = NW * 32;
  const bool tma = w_aligned && (K % 8 == 0) &&
                   make_tensor_map_2d_f16(&tmap, weights_fp16, (uint64_t)M, (uint64_t)K, rows, 16);
  sa.stages = small_ng ? 6 : 8;
  const size_t smem = (size_t)sa.stages * rows * 32;  // ring buffer, then finalize scratch
  sa.scratch_bytes = smem;
  mb_status st;
  if (NW == 8) {
    if (tma)
      st = sens ? launch_stats<8, true, true>(tmap, sa, smem, stream)
                : launch_stats<8, false, true>(tmap, sa, smem, stream);
    else
      st = sens ? launch_stats<8, true, false>(tmap, sa, smem, stream)
                : launch_stats<8, false, false>(tmap, sa, smem, stream);
  } else {
    if (tma)
      st = sens ? launch_stats<4, true, true>(tmap, sa, smem, stream)
                : launch_stats<4, false, true>(tmap, sa, smem, stream);
    else
      st = sens ? launch_stats<4, true, false>(tmap, sa, smem, stream)
                : launch_stats<4, false, false>(tmap, sa, smem, stream);
  }
  if (st) return st;

  EncodeArgs ea;
  ea.W = sa.W;
  ea.M = M;
  ea.K = K;
  ea.ng = (int)ng;
  ea.w_aligned = w_aligned;
  ea.ws = ws;
  ea.cl = sa.cl;
  ea.packed2 = packed_2bit;
  ea.packed4 = packed_4bit;
  ea.scales1 = static_cast<__half*>(scales_1st_fp16);
  ea.zeros1 = zeros_1st;
  ea.scales2 = static_cast<__half*>(scales_2nd_fp16);
  ea.zeros2 = zeros_2nd;
  ea.sq = scales_1st_quant;
  ea.row_ptrs = outlier_row_ptrs;
  ea.nnz = nnz_device;
  ea.fma_mode = kOutlierFma;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(ng, kEncThreads), (unsigned)ceil_div(M, kEncRows));
  cfg.blockDim = dim3(kEncThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MB_CUDA_TRY(cudaLaunchKernelEx(&cfg, encode_kernel, ea));
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
      static_cast<const __half*>(weights_fp16), M, K, (int)ng, ws.params, ws.prec,
      outlier_row_ptrs, static_cast<__half*>(outlier_values_fp16), outlier_col_indices,
      kOutlierFma);
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
  MB_CUDA_TRY(cudaMemcpyAsync(flags, &ws.hdr->status, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                              stream));
  MB_CUDA_TRY(cudaStreamSynchronize(stream));
  return MB_OK;
}
