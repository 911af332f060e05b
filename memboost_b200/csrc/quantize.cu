// memboost quantize on sm_100a.
//
// Replaces the reference's six-kernel pipeline with host round trips
// (core/torch_ops.cu:105-264 driving core/quantize.cu:72-321) by three
// stream-ordered kernels and no host synchronisation:
//
//   stats   streams W once from HBM in 128 x 128 tiles through TMA, one warp
//           per 16-column group (quantize.cu:72-128): min / max, and an fp64
//           prediction of the group's serial fp32 sensitivity sum with a
//           rigorous error interval.  The last CTA of each column tile
//           derives its groups' scale / zero / code thresholds for both
//           precisions (quantize.cu:153-176); the last of those selects the
//           4-bit groups (torch_ops.cu:149-179): every group whose interval
//           lies clear of the top-k boundary is decided from the intervals,
//           the few that straddle it are left pending.  When nothing is
//           pending it also builds the 2nd-order tables (quantize.cu:245-281).
//   encode  reads W again (from L2) and writes both packed arrays, scales_1st
//           and zeros_1st of every decided group (quantize.cu:132-242).  When
//           groups are pending, extra CTAs compute their exact serial sums
//           (transfer functions per chunk of rows, assembled in order) and
//           the last of them completes the selection and the tables.
//   post    writes the 2nd-order codes / scales / zeros, encodes the pending
//           groups and turns per-row outlier counts into row pointers
//           (quantize.cu:274-299, torch_ops.cu:210-229).
//   extract (second entry point) CSR values / columns in ascending column
//           order (quantize.cu:301-321).
//
// Arithmetic that decides an output bit uses the reference's fp32 operations,
// written with explicit rounding intrinsics so the compiler cannot contract
// or reorder them.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>

#include "mb_common.cuh"
#include "mb_tma.cuh"

namespace mb {
namespace {

constexpr int kFlagRegular = 1;  // threshold path valid; group cannot hold outliers
constexpr uint32_t kStatusTie = 1u;
constexpr uint32_t kStatusTimeout = 2u;

// stats tiles: 128 columns (8 groups) x 128 rows
constexpr int kTileCols = 128;
constexpr int kTileGroups = kTileCols / kGroup1;  // 8: one warp per group
constexpr int kChunkRows = 128;                   // rows per tile = runs per chunk
constexpr int kStatsThreads = 32 * kTileGroups;   // 256
constexpr int kSteps = kChunkRows / 32;
constexpr int kBoxBytes = kChunkRows * 128;       // one 64-column TMA box (16 KB)
constexpr int kTileBytes = 2 * kBoxBytes;         // 32 KB
constexpr int kStatsSmem = kTileBytes + 1024;     // + alignment slack

// exact sums of pending groups
constexpr int kMaxItems = 8;             // program items per (group, chunk)
constexpr int kItemWindow = 0x40000000;  // item.x of a window
constexpr uint32_t kCntOverflow = 1u << 18;  // icount: the chunk's program overflowed
constexpr uint32_t kGrpNaN = 1u, kGrpInf = 2u, kGrpLoose = 4u;  // per-group prediction flags
constexpr double kEps24 = 5.9604644775390625e-08;  // 2^-24
constexpr int kExactCtas = 148;                    // exact-sum CTAs of the encode grid

// encode: one thread per (group slot, block of kEncRows rows)
constexpr int kEncRows = 16;

// Outlier-test arithmetic of the reference kernel: the product
// scale*(q-zero) fused into the subtraction (one rounding).  Established
// against the compiled reference by tests/test_gpu_parity.py.
constexpr int kOutlierFma = 1;

// Per-group parameters of one precision.  Every row of a group shares them
// (in the reference scale and zero depend only on the group's min/max).
struct __align__(16) GroupParams {
  float gmin, gmax, scale, thr;
  int zero, levels, flags, scale_h;  // scale_h: fp16 bit pattern of scales_1st
  uint16_t thresh[16];               // fp16 patterns T_1..T_{L-1}; 0x7C00 = never
};
static_assert(sizeof(GroupParams) == 64, "GroupParams must stay 64 bytes");

struct __align__(16) Header {
  uint32_t ticket_ct;      // column tiles whose groups are assembled
  uint32_t ticket_post;    // post CTAs finished
  uint32_t status;         // kStatus* bits
  uint32_t any_irregular;  // a group of its selected precision may hold outliers
  uint32_t n2;             // decided 2-bit groups at the front of `order`
  uint32_t n_dec;          // decided groups (2-bit then 4-bit) at the front of `order`
  uint32_t n_pend;         // pending groups after them (ascending)
  uint32_t need;           // how many pending groups are 4-bit
  uint32_t ticket_exact;   // pending groups whose exact sum is assembled
  uint32_t pad[7];
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
  uint32_t* ct_count;   // [nct] stats tiles finished per column tile (zeroed with hdr)
  double* cpred;        // [ng * nrc] chunk prediction sums
  float2* cminmax;      // [ng * nrc] chunk min / max
  uint32_t* cflag;      // [ng * nrc] chunk NaN / inf bits
  double* gpred;        // [ng] predicted sensitivity
  double* gmom;         // [ng] sum over chunks of terms * inclusive prediction
  uint32_t* gflag;      // [ng] kGrp* bits
  uint32_t* gticket;    // [ng] exact-sum chunk programs finished (pending groups)
  int4* items;          // [ng * nrc * kMaxItems] chunk programs (pending groups)
  uint32_t* icount;     // [ng * nrc] item count | NaN / inf / overflow bits
  float* gmin;
  float* gmax;
  float* sens;          // [ng] exact sums (pending groups)
  GroupParams* params;  // [2 * ng]: 2g = 2-bit, 2g + 1 = 4-bit
  float4* chunk_tab;    // [ntab_full + 1]: (min, fp32 scale2, fp16 bits of scale2, zero2)
  int32_t* row_counts;  // [M]
  uint8_t* prec;        // [ng] selected precision (copy of group_precision)
  int32_t* order;       // [ng] decided 2-bit, decided 4-bit, then pending groups
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
  const int64_t nct = ceil_div(K, kTileCols), nrc = ceil_div(M, kChunkRows), nrec = ng * nrc;
  char* p_hdr = take(sizeof(Header) + sizeof(uint32_t) * nct);  // zeroed per call
  char* p_cp = take(sizeof(double) * nrec);
  char* p_mm = take(sizeof(float2) * nrec);
  char* p_cf = take(sizeof(uint32_t) * nrec);
  char* p_gp = take(sizeof(double) * ng);
  char* p_gm = take(sizeof(double) * ng);
  char* p_gf = take(sizeof(uint32_t) * ng);
  char* p_gt = take(sizeof(uint32_t) * ng);
  char* p_it = take(sizeof(int4) * kMaxItems * nrec);
  char* p_ic = take(sizeof(uint32_t) * nrec);
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
    ws->ct_count = reinterpret_cast<uint32_t*>(p_hdr + sizeof(Header));
    ws->cpred = reinterpret_cast<double*>(p_cp);
    ws->cminmax = reinterpret_cast<float2*>(p_mm);
    ws->cflag = reinterpret_cast<uint32_t*>(p_cf);
    ws->gpred = reinterpret_cast<double*>(p_gp);
    ws->gmom = reinterpret_cast<double*>(p_gm);
    ws->gflag = reinterpret_cast<uint32_t*>(p_gf);
    ws->gticket = reinterpret_cast<uint32_t*>(p_gt);
    ws->items = reinterpret_cast<int4*>(p_it);
    ws->icount = reinterpret_cast<uint32_t*>(p_ic);
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

// Run r (0..127) of tile group gi from a tile in shared memory: two 64-column
// TMA boxes written with the 128-byte swizzle (16-byte chunk c of row r sits
// at chunk c ^ (r & 7)), so a warp's 32 runs hit distinct banks.
__device__ __forceinline__ Row16 tile_run(const uint8_t* buf, int gi, int r) {
  const uint8_t* base = buf + (gi >> 2) * kBoxBytes + r * 128;
  const int c0 = 2 * (gi & 3), sw = r & 7;
  Row16 v;
  v.lo = *reinterpret_cast<const uint4*>(base + ((c0 ^ sw) << 4));
  v.hi = *reinterpret_cast<const uint4*>(base + (((c0 + 1) ^ sw) << 4));
  return v;
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

// Parameters of group g for both precisions (one warp): lanes 0-2 find the
// 2-bit thresholds, lanes 3-17 the 4-bit ones.
__device__ void group_params_warp(GroupParams* params, int64_t g, float mn, float mx, int lane) {
  GroupParams* p2 = params + 2 * g;
  GroupParams* p4 = p2 + 1;
  if (lane < 18) {
    const bool four = lane >= 3;
    const int L = four ? 16 : 4;
    const int level = four ? lane - 2 : lane + 1;
    GroupParams p;
    group_scalars(mn, mx, L, p);
    const uint16_t T =
        (p.flags & kFlagRegular) ? find_threshold(mn, p.scale, L, level) : (uint16_t)0x7C00;
    GroupParams* d = four ? p4 : p2;
    d->thresh[level - 1] = T;
    if (lane == 0 || lane == 3) {
      d->gmin = p.gmin;
      d->gmax = p.gmax;
      d->scale = p.scale;
      d->thr = p.thr;
      d->zero = p.zero;
      d->levels = p.levels;
      d->flags = p.flags;
      d->scale_h = p.scale_h;
    }
  } else {
    const int jx = lane - 18;  // 0..13: unused threshold slots
    if (jx < 13)
      p2->thresh[3 + jx] = 0x7C00;
    else
      p4->thresh[15] = 0x7C00;
  }
}

// ---------------------------------------------------------------------------
// The reference's sensitivity of a group is the serial fp32 sum of its M*16
// terms t = (h > 1e-8 ? w*w/h : w*w), row by row (quantize.cu:72-98); every
// term is >= 0 or NaN, so the sum never decreases.  Only the ranking of the
// sums matters (they choose the 4-bit groups), so:
//
//  * The stats pass predicts each sum as P = sum(w*w * RN(1/h)) (fp32 per row,
//    fp64 across rows).  P is within 24 * 2^-24 (relative) of the exact real
//    sum T of the terms, and the fp32 serial sum S is within
//    2^-24 * sum_j S_j of T (each add errs by at most half an ulp of its
//    result).  Per chunk of 128 rows, sum_j S_j <= (1 + D)(1 + 24 * 2^-24) *
//    sum_chunks(terms in chunk * predicted prefix through the chunk) with
//    D = n 2^-24 / (1 - n 2^-24) bounding the drift anywhere; that moment is
//    kept per group.  This gives a rigorous interval around every S.
//  * Groups whose interval lies clear of the top-k boundary are decided from
//    the intervals; only the groups that straddle it ("pending") need their
//    exact S, computed as below.  The result is the same selection as from
//    all exact sums: equal sums that straddle the boundary can only occur
//    among pending groups.
//
// Exact S.  While S stays inside one binade [2^e, 2^(e+1)) all fp32 values
// there are multiples of q = 2^(e-23), so fl(S + t) = S + q * rint(t / q)
// exactly, except that a tie (t / q with fraction .5) rounds to the even
// multiple, which depends on the parity of S / q (and always leaves S / q
// even).  A run of terms (one row's 16) inside binade e is therefore
// summarised by a transfer function of the parity: (increment, parity out)
// for parity 0 and for parity 1; transfer functions compose associatively.
// Each chunk of 128 runs is processed by one warp: the predicted prefix
// before each run and the drift bound prove (or fail to prove) the binade the
// sum stays in; proven runs merge into "stretches" (one binade), unproven
// runs (next to binade crossings) into "windows".  The last warp of the group
// walks the chunk programs from S = 0: a stretch is applied after checking
// that the exact S is in its binade and stays there (else it is replayed), a
// window is replayed exactly.  Non-finite terms settle a group at once: the
// sum is NaN if any term is NaN, else +inf if any term is inf.
// ---------------------------------------------------------------------------
enum RunKind : int { kRunZero = 0, kRunProven = 1, kRunUnproven = 2 };

struct RunTF {
  int kind;
  int e;           // binade (kRunProven)
  int inc0, inc1;  // increments in units of q for incoming parity 0 / 1
  int pout;        // bit 0: parity out for parity 0 in; bit 1: for parity 1 in
};

__device__ __forceinline__ int f32_binade(float s) {  // s > 0, normal
  return (int)((__float_as_uint(s) >> 23) & 0xFFu) - 127;
}
__device__ __forceinline__ int f64_binade(double d) {  // d > 0, normal
  return (int)((__double2hiint(d) >> 20) & 0x7FF) - 1023;
}
__device__ __forceinline__ float pow2f(int k) {  // 2^k, -126 <= k <= 127
  return __uint_as_float((uint32_t)(k + 127) << 23);
}

// Per-column division constants of one group: packed (RN(1/h), -h) pairs and
// the group's mode (0: no division, 1: corrected product, 2: IEEE division).
struct GroupDiv {
  uint64_t R2[8], NH2[8];
  int mode;
};

// One warp: lanes 0..15 take one column each.  For h in [2^-60, 2^60] the
// correctly rounded quotient x / h is
//   q0 = x * r,  q1 = fma(fma(-q0, h, x), r, q0),  r = RN(1/h)
// for every x = w*w of an fp16 w (checked exhaustively for all fp32 divisor
// significands by tests/test_division.py); other h take an IEEE division.
// Columns without a division (h <= 1e-8 or NaN) use h = r = 1, for which the
// same operations are exact.  Returns true if the group's prediction is
// reliable (every r normal; a huge h makes RN(1/h) subnormal).
__device__ __forceinline__ bool load_group_div(const float* hess, int64_t c0, int64_t K, int lane,
                                               GroupDiv* gd) {
  float r = 1.0f, nh = -1.0f;
  bool div = false, slow = false;
  if (lane < 16 && c0 + lane < K) {
    const float h = __ldg(hess + c0 + lane);
    if (h > 1e-8f) {
      r = __frcp_rn(h);
      nh = -h;
      div = h != 1.0f;
      slow = !(h >= 0x1p-60f && h <= 0x1p60f);
    }
  }
  const float r_hi = __shfl_down_sync(0xffffffffu, r, 1);
  const float nh_hi = __shfl_down_sync(0xffffffffu, nh, 1);
  if (lane < 16 && (lane & 1) == 0) {
    gd->R2[lane >> 1] = f2_pack(r, r_hi);
    gd->NH2[lane >> 1] = f2_pack(nh, nh_hi);
  }
  const bool any_div = __any_sync(0xffffffffu, div), any_slow = __any_sync(0xffffffffu, slow);
  if (lane == 0) gd->mode = any_slow ? 2 : (any_div ? 1 : 0);
  return !any_slow;
}

// w*w of a run's 16 fp16 values; `valid` bit i clear -> 0
__device__ __forceinline__ void run_squares(const Row16& v, uint32_t valid, uint64_t (&X2)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t w = row_word(v, k);
    float x0 = f16_square((uint16_t)(w & 0xFFFFu)), x1 = f16_square((uint16_t)(w >> 16));
    if (!((valid >> (2 * k)) & 1u)) x0 = 0.0f;
    if (!((valid >> (2 * k + 1)) & 1u)) x1 = 0.0f;
    X2[k] = f2_pack(x0, x1);
  }
}

// The run's prediction sum(x * r) in fp32 (NaN / inf propagate).
__device__ __forceinline__ float run_pred(const uint64_t (&X2)[8], const uint64_t* R2) {
  uint64_t acc = f2_pack(0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < 8; ++k) acc = f2_fma(X2[k], R2[k], acc);
  float a0, a1;
  f2_unpack(acc, a0, a1);
  return __fadd_rn(a0, a1);
}

__device__ __forceinline__ void run_terms(const uint64_t (&X2)[8], const uint64_t* R2,
                                          const uint64_t* NH2, int mode, uint64_t (&T2)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (mode == 0) {
      T2[k] = X2[k];
    } else if (mode == 1) {
      const uint64_t q0 = f2_mul(X2[k], R2[k]);
      T2[k] = f2_fma(f2_fma(q0, NH2[k], X2[k]), R2[k], q0);
    } else {
      float x0, x1, h0, h1;
      f2_unpack(X2[k], x0, x1);
      f2_unpack(NH2[k], h0, h1);
      T2[k] = f2_pack(__fdiv_rn(x0, -h0), __fdiv_rn(x1, -h1));
    }
  }
}

// Transfer function of a run of terms inside binade e (0 <= t / q < 2^23 for
// every term, which holds whenever the run provably stays inside the binade).
__device__ __forceinline__ void run_tf(const uint64_t (&T2)[8], int e, RunTF& tf) {
  const float iq = pow2f(23 - e);
  const uint64_t iq2 = f2_pack(iq, iq);
  const uint64_t magic2 = f2_pack(8388608.0f, 8388608.0f);
  const uint64_t nq2 = f2_pack(-0.25f, -0.25f);
  uint64_t acc = f2_pack(0.0f, 0.0f);
  uint32_t sgn = 0xFFFFFFFFu;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint64_t a2 = f2_mul(T2[k], iq2);
    const uint64_t k2 = f2_sub(f2_add(a2, magic2), magic2);  // rint, ties to even
    acc = f2_add(acc, k2);
    const uint64_t d2 = f2_sub(a2, k2);
    const uint64_t p2 = f2_fma(d2, d2, nq2);  // >= 0 only for |d| = 0.5
    sgn &= (uint32_t)p2 & (uint32_t)(p2 >> 32);
  }
  float l0, l1;
  f2_unpack(acc, l0, l1);
  tf.kind = kRunProven;
  tf.e = e;
  if (sgn >> 31) {  // no tie: the increment does not depend on the parity
    const int s = (int)__fadd_rn(l0, l1);
    tf.inc0 = tf.inc1 = s;
    tf.pout = (s & 1) ? 1 : 2;
    return;
  }
  // a tie: follow both parities term by term
  int inc[2] = {0, 0}, p[2] = {0, 1};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float t[2];
    f2_unpack(T2[k], t[0], t[1]);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float a = __fmul_rn(t[u], iq);
      const float kk = __fsub_rn(__fadd_rn(a, 8388608.0f), 8388608.0f);
      const float d = __fsub_rn(a, kk);
      if (d == 0.5f || d == -0.5f) {
        const int f = (int)__fsub_rn(a, 0.5f);  // exact floor
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          inc[v] += f + ((p[v] + f) & 1);
          p[v] = 0;
        }
      } else {
        const int ki = (int)kk;
#pragma unroll
        for (int v = 0; v < 2; ++v) {
          inc[v] += ki;
          p[v] ^= ki & 1;
        }
      }
    }
  }
  tf.inc0 = inc[0];
  tf.inc1 = inc[1];
  tf.pout = p[0] | (p[1] << 1);
}

// Classify a run from the predicted prefix before it (p_rs) and after it
// (p_re); `elems` = terms added since the point the prefix is predicted from
// (the drift bound grows with it).  The fp32 sum after n terms lies within
// n * 2^-24 (relative) of the true prefix, and the prediction within
// 24 * 2^-24 of it; (elems + 64) * 2^-24 covers both with margin.
__device__ __forceinline__ void classify_run(const uint64_t (&T2)[8], bool finite, double p_rs,
                                             double p_re, double elems, RunTF& tf) {
  bool zero = true;
#pragma unroll
  for (int k = 0; k < 8; ++k) zero &= (T2[k] & 0x7FFFFFFF7FFFFFFFull) == 0ull;
  if (zero && finite) {
    tf.kind = kRunZero;
    tf.e = 0;
    tf.inc0 = tf.inc1 = 0;
    tf.pout = 2;
    return;
  }
  const double d_s = (elems + 64.0) * kEps24, d_e = (elems + 80.0) * kEps24;
  const double lo = p_rs * (1.0 - d_s), hi = p_re * (1.0 + 2.0 * d_e);
  if (finite && d_e < 0.25 && lo >= 0x1p-100 && hi < 0x1p127 && f64_binade(lo) == f64_binade(hi)) {
    run_tf(T2, f64_binade(lo), tf);
  } else {
    tf.kind = kRunUnproven;
    tf.e = 0;
    tf.inc0 = tf.inc1 = 0;
    tf.pout = 2;
  }
}

// Apply a proven run or stretch (binade e, increments for parity 0 / 1) to
// the exact sum; false (s unchanged) if s is not in binade e or would leave it.
__device__ __forceinline__ bool apply_tf(float& s, int e, int inc0, int inc1) {
  if (!(s > 0.0f) || !(s < 0x1p127f) || f32_binade(s) != e) return false;
  const int m = (int)__fmul_rn(s, pow2f(23 - e));
  const int m2 = m + ((m & 1) ? inc1 : inc0);
  if (m2 >= (1 << 24)) return false;
  s = __fmul_rn((float)m2, pow2f(e - 23));
  return true;
}

__device__ __forceinline__ float serial_add(float s, const uint64_t (&T2)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float t0, t1;
    f2_unpack(T2[k], t0, t1);
    s = __fadd_rn(__fadd_rn(s, t0), t1);
  }
  return s;
}

// Program builder of one chunk (state uniform across the warp; lane 0
// writes the items).
struct ProgBuilder {
  int open;  // 0 none, 1 stretch, 2 window
  int e, inc0, inc1, pout, a, b;
  int count;
  bool overflow;
};

__device__ __forceinline__ void prog_emit(ProgBuilder& pb, int4* items, int lane) {
  if (pb.open == 0) return;
  if (pb.count < kMaxItems) {
    if (lane == 0) {
      const int w = (pb.pout & 3) | (pb.a << 2) | (pb.b << 17);
      items[pb.count] = pb.open == 1 ? make_int4(pb.e, pb.inc0, pb.inc1, w)
                                     : make_int4(kItemWindow, 0, 0, w);
    }
    ++pb.count;
  } else {
    pb.overflow = true;
  }
  pb.open = 0;
}

// Append run j to the program.
__device__ __forceinline__ void prog_add(ProgBuilder& pb, const RunTF& tf, int j, int4* items,
                                         int lane) {
  if (tf.kind == kRunZero) {  // contributes nothing anywhere
    if (pb.open) pb.b = j + 1;
    return;
  }
  if (tf.kind == kRunProven) {
    if (pb.open == 1 && pb.e == tf.e) {
      const int p0 = pb.pout & 1, p1 = (pb.pout >> 1) & 1;
      const int n0 = pb.inc0 + (p0 ? tf.inc1 : tf.inc0);
      const int n1 = pb.inc1 + (p1 ? tf.inc1 : tf.inc0);
      pb.inc0 = n0;
      pb.inc1 = n1;
      pb.pout = ((tf.pout >> p0) & 1) | (((tf.pout >> p1) & 1) << 1);
      pb.b = j + 1;
    } else {
      prog_emit(pb, items, lane);
      pb.open = 1;
      pb.e = tf.e;
      pb.inc0 = tf.inc0;
      pb.inc1 = tf.inc1;
      pb.pout = tf.pout;
      pb.a = j;
      pb.b = j + 1;
    }
    return;
  }
  if (pb.open == 2) {
    pb.b = j + 1;
  } else {
    prog_emit(pb, items, lane);
    pb.open = 2;
    pb.a = j;
    pb.b = j + 1;
  }
}

// Add one step (32 runs, lane = run) to the program.  Fast path: every run is
// zero or proven in the open stretch's binade without ties.
__device__ __forceinline__ void prog_step(ProgBuilder& pb, const RunTF& tf, int run0, int4* items,
                                          int lane) {
  const bool simple = tf.kind == kRunZero || (tf.kind == kRunProven && tf.inc0 == tf.inc1 &&
                                              ((tf.pout & 3) == ((tf.inc0 & 1) ? 1 : 2)));
  const unsigned prov = __ballot_sync(0xffffffffu, tf.kind == kRunProven);
  const int e0 = __shfl_sync(0xffffffffu, tf.e, prov ? __ffs(prov) - 1 : 0);
  const bool fast = __all_sync(0xffffffffu, simple && (tf.kind == kRunZero || tf.e == e0)) &&
                    (prov == 0u || pb.open == 0 || (pb.open == 1 && pb.e == e0));
  if (fast) {
    if (prov == 0u) {
      if (pb.open) pb.b = run0 + 32;
      return;
    }
    const int s =
        (int)__reduce_add_sync(0xffffffffu, (unsigned)(tf.kind == kRunProven ? tf.inc0 : 0));
    if (pb.open == 0) {  // the stretch starts at the step's first proven run
      pb.open = 1;
      pb.e = e0;
      pb.inc0 = pb.inc1 = 0;
      pb.pout = 2;
      pb.a = run0 + __ffs(prov) - 1;
    }
    pb.inc0 += s;
    pb.inc1 += s;
    if (s & 1) pb.pout ^= 3;
    pb.b = run0 + 32;
    return;
  }
  for (int j = 0; j < 32; ++j) {
    RunTF t;
    t.kind = __shfl_sync(0xffffffffu, tf.kind, j);
    t.e = __shfl_sync(0xffffffffu, tf.e, j);
    t.inc0 = __shfl_sync(0xffffffffu, tf.inc0, j);
    t.inc1 = __shfl_sync(0xffffffffu, tf.inc1, j);
    t.pout = __shfl_sync(0xffffffffu, tf.pout, j);
    prog_add(pb, t, run0 + j, items, lane);
  }
}

struct QArgs {
  const __half* W;
  int64_t M, K;
  int ng, nct, nrc;
  const float* hess;
  Workspace ws;
  uint8_t* gp;
  ChunkLayout cl;
  int n4;      // 4-bit groups to select
  int select;  // the selection runs (sensitivity needed)
  int w_aligned;
  // encode / post outputs
  int32_t* packed2;
  int32_t* packed4;
  __half* scales1;
  int8_t* zeros1;
  __half* scales2;
  int8_t* zeros2;
  uint8_t* sq;
  int32_t* row_ptrs;
  int32_t* nnz;
  int enc_nbx;  // encode grid: slot blocks (x) per row block
  int enc_nby;  // row blocks
};

// Replay runs [a, b) of group g's chunk rc exactly, starting from s.  Runs go
// 32 at a time (lane = run): each batch is classified again from the exact s
// (the drift bound restarts at 0, so only runs that really contain a binade
// crossing stay unproven), proven runs are applied as transfer functions and
// the others term by term.  The next batch's rows load while one is processed.
__device__ __noinline__ void replay_runs(const QArgs& A, const GroupDiv& gd, int g, int rc, int a,
                                         int b, float& s, int lane) {
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, A.K - c0);
  const bool vec = A.w_aligned && gs == kGroup1 && (A.K & 7) == 0;
  const uint32_t cmask = gs >= 16 ? 0xFFFFu : ((1u << gs) - 1u);
  auto fetch = [&](int j0, Row16& v) -> bool {
    const int j = j0 + lane;
    const int64_t r = (int64_t)rc * kChunkRows + j;
    const bool ok = j < b && r < A.M;
    if (ok) v = load_row16(A.W, r, A.K, c0, gs, vec);
    return ok;
  };
  Row16 nv;
  bool nvalid = fetch(a, nv);
  for (int j0 = a; j0 < b; j0 += 32) {
    const Row16 v = nv;
    const bool valid = nvalid;
    if (j0 + 32 < b) nvalid = fetch(j0 + 32, nv);
    uint64_t T2[8];
    bool finite = true;
    double sum = 0.0;
    if (valid) {
      uint64_t X2[8];
      run_squares(v, cmask, X2);
      run_terms(X2, gd.R2, gd.NH2, gd.mode, T2);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float t0, t1;
        f2_unpack(T2[k], t0, t1);
        finite &= isfinite(t0) && isfinite(t1);
        sum += (double)t0 + (double)t1;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) T2[k] = 0ull;
    }
    double incl = sum;  // prefix from the exact s at the start of this batch
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const double p_rs = (double)s + (incl - sum), p_re = (double)s + incl;
    RunTF tf;
    classify_run(T2, finite, p_rs, p_re, 16.0 * lane, tf);
    // fast path: all runs zero, or proven in s's binade without ties
    const bool simple = tf.kind == kRunZero || (tf.kind == kRunProven && tf.inc0 == tf.inc1 &&
                                                s > 0.0f && s < 0x1p127f &&
                                                tf.e == f32_binade(s));
    if (__all_sync(0xffffffffu, simple)) {
      const int tot =
          (int)__reduce_add_sync(0xffffffffu, (unsigned)(tf.kind == kRunProven ? tf.inc0 : 0));
      if (tot == 0) continue;
      float s2 = s;
      if (apply_tf(s2, f32_binade(s), tot, tot)) {
        s = s2;
        continue;
      }
    }
    for (int u = 0; u < 32; ++u) {
      const int kind = __shfl_sync(0xffffffffu, tf.kind, u);
      if (kind == kRunZero) continue;
      const int e = __shfl_sync(0xffffffffu, tf.e, u);
      const int i0 = __shfl_sync(0xffffffffu, tf.inc0, u);
      const int i1 = __shfl_sync(0xffffffffu, tf.inc1, u);
      if (kind == kRunProven && apply_tf(s, e, i0, i1)) continue;
      uint64_t U2[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) U2[k] = __shfl_sync(0xffffffffu, T2[k], u);
      s = serial_add(s, U2);
    }
  }
}

// Replay every run from (chunk c0, run r0) up to (chunk c1, run r1), exclusive.
__device__ void replay_span(const QArgs& A, const GroupDiv& gd, int g, int c0, int r0, int c1,
                            int r1, float& s, int lane) {
  for (int c = c0; c <= c1 && c < A.nrc; ++c) {
    const int a = c == c0 ? r0 : 0, b = c == c1 ? r1 : kChunkRows;
    if (a < b) replay_runs(A, gd, g, c, a, b, s, lane);
  }
}

// The exact sensitivity of group g from its chunk programs.  Consecutive
// stretches in one binade compose without the sum (composition is
// associative); the composite is applied to the exact sum when the binade
// changes or a window comes, and replayed if the check in apply_tf fails.
__device__ __noinline__ float assemble_group(const QArgs& A, const GroupDiv& gd, int g,
                                             int lane) {
  float S = 0.0f;
  int p_open = 0, p_e = 0, p_i0 = 0, p_i1 = 0, p_po = 2, p_c = 0, p_r = 0;
  auto flush = [&](int c_end, int r_end) {
    if (!p_open) return;
    p_open = 0;
    if (!apply_tf(S, p_e, p_i0, p_i1)) replay_span(A, gd, g, p_c, p_r, c_end, r_end, S, lane);
  };
  const int nrc = A.nrc;
  for (int cb = 0; cb < nrc && isfinite(S); cb += 32) {
    const size_t rec = (size_t)g * nrc + cb + lane;
    const bool have = cb + lane < nrc;
    const uint32_t cw = have ? __ldcg(A.ws.icount + rec) : 0u;
    int4 it[kMaxItems];
#pragma unroll
    for (int k = 0; k < kMaxItems; ++k)
      it[k] = (have && k < (int)(cw & 0xFFFFu)) ? __ldcg(A.ws.items + rec * kMaxItems + k)
                                                 : make_int4(0, 0, 0, 0);
    const int nc = min(32, nrc - cb);
    for (int c = 0; c < nc && isfinite(S); ++c) {
      const int chunk = cb + c;
      const uint32_t w = __shfl_sync(0xffffffffu, cw, c);
      if (w & kCntOverflow) {
        flush(chunk, 0);
        replay_runs(A, gd, g, chunk, 0, kChunkRows, S, lane);
        continue;
      }
      const int n = (int)(w & 0xFFFFu);
#pragma unroll
      for (int k = 0; k < kMaxItems; ++k) {
        if (k < n) {
          const int ix = __shfl_sync(0xffffffffu, it[k].x, c);
          const int iy = __shfl_sync(0xffffffffu, it[k].y, c);
          const int iz = __shfl_sync(0xffffffffu, it[k].z, c);
          const int iw = __shfl_sync(0xffffffffu, it[k].w, c);
          const int ra = (iw >> 2) & 0x7FFF, rb = (iw >> 17) & 0x7FFF;
          if (ix == kItemWindow) {
            flush(chunk, ra);
            replay_runs(A, gd, g, chunk, ra, rb, S, lane);
          } else if (p_open && p_e == ix) {
            const int q0 = p_po & 1, q1 = (p_po >> 1) & 1;
            p_i0 += q0 ? iz : iy;
            p_i1 += q1 ? iz : iy;
            p_po = ((iw >> q0) & 1) | (((iw >> q1) & 1) << 1);
          } else {
            flush(chunk, ra);
            p_open = 1;
            p_e = ix;
            p_i0 = iy;
            p_i1 = iz;
            p_po = iw & 3;
            p_c = chunk;
            p_r = ra;
          }
        }
      }
    }
  }
  flush(nrc, 0);
  return S;
}

// Program of chunk rc of pending group g (one warp; rows from global memory).
__device__ __noinline__ void exact_chunk(const QArgs& A, const GroupDiv& gd, int g, int rc,
                                         int lane) {
  const int64_t c0 = (int64_t)g * kGroup1;
  const int gs = (int)min64(kGroup1, A.K - c0);
  const bool vec = A.w_aligned && gs == kGroup1 && (A.K & 7) == 0;
  const uint32_t cmask = gs >= 16 ? 0xFFFFu : ((1u << gs) - 1u);
  const size_t rec = (size_t)g * A.nrc + rc;
  // predicted prefix before the chunk
  double pstart = 0.0;
  for (int j = lane; j < rc; j += 32) pstart += __ldcg(A.ws.cpred + (size_t)g * A.nrc + j);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pstart += __shfl_xor_sync(0xffffffffu, pstart, o);
  const int64_t row0 = (int64_t)rc * kChunkRows;
  int4* items = A.ws.items + rec * kMaxItems;
  ProgBuilder pb;
  pb.open = 0;
  pb.count = 0;
  pb.overflow = false;
  pb.e = pb.inc0 = pb.inc1 = pb.a = pb.b = 0;
  pb.pout = 2;
  double ctot = 0.0;
  for (int s = 0; s < kSteps; ++s) {
    const int r = s * 32 + lane;
    const bool rvalid = row0 + r < A.M;
    Row16 v;
    v.lo = v.hi = make_uint4(0, 0, 0, 0);
    if (rvalid) v = load_row16(A.W, row0 + r, A.K, c0, gs, vec);
    uint64_t X2[8], T2[8];
    run_squares(v, rvalid ? cmask : 0u, X2);
    float p = run_pred(X2, gd.R2);
    if (!isfinite(p)) p = 0.0f;
    run_terms(X2, gd.R2, gd.NH2, gd.mode, T2);
    bool fin = true;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float x0, x1;
      f2_unpack(T2[k], x0, x1);
      fin &= isfinite(x0) && isfinite(x1);
    }
    double incl = (double)p;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    double excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = 0.0;
    const double p_rs = pstart + ctot + excl;
    ctot += __shfl_sync(0xffffffffu, incl, 31);
    RunTF tf;
    classify_run(T2, fin, p_rs, p_rs + (double)p, 16.0 * (double)(row0 + r), tf);
    prog_step(pb, tf, s * 32, items, lane);
  }
  prog_emit(pb, items, lane);
  if (lane == 0)
    A.ws.icount[rec] = (uint32_t)min(pb.count, kMaxItems) | (pb.overflow ? kCntOverflow : 0u);
}

// ---------------------------------------------------------------------------
// Selection helpers.
// ---------------------------------------------------------------------------
template <int NT>
__device__ __forceinline__ void sync_nt() {
  if (NT == 32)
    __syncwarp();
  else
    __syncthreads();
}

// k-th largest (1-based, 1 <= k <= n) of n 32-bit keys key(i), by 4 passes
// of 8 bits; returns the key and, in *need_eq, how many keys equal to it the
// k largest include.  All NT threads call it with the same arguments.
template <int NT, typename KeyF>
__device__ uint32_t kth_largest(int n, int k, KeyF key, uint32_t* hist, uint32_t* s2,
                                uint32_t* need_eq) {
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  if (tid == 0) {
    s2[0] = 0;
    s2[1] = (uint32_t)k;
  }
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += NT) hist[i] = 0;
    sync_nt<NT>();
    const uint32_t prefix = s2[0];
    for (int i = tid; i < n; i += NT) {
      const uint32_t kk = key(i);
      if ((kk & mask) == prefix) atomicAdd(&hist[(kk >> shift) & 255u], 1u);
    }
    sync_nt<NT>();
    if (warp == 0) {
      // suffix sums over bins, highest bin first; lane l owns bins 8l..8l+7
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = hist[lane * 8 + j];
        tot += c[j];
      }
      uint32_t suf = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_down_sync(0xffffffffu, suf, o);
        if (lane + o < 32) suf += y;
      }
      const uint32_t need = s2[1];
      const uint32_t above = suf - tot;
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
        s2[0] = prefix | ((uint32_t)(lane * 8 + b) << shift);
        s2[1] = need - acc;
      }
    }
    mask |= 0xFFu << shift;
    sync_nt<NT>();
  }
  *need_eq = s2[1];
  const uint32_t T = s2[0];
  sync_nt<NT>();
  return T;
}

// Sortable key of a non-negative float or NaN (NaN above +inf, as the bit
// patterns of the reference's comparisons would order them).
__device__ __forceinline__ uint32_t sens_key(float s) {
  return isnan(s) ? 0xFFFFFFFFu : __float_as_uint(s);
}

// 2nd-order tables, group order and any_irregular once every group's
// precision is in ws.prec (quantize.cu:245-272 over the flattened [M, ng]
// scales; scales_1st[r, g] depends only on g, so full chunks repeat with
// period ng / gcd(ng, 256)).  Also writes the group_precision output.
// With rebuild_order false (the selection completed after encode started)
// `order` and the decided / pending counts stay as they are.
template <int NT>
__device__ void finalize_tables(const QArgs& a, float* s1, size_t s1_bytes, uint32_t* s_wsum,
                                int* s_irr, bool rebuild_order) {
  const int ng = a.ng;
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  constexpr int NWARP = NT / 32;
  if (tid == 0) *s_irr = 0;
  sync_nt<NT>();
  const bool s1_in_smem = (size_t)ng * sizeof(float) <= s1_bytes;
  int irr = 0;
  for (int g = tid; g < ng; g += NT) {
    const uint8_t pr = a.ws.prec[g];
    a.gp[g] = pr;
    const GroupParams& p = a.ws.params[2 * g + pr];
    if (s1_in_smem) s1[g] = __half2float(__ushort_as_half((uint16_t)p.scale_h));
    irr |= !(p.flags & kFlagRegular);
  }
  if (irr) atomicOr(s_irr, 1);
  sync_nt<NT>();
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
  if (rebuild_order) {
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
    sync_nt<NT>();
    if (lane == 31) s_wsum[warp] = incl;
    sync_nt<NT>();
    uint32_t off = 0, total2 = 0;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      if (w < warp) off += s_wsum[w];
      total2 += s_wsum[w];
    }
    uint32_t pos2 = off + incl - n2;
    uint32_t pos4 = total2 + (uint32_t)i0 - pos2;
    for (int i = i0; i < i1; ++i) {
      if (a.ws.prec[i] == 0)
        a.ws.order[pos2++] = i;
      else
        a.ws.order[pos4++] = i;
    }
    if (tid == 0) a.ws.hdr->n2 = total2;
  }
  sync_nt<NT>();
  if (tid == 0) {
    a.ws.hdr->any_irregular = *s_irr;
    if (rebuild_order) {
      a.ws.hdr->n_dec = (uint32_t)ng;
      a.ws.hdr->n_pend = 0;
    }
  }
}

// Interval of group g's fp32 serial sum as sortable keys (lo rounded down,
// hi rounded up).  NaN / inf groups are exact.
__device__ __forceinline__ void sens_interval(const QArgs& a, int g, uint32_t& klo,
                                              uint32_t& khi) {
  const uint32_t f = __ldcg(a.ws.gflag + g);
  if (f & kGrpNaN) {
    klo = khi = 0xFFFFFFFFu;
    return;
  }
  if (f & kGrpInf) {
    klo = khi = 0x7F800000u;
    return;
  }
  const double n = 16.0 * (double)a.M;
  const double dcr = n * kEps24;
  if ((f & kGrpLoose) || dcr >= 0.5) {
    klo = 0u;
    khi = 0x7F800000u;
    return;
  }
  const double P = __ldcg(a.ws.gpred + g), mom = __ldcg(a.ws.gmom + g);
  const double eps = 24.0 * kEps24;
  const double D = dcr / (1.0 - dcr);
  const double E = kEps24 * (1.0 + eps) * (1.0 + D) * mom * (1.0 + 1e-6) + n * 0x1p-148;
  const double lo = fmax(P * (1.0 - eps) - E, 0.0), hi = P * (1.0 + eps) + E;
  klo = __float_as_uint(__double2float_rd(lo));
  khi = __float_as_uint(__double2float_ru(hi));  // +inf past FLT_MAX
}

// The selection from the intervals (the last stats CTA; NT threads).  Group g
// is certainly 4-bit if its lower bound exceeds the (n4+1)-th largest upper
// bound (at most n4 groups, g included, can reach its sum), certainly 2-bit
// if its upper bound is below the n4-th largest lower bound (n4 groups surely
// exceed it).  The rest are pending; if all or none of them must be 4-bit
// the selection is complete, otherwise their exact sums decide.
template <int NT>
__device__ void select_from_intervals(const QArgs& a, uint8_t* scratch, size_t scratch_bytes) {
  const int ng = a.ng, n4 = a.n4;
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  constexpr int NWARP = NT / 32;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s2[2];
  __shared__ uint32_t s_wsum[NWARP];
  __shared__ uint32_t s_cnt[2];
  __shared__ int s_irr;
  uint32_t* klo = reinterpret_cast<uint32_t*>(scratch);
  uint32_t* khi = klo + ng;
  const bool keys_in_smem = (size_t)ng * 8 <= scratch_bytes;
  auto lo_of = [&](int g) -> uint32_t {
    if (keys_in_smem) return klo[g];
    uint32_t l, h;
    sens_interval(a, g, l, h);
    return l;
  };
  auto hi_of = [&](int g) -> uint32_t {
    if (keys_in_smem) return khi[g];
    uint32_t l, h;
    sens_interval(a, g, l, h);
    return h;
  };
  int pending = 0;
  if (a.select && n4 > 0) {
    if (keys_in_smem)
      for (int g = tid; g < ng; g += NT) sens_interval(a, g, klo[g], khi[g]);
    if (tid == 0) s_cnt[0] = s_cnt[1] = 0;
    sync_nt<NT>();
    uint32_t eq;
    const uint32_t Alo = kth_largest<NT>(ng, n4, lo_of, hist, s2, &eq);
    const bool all_in = n4 >= ng;
    const uint32_t Bhi = all_in ? 0u : kth_largest<NT>(ng, n4 + 1, hi_of, hist, s2, &eq);
    uint32_t c_in = 0, c_pend = 0;
    for (int g = tid; g < ng; g += NT) {
      const uint32_t l = lo_of(g), h = hi_of(g);
      uint8_t p;
      if (all_in || l > Bhi)
        p = 1;
      else if (h < Alo)
        p = 0;
      else
        p = 2;
      c_in += p == 1;
      c_pend += p == 2;
      a.ws.prec[g] = p;
    }
    c_in = __reduce_add_sync(0xffffffffu, c_in);
    c_pend = __reduce_add_sync(0xffffffffu, c_pend);
    if (lane == 0) {
      atomicAdd(&s_cnt[0], c_in);
      atomicAdd(&s_cnt[1], c_pend);
    }
    sync_nt<NT>();
    const int need = n4 - (int)s_cnt[0], np = (int)s_cnt[1];
    if (np > 0 && (need <= 0 || need >= np)) {
      // all pending groups take the same precision
      for (int g = tid; g < ng; g += NT)
        if (a.ws.prec[g] == 2) a.ws.prec[g] = need > 0 ? 1 : 0;
    } else if (np > 0) {
      pending = 1;
      if (tid == 0) a.ws.hdr->need = (uint32_t)need;
    }
  } else {
    for (int g = tid; g < ng; g += NT) a.ws.prec[g] = 0;
  }
  sync_nt<NT>();
  if (!pending) {
    finalize_tables<NT>(a, reinterpret_cast<float*>(scratch), scratch_bytes, s_wsum, &s_irr,
                        true);
    return;
  }
  // pending: order = decided 2-bit, decided 4-bit, pending (each ascending)
  const int per = (ng + NT - 1) / NT;
  const int i0 = min(ng, tid * per), i1 = min(ng, i0 + per);
  uint32_t c[3] = {0, 0, 0};
  for (int i = i0; i < i1; ++i) ++c[a.ws.prec[i]];
  uint32_t pos[3], tot[3];
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    uint32_t incl = c[t];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    sync_nt<NT>();
    if (lane == 31) s_wsum[warp] = incl;
    sync_nt<NT>();
    uint32_t off = 0, all = 0;
    for (int w = 0; w < NWARP; ++w) {
      if (w < warp) off += s_wsum[w];
      all += s_wsum[w];
    }
    pos[t] = off + incl - c[t];
    tot[t] = all;
  }
  pos[1] += tot[0];
  pos[2] += tot[0] + tot[1];
  for (int i = i0; i < i1; ++i) {
    const uint8_t p = a.ws.prec[i];
    a.ws.order[pos[p]++] = i;
    if (p == 2) a.ws.gticket[i] = 0;
  }
  if (tid == 0) {
    a.ws.hdr->n2 = tot[0];
    a.ws.hdr->n_dec = tot[0] + tot[1];
    a.ws.hdr->n_pend = tot[2];
    a.ws.hdr->ticket_exact = 0;
  }
}

// ---------------------------------------------------------------------------
// stats kernel: one CTA per 128 x 128 tile (row chunks of a column tile are
// consecutive blocks), one warp per group.
// ---------------------------------------------------------------------------
template <bool kSens>
__global__ void __launch_bounds__(kStatsThreads)
    stats_kernel(const __grid_constant__ CUtensorMap tmap, const QArgs A, int use_tma) {
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* buf = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) &
                                            ~(uintptr_t)1023);
  __shared__ uint64_t full_bar;
  __shared__ GroupDiv s_div[kTileGroups];
  __shared__ int s_flag;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t M = A.M, K = A.K;
  const int nct = A.nct, nrc = A.nrc;
  const int rc = (int)(blockIdx.x % (unsigned)nrc), ct = (int)(blockIdx.x / (unsigned)nrc);
  const int64_t row0 = (int64_t)rc * kChunkRows;

  if (use_tma) {
    if (tid == 0) {
      mbar_init(&full_bar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(&full_bar, kTileBytes);
      tma_load_2d(buf, &tmap, &full_bar, ct * kTileCols, (int)row0);
      tma_load_2d(buf + kBoxBytes, &tmap, &full_bar, ct * kTileCols + 64, (int)row0);
    }
  } else {
    // the same swizzled layout from plain loads; NaN outside the matrix
    for (int e = tid; e < kChunkRows * kTileCols; e += kStatsThreads) {
      const int r = e / kTileCols, c = e % kTileCols;
      const int64_t gr = row0 + r, gc = (int64_t)ct * kTileCols + c;
      const uint16_t v =
          (gr < M && gc < K) ? __half_as_ushort(A.W[gr * K + gc]) : (uint16_t)0x7E00;
      const int half = c >> 6, cc = c & 63;
      *reinterpret_cast<uint16_t*>(buf + half * kBoxBytes + r * 128 +
                                   (((cc >> 3) ^ (r & 7)) << 4) + (cc & 7) * 2) = v;
    }
  }
  const int gi = warp;
  const int64_t g = (int64_t)ct * kTileGroups + gi;
  const int64_t c0 = g * kGroup1;
  bool loose = false;
  if (kSens && g < A.ng) loose = !load_group_div(A.hess, c0, K, lane, &s_div[gi]);
  bool ok = true;
  if (use_tma && tid == 0) ok = mbar_wait(&full_bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(&A.ws.hdr->status, kStatusTimeout);
      (void)mbar_wait(&full_bar, 0);  // bounded: the loads must land before exit
    }
  }
  __syncthreads();

  if (g < A.ng) {
    const int gs = (int)min64(kGroup1, K - c0);
    const uint32_t cmask = gs >= 16 ? 0xFFFFu : ((1u << gs) - 1u);
    const bool edge = (row0 + kChunkRows > M) || gs < kGroup1;
    const size_t rec = (size_t)g * nrc + rc;
    __half2 hmn = __float2half2_rn(INFINITY), hmx = __float2half2_rn(-INFINITY);
    const __half2 hnan = __float2half2_rn(NAN);
    double csum = 0.0;
    bool any_nan = false, any_inf = false;
#pragma unroll
    for (int s = 0; s < kSteps; ++s) {
      const int r = s * 32 + lane;
      const bool rvalid = row0 + r < M;
      const Row16 v = tile_run(buf, gi, r);
      const uint32_t vmask = rvalid ? cmask : 0u;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        __half2 w2 = as_h2(row_word(v, k));
        if (edge) {
          const bool v0 = (vmask >> (2 * k)) & 1u, v1 = (vmask >> (2 * k + 1)) & 1u;
          w2 = __halves2half2(v0 ? __low2half(w2) : __low2half(hnan),
                              v1 ? __high2half(w2) : __high2half(hnan));
        }
        hmn = __hmin2(hmn, w2);
        hmx = __hmax2(hmx, w2);
      }
      if (kSens) {
        uint64_t X2[8];
        run_squares(v, vmask, X2);
        const float p = run_pred(X2, s_div[gi].R2);
        any_nan |= isnan(p);
        any_inf |= isinf(p);
        csum += isfinite(p) ? (double)p : 0.0;
      }
    }
    float mn = fminf(__half2float(__low2half(hmn)), __half2float(__high2half(hmn)));
    float mx = fmaxf(__half2float(__low2half(hmx)), __half2float(__high2half(hmx)));
    mn = warp_min(mn);
    mx = warp_max(mx);
    if (kSens) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) csum += __shfl_xor_sync(0xffffffffu, csum, o);
      const uint32_t fl = (__any_sync(0xffffffffu, any_nan) ? kGrpNaN : 0u) |
                          (__any_sync(0xffffffffu, any_inf) ? kGrpInf : 0u) |
                          (loose ? kGrpLoose : 0u);
      if (lane == 0) {
        A.ws.cpred[rec] = csum;
        A.ws.cflag[rec] = fl;
      }
    }
    if (lane == 0) A.ws.cminmax[rec] = make_float2(mn, mx);
  }
  // zero this tile's share of the per-row outlier counts
  if (ct == 0)
    for (int r = tid; r < kChunkRows; r += kStatsThreads)
      if (row0 + r < M) A.ws.row_counts[row0 + r] = 0;

  // ---- last tile of the column tile: its groups' totals and parameters ----
  __threadfence();
  __syncthreads();
  if (tid == 0) s_flag = atomicAdd(&A.ws.ct_count[ct], 1u) == (unsigned)nrc - 1u;
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  if (g < A.ng) {
    float mn = INFINITY, mx = -INFINITY;
    uint32_t flags = 0;
    double carry = 0.0, mom = 0.0;
    for (int j0 = 0; j0 < nrc; j0 += 32) {
      const int j = j0 + lane;
      const size_t rec = (size_t)g * nrc + j;
      double v = 0.0;
      if (j < nrc) {
        const float2 m = __ldcg(A.ws.cminmax + rec);
        mn = fminf(mn, m.x);
        mx = fmaxf(mx, m.y);
        if (kSens) {
          v = __ldcg(A.ws.cpred + rec);
          flags |= __ldcg(A.ws.cflag + rec);
        }
      }
      if (kSens) {
        double incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const double y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const double terms = 16.0 * (double)min64(kChunkRows, M - (int64_t)j * kChunkRows);
        if (j < nrc) mom += terms * (carry + incl);
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    mn = warp_min(mn);
    mx = warp_max(mx);
    // the reference starts from +-1e10f and ignores NaN: clamp the exact min / max
    mn = fminf(1e10f, mn);
    mx = fmaxf(-1e10f, mx);
    if (kSens) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mom += __shfl_xor_sync(0xffffffffu, mom, o);
      flags = __reduce_or_sync(0xffffffffu, flags);
    }
    if (lane == 0) {
      A.ws.gmin[g] = mn;
      A.ws.gmax[g] = mx;
      if (kSens) {
        A.ws.gpred[g] = carry;
        A.ws.gmom[g] = mom;
        A.ws.gflag[g] = flags;
      }
    }
    group_params_warp(A.ws.params, g, mn, mx, lane);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_flag = atomicAdd(&A.ws.hdr->ticket_ct, 1u) == (unsigned)nct - 1u;
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  select_from_intervals<kStatsThreads>(A, buf, kTileBytes);
}

// ---------------------------------------------------------------------------
// encode: rows of one group slot, 2 rows per step.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool is_outlier(float x, float scale, int zero, float thr, int q,
                                           int fma_mode) {
  const float qz = (float)(q - zero);
  const float err = fma_mode ? fabsf(__fmaf_rn(-scale, qz, x))
                             : fabsf(__fsub_rn(x, __fmul_rn(scale, qz)));
  return err > thr;
}

__device__ void encode_rows(const QArgs& a, int g, int64_t r0, int64_t r1) {
  const int64_t K = a.K;
  const int ng = a.ng;
  const bool four = a.ws.prec[g] != 0;
  const GroupParams& pp = a.ws.params[2 * g + (four ? 1 : 0)];
  const float gmin = pp.gmin, scale = pp.scale, thr = pp.thr;
  const int zero = pp.zero, levels = pp.levels;
  const bool regular = (pp.flags & kFlagRegular) != 0;
  const __half sh = __ushort_as_half((uint16_t)pp.scale_h);
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
  const uint32_t keep4b = gs >= 16 ? 0xFFFFFFFFu : (gs <= 8 ? 0u : ((1u << (4 * (gs - 8))) - 1u));
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
            cnt += is_outlier(x, scale, zero, thr, q, kOutlierFma);
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
      reinterpret_cast<int2*>(a.packed4)[si] = four ? make_int2((int)wa, (int)wb) : make_int2(0, 0);
      a.scales1[si] = sh;
      a.zeros1[si] = (int8_t)zero;
      if (cnt) atomicAdd(a.ws.row_counts + r, cnt);
    }
  }
}

// Exact sums of the pending groups (the first kExactCtas blocks of the encode
// grid): warps take (pending group, chunk) work items; the last chunk of a
// group assembles its exact sum, the last group completes the selection.
__device__ __noinline__ void exact_ctas(const QArgs& a) {
  const Header* hdr = a.ws.hdr;
  const uint32_t np = *reinterpret_cast<const volatile uint32_t*>(&hdr->n_pend);
  if (np == 0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t ndec = *reinterpret_cast<const volatile uint32_t*>(&hdr->n_dec);
  __shared__ GroupDiv s_div[8];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s2[2];
  __shared__ uint32_t s_wsum[1];
  __shared__ int s_irr;
  const int64_t nwork = (int64_t)np * a.nrc;
  for (int64_t w = (int64_t)blockIdx.x * 8 + warp; w < nwork; w += (int64_t)kExactCtas * 8) {
    const int u = (int)(w / a.nrc), c = (int)(w % a.nrc);
    const int g = a.ws.order[ndec + u];
    load_group_div(a.hess, (int64_t)g * kGroup1, a.K, lane, &s_div[warp]);
    __syncwarp();
    exact_chunk(a, s_div[warp], g, c, lane);
    __threadfence();
    uint32_t last = 0;
    if (lane == 0) last = atomicAdd(&a.ws.gticket[g], 1u) == (unsigned)a.nrc - 1u;
    if (!__shfl_sync(0xffffffffu, last, 0)) continue;
    __threadfence();
    // the group's chunk programs are complete: its exact sum
    float S;
    uint32_t fl = 0;
    for (int j = lane; j < a.nrc; j += 32) fl |= __ldcg(a.ws.cflag + (size_t)g * a.nrc + j);
    fl = __reduce_or_sync(0xffffffffu, fl);
    if (fl & kGrpNaN)
      S = __int_as_float(0x7fc00000);
    else if (fl & kGrpInf)
      S = INFINITY;
    else
      S = assemble_group(a, s_div[warp], g, lane);
    if (lane == 0) a.ws.sens[g] = S;
    __threadfence();
    if (lane == 0) last = atomicAdd(&a.ws.hdr->ticket_exact, 1u) == np - 1u;
    if (!__shfl_sync(0xffffffffu, last, 0)) continue;
    __threadfence();
    // every pending sum is known: the top `need` of them are 4-bit (equal
    // sums by lowest group index; equal sums straddling the boundary set the
    // tie flag, as the reference's std::sort leaves their order open)
    const int need = (int)*reinterpret_cast<const volatile uint32_t*>(&hdr->need);
    const int32_t* pend = a.ws.order + ndec;
    auto key = [&](int i) -> uint32_t { return sens_key(__ldcg(a.ws.sens + pend[i])); };
    uint32_t need_eq;
    const uint32_t T = kth_largest<32>((int)np, need, key, hist, s2, &need_eq);
    uint32_t rank = 0, total_eq = 0;
    for (int i0 = 0; i0 < (int)np; i0 += 32) {
      const int i = i0 + lane;
      const uint32_t k = i < (int)np ? key(i) : 0u;
      const bool eq = i < (int)np && k == T;
      const unsigned b = __ballot_sync(0xffffffffu, eq);
      const uint32_t my_rank = rank + __popc(b & ((1u << lane) - 1u));
      if (i < (int)np) a.ws.prec[pend[i]] = (k > T || (eq && my_rank < need_eq)) ? 1 : 0;
      rank += __popc(b);
      total_eq += __popc(b);
    }
    if (lane == 0 && total_eq > need_eq) atomicOr(&a.ws.hdr->status, kStatusTie);
    __syncwarp();
    // decided slots of `order` are being encoded meanwhile: keep it as is
    finalize_tables<32>(a, nullptr, 0, s_wsum, &s_irr, false);
  }
}

// encode grid: the first kExactCtas blocks compute exact sums of pending
// groups (and exit at once when none are pending); the rest encode decided
// group slots, one thread per (slot, block of kEncRows rows).
__global__ void __launch_bounds__(256) encode_kernel(const QArgs a) {
  grid_dependency_wait();  // stats (and its selection) complete
  if (blockIdx.x < (unsigned)kExactCtas) {
    exact_ctas(a);
    return;
  }
  const int b = (int)blockIdx.x - kExactCtas;
  const int bx = b % a.enc_nbx, by = b / a.enc_nbx;
  const uint32_t ndec = a.ws.hdr->n_dec;
  const int slot = bx * 256 + threadIdx.x;
  if (slot >= (int)ndec) return;
  const int g = a.ws.order[slot];
  const int64_t r0 = (int64_t)by * kEncRows;
  encode_rows(a, g, r0, min64(a.M, r0 + kEncRows));
}

// ---------------------------------------------------------------------------
// post: 2nd-order scales / zeros / codes (quantize.cu:245-281 over the
// flattened [M, ng] scales), the pending groups' codes, and the outlier row
// pointers (torch_ops.cu:210-229).
// ---------------------------------------------------------------------------
constexpr int kPostRows = 16;

__global__ void __launch_bounds__(256) post_kernel(const QArgs a) {
  grid_dependency_wait();  // encode (and the exact selection) complete
  const Header* hdr = a.ws.hdr;
  const int64_t M = a.M;
  const int ng = a.ng;
  const int tid = threadIdx.x;
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + tid;
  const int64_t gthreads = (int64_t)gridDim.x * blockDim.x;
  const ChunkLayout& cl = a.cl;
  for (int64_t c = gtid; c < cl.ng2; c += gthreads) {
    const float4 e = a.ws.chunk_tab[c < cl.nfull ? (int)(c % cl.period) : cl.ntab_full];
    a.scales2[c] = __ushort_as_half((uint16_t)__float_as_int(e.z));
    a.zeros2[c] = (int8_t)__float_as_int(e.w);
  }
  // 2nd-order codes (quantize.cu:274-280): block b covers rows
  // [b * kPostRows, ...), thread t groups t, t + 256, ...  Flat index r*ng + g
  // lies in full chunk (jt >> 8) of one period (period * 256 = lcm(ng, 256)
  // flat indices), advanced by ng per row.
  const int P256 = cl.period * kGroup2;
  const int64_t full_end = cl.nfull * kGroup2;
  for (int64_t rb = blockIdx.x; rb * kPostRows < M; rb += gridDim.x) {
    const int64_t r0 = rb * kPostRows, r1 = min64(M, r0 + kPostRows);
    for (int g = tid; g < ng; g += blockDim.x) {
      const float s1f = __half2float(
          __ushort_as_half((uint16_t)a.ws.params[2 * g + a.ws.prec[g]].scale_h));
      int jt = (int)((r0 * ng + g) % P256);
      for (int64_t r = r0; r < r1; ++r) {
        const int64_t si = r * ng + g;
        const float4 ch = a.ws.chunk_tab[si < full_end ? (jt >> 8) : cl.ntab_full];
        const int q2 = f2i_rz(roundf(__fdiv_rn(__fsub_rn(s1f, ch.x), ch.y)));
        a.sq[si] = (uint8_t)max(0, min(15, q2));
        jt += ng;
        if (jt >= P256) jt -= P256;
      }
    }
  }
  // the pending groups, now decided
  const uint32_t np = hdr->n_pend, ndec = hdr->n_dec;
  const int64_t nrb = ceil_div(M, kEncRows);
  for (int64_t w = gtid; w < (int64_t)np * nrb; w += gthreads) {
    const int u = (int)(w / nrb);
    const int64_t r0 = (w % nrb) * kEncRows;
    encode_rows(a, a.ws.order[ndec + u], r0, min64(M, r0 + kEncRows));
  }
  const bool any_irr = hdr->any_irregular != 0;
  if (!any_irr) {
    for (int64_t r = gtid; r <= M; r += gthreads) a.row_ptrs[r] = 0;
    if (gtid == 0) *a.nnz = 0;
    return;
  }
  // the last CTA turns per-row counts into row pointers
  __shared__ int s_last;
  __shared__ long long part[256];
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&a.ws.hdr->ticket_post, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int nt = blockDim.x;
  const int64_t per = ceil_div(M, (int64_t)nt);
  const int64_t q0 = min64(M, tid * per), q1 = min64(M, q0 + per);
  long long s = 0;
  for (int64_t r = q0; r < q1; ++r) s += __ldcg(a.ws.row_counts + r);
  part[tid] = s;
  __syncthreads();
  for (int o = 1; o < nt; o <<= 1) {
    const long long y = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += y;
    __syncthreads();
  }
  long long run = part[tid] - s;
  if (tid == 0) a.row_ptrs[0] = 0;
  for (int64_t r = q0; r < q1; ++r) {
    run += __ldcg(a.ws.row_counts + r);
    a.row_ptrs[r + 1] = (int32_t)run;
  }
  if (tid == nt - 1) *a.nnz = (int32_t)part[tid];
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

mb_status check_common(const void* weights, int64_t M, int64_t K) {
  MB_REQUIRE(weights != nullptr, "weights must not be null");
  MB_REQUIRE(M > 0 && K > 0, "weights must be a non-empty 2D [M, K] matrix");
  MB_REQUIRE(M * ceil_div(K, kGroup1) < (int64_t)INT32_MAX && M * K < (int64_t)INT32_MAX,
             "weights too large: M*K must be below 2^31 (int32 outlier indexing)");
  return MB_OK;
}

template <typename Kern, typename... Args>
mb_status launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, args...));
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
  const int64_t nct = ceil_div(K, kTileCols), nrc = ceil_div(M, kChunkRows);
  MB_REQUIRE(nct * nrc < (int64_t)INT32_MAX, "too many tiles");
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

  MB_CUDA_TRY(cudaMemsetAsync(ws.hdr, 0, sizeof(Header) + sizeof(uint32_t) * nct, stream));

  QArgs qa;
  qa.W = static_cast<const __half*>(weights_fp16);
  qa.M = M;
  qa.K = K;
  qa.ng = (int)ng;
  qa.nct = (int)nct;
  qa.nrc = (int)nrc;
  qa.hess = hessian_diag;
  qa.ws = ws;
  qa.gp = group_precision;
  qa.cl = chunk_layout(M, ng);
  qa.n4 = (int)n4;
  qa.select = sens;
  qa.w_aligned = w_aligned;
  qa.packed2 = packed_2bit;
  qa.packed4 = packed_4bit;
  qa.scales1 = static_cast<__half*>(scales_1st_fp16);
  qa.zeros1 = zeros_1st;
  qa.scales2 = static_cast<__half*>(scales_2nd_fp16);
  qa.zeros2 = zeros_2nd;
  qa.sq = scales_1st_quant;
  qa.row_ptrs = outlier_row_ptrs;
  qa.nnz = nnz_device;
  qa.enc_nbx = (int)ceil_div(ng, 256);
  qa.enc_nby = (int)ceil_div(M, kEncRows);
  MB_REQUIRE((int64_t)qa.enc_nbx * qa.enc_nby + kExactCtas < (int64_t)INT32_MAX,
             "too many rows for the encode grid");

  // TMA needs a 16-byte aligned base and a row pitch that is a multiple of 16
  // bytes; other inputs fill the same shared-memory layout with plain loads.
  CUtensorMap tmap;
  std::memset(&tmap, 0, sizeof(tmap));
  const bool tma = w_aligned && (K % 8 == 0) &&
                   make_tensor_map_2d_16bit_sw128(&tmap, weights_fp16, false, (uint64_t)M,
                                                  (uint64_t)K, kChunkRows, 64);
  {
    auto kern = sens ? stats_kernel<true> : stats_kernel<false>;
    static std::atomic<uint64_t> attr_done[2] = {{0}, {0}};
    MB_CUDA_TRY(set_smem_limit_once(kern, kStatsSmem, attr_done[sens ? 1 : 0]));
    kern<<<(unsigned)(nct * nrc), kStatsThreads, kStatsSmem, stream>>>(tmap, qa, tma ? 1 : 0);
    MB_LAUNCH_CHECK("stats_kernel");
  }
  if (mb_status st = launch_pdl(encode_kernel, dim3((unsigned)(kExactCtas + qa.enc_nbx * qa.enc_nby)),
                                dim3(256), 0, stream, qa))
    return st;
  int dev = 0, sms = 148;
  MB_CUDA_TRY(cudaGetDevice(&dev));
  MB_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t post_grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(M, kPostRows), 8LL * sms));
  return launch_pdl(post_kernel, dim3((unsigned)post_grid), dim3(256), 0, stream, qa);
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
