// memboost quantize on sm_100a.
//
// Replaces the reference's six-kernel pipeline with host round trips
// (core/torch_ops.cu:105-264 driving core/quantize.cu:72-321) by three
// stream-ordered kernels chained with programmatic dependent launch and no
// host synchronisation:
//
//   stats    streams W from HBM in 128 x 128 tiles through TMA, each CTA a
//            contiguous column-major range of tiles, one warp per 16-column
//            group (quantize.cu:72-128): per-column sums of w*w per 128-row
//            chunk, and per segment (a CTA's chunks of one column tile)
//            min / max and an fp64 prediction of the group's serial fp32
//            sensitivity sum.  The CTA completing a column tile combines its
//            segments: min / max, scale / zero / code thresholds for both
//            precisions (quantize.cu:153-176) and a rigorous interval around
//            each sensitivity.  The CTA completing the last column tile
//            selects the 4-bit groups (torch_ops.cu:149-179): every group
//            whose interval lies clear of the top-k boundary is decided, the
//            few that straddle it are left pending.
//   exact    the 2nd-order chunk table (quantize.cu:245-272) when nothing
//            is pending; otherwise the pending groups' exact serial sums
//            (transfer functions per chunk of rows, assembled in order), the
//            last of which completes the selection and the table.
//   encode   reads W again and writes both packed arrays,
//            scales_1st, zeros_1st and the 2nd-order codes
//            (quantize.cu:132-242, 274-280), counts outliers per row, and
//            writes the 2nd-order scales / zeros and the outlier row
//            pointers (quantize.cu:245-272, 284-299, torch_ops.cu:210-229).
//   extract  (second entry point) CSR values / columns in ascending column
//            order (quantize.cu:301-321).
//
// Arithmetic that decides an output bit uses the reference's fp32 operations,
// written with explicit rounding intrinsics so the compiler cannot contract
// or reorder them.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <vector>

#include "mb_common.cuh"
#include "mb_tma.cuh"

namespace mb {
namespace {

constexpr int kFlagRegular = 1;  // threshold path valid; group cannot hold outliers
constexpr uint32_t kStatusTie = 1u;
constexpr uint32_t kStatusTimeout = 2u;
// a 2nd-order zero point round(-min / scale_2nd) fell outside [-128, 127] and
// wrapped in its int8 cast (the reference's format, quantize.cu:267-272)
constexpr uint32_t kStatusZero2Wrap = 4u;
// more outliers than the caller's CSR capacity (mb_quantize_csr): the CSR
// values / columns were not written
constexpr uint32_t kStatusCsrOverflow = 8u;

// stats tiles: 128 columns (8 groups) x 128 rows
constexpr int kTileCols = 128;
constexpr int kTileGroups = kTileCols / kGroup1;  // 8: one warp per group
constexpr int kChunkRows = 128;                   // rows per tile = runs per chunk
constexpr int kStatsThreads = 32 * kTileGroups;   // 256
constexpr int kSteps = kChunkRows / 32;
constexpr int kBoxBytes = kChunkRows * 128;       // one 64-column TMA box (16 KB)
constexpr int kTileBytes = 2 * kBoxBytes;         // 32 KB
constexpr int kStages = 3;     // stats tile ring per CTA (two CTAs per SM)
constexpr int kEncStages = 2;  // encode tile ring (its staging buffers take the rest)
constexpr int kStatsSmem = kStages * kTileBytes + 1024;   // + alignment slack
constexpr int kCombSmem = 96 * 1024;  // the selection's key / cost scratch
constexpr int kEncSmem = kEncStages * kTileBytes + 1024;
// encode CTA size: 8 warps, two CTAs per SM.  The items are taken from a
// shared counter, so any warp count works; 10 or 12 warps (96 / 80
// registers a thread) measured 3% / 13% slower on the 7B MLP pair.
constexpr int kEncThreads = 256;
static_assert(kEncThreads % 32 == 0 && kEncThreads >= 256, "encode needs >= 8 warps");
// full-tile write-out: threads [0, 256) store the packed words; the per-row
// arrays go to threads [256, kEncThreads) (or [0, 128) with 256 threads)
constexpr int kRowWriter0 = kEncThreads > 256 ? 256 : 0;
constexpr int kRowWriters = kEncThreads > 256 ? kEncThreads - 256 : kChunkRows;

// exact sums of pending groups
constexpr int kMaxItems = 8;             // program items per (group, chunk)
constexpr int kItemWindow = 0x40000000;  // item.x of a window
constexpr uint32_t kCntOverflow = 1u << 18;  // icount: the chunk's program overflowed
constexpr uint32_t kGrpNaN = 1u, kGrpInf = 2u, kGrpLoose = 4u;  // per-group prediction flags
constexpr double kEps24 = 5.9604644775390625e-08;  // 2^-24
constexpr int kExactCtas = 148;                    // CTAs of the exact-sum kernel
constexpr int kMaxEncGrid = 4096;                  // encode CTAs (persistent grid) at most
constexpr int kMaxStatsGrid = 1024;                // stats CTAs (persistent grid) at most

// The stats grid never exceeds the tile count or kMaxStatsGrid (the segment
// records are sized by it).
__host__ __device__ __forceinline__ int64_t stats_grid_cap(int64_t ntiles) {
  return ntiles < kMaxStatsGrid ? ntiles : kMaxStatsGrid;
}

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
  uint32_t tile_stats;     // next stats tile
  uint32_t tile_encode;    // next encode tile
  uint32_t n_straddle;     // groups whose sensitivity interval straddled the boundary
  uint32_t pad[4];
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

// One stats CTA's share of one group: its consecutive row chunks of the
// group's column tile (a segment).  sum: prediction of the segment's rows;
// mom: sum over its chunks of terms * prediction through the chunk (from the
// segment's first chunk); rows: rows covered; flags: kGrp* bits.
struct __align__(16) SegRec {
  double sum, mom;
  float mn, mx;
  uint32_t rows, flags;
};
static_assert(sizeof(SegRec) == 32, "SegRec must stay 32 bytes");

struct Workspace {
  Header* hdr;
  uint32_t* ct_count;   // [nct] stats tiles finished per column tile (zeroed with hdr)
  float* ccol;          // [ng * nrc * 16] per-column sums of w*w over the chunk
  SegRec* seg;          // [(stats CTAs + nct) * 8]: segment id (CTA + column tile), group
  double* gpred;        // [ng] predicted sensitivity
  double* gmom;         // [ng] sum over chunks of terms * inclusive prediction
  uint32_t* gflag;      // [ng] kGrp* bits
  uint2* gkey;          // [ng] sortable lower / upper bound of the sensitivity
  uint32_t* gticket;    // [ng] exact-sum chunk programs finished (pending groups)
  int4* items;          // [ng * nrc * kMaxItems] chunk programs (pending groups)
  uint32_t* icount;     // [ng * nrc] item count | NaN / inf / overflow bits
  float* gmin;
  float* gmax;
  uint32_t* gscale;     // [ng] fp16 scale_1st of the 2-bit (low) and 4-bit (high) params
  uint8_t* greg;        // [ng] bit 0 / 1: the 2-bit / 4-bit params are regular
  float* sens;          // [ng] exact sums (pending groups)
  GroupParams* params;  // [2 * ng]: 2g = 2-bit, 2g + 1 = 4-bit
  float4* chunk_tab;    // [ntab_full + 1]: (min, fp32 scale2, fp16 bits of scale2, zero2)
  uint8_t* sq_pat;      // [ntab_full * 256]: 2nd-order codes of the distinct full chunks
  int32_t* row_counts;  // [M]
  uint8_t* prec;        // [ng] selected precision (copy of group_precision)
  int32_t* order;       // [ng] decided 2-bit, decided 4-bit, then pending groups
  int32_t* enc_start;   // [kMaxEncGrid + 1] first tile of each encode CTA
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
  char* p_cc = take(sizeof(float) * 16 * nrec);
  char* p_sg = take(sizeof(SegRec) * kTileGroups * (size_t)(stats_grid_cap(nct * nrc) + nct));
  char* p_gp = take(sizeof(double) * ng);
  char* p_gm = take(sizeof(double) * ng);
  char* p_gf = take(sizeof(uint32_t) * ng);
  char* p_gk = take(sizeof(uint2) * ng);
  char* p_gt = take(sizeof(uint32_t) * ng);
  char* p_it = take(sizeof(int4) * kMaxItems * nrec);
  char* p_ic = take(sizeof(uint32_t) * nrec);
  char* p_gmin = take(sizeof(float) * ng);
  char* p_gmax = take(sizeof(float) * ng);
  char* p_gsc = take(sizeof(uint32_t) * ng);
  char* p_grg = take(ng);
  char* p_sens = take(sizeof(float) * ng);
  char* p_par = take(sizeof(GroupParams) * 2 * ng);
  char* p_ch = take(sizeof(float4) * (cl.ntab_full + 1));
  char* p_sq = take((size_t)kGroup2 * std::max(1, cl.ntab_full));
  char* p_rc = take(sizeof(int32_t) * M);
  char* p_pr = take(ng);
  char* p_or = take(sizeof(int32_t) * ng);
  char* p_es = take(sizeof(int32_t) * (kMaxEncGrid + 1));
  if (ws) {
    ws->hdr = reinterpret_cast<Header*>(p_hdr);
    ws->ct_count = reinterpret_cast<uint32_t*>(p_hdr + sizeof(Header));
    ws->ccol = reinterpret_cast<float*>(p_cc);
    ws->seg = reinterpret_cast<SegRec*>(p_sg);
    ws->gpred = reinterpret_cast<double*>(p_gp);
    ws->gmom = reinterpret_cast<double*>(p_gm);
    ws->gflag = reinterpret_cast<uint32_t*>(p_gf);
    ws->gkey = reinterpret_cast<uint2*>(p_gk);
    ws->gticket = reinterpret_cast<uint32_t*>(p_gt);
    ws->items = reinterpret_cast<int4*>(p_it);
    ws->icount = reinterpret_cast<uint32_t*>(p_ic);
    ws->gmin = reinterpret_cast<float*>(p_gmin);
    ws->gmax = reinterpret_cast<float*>(p_gmax);
    ws->gscale = reinterpret_cast<uint32_t*>(p_gsc);
    ws->greg = reinterpret_cast<uint8_t*>(p_grg);
    ws->sens = reinterpret_cast<float*>(p_sens);
    ws->params = reinterpret_cast<GroupParams*>(p_par);
    ws->chunk_tab = reinterpret_cast<float4*>(p_ch);
    ws->sq_pat = reinterpret_cast<uint8_t*>(p_sq);
    ws->row_counts = reinterpret_cast<int32_t*>(p_rc);
    ws->prec = reinterpret_cast<uint8_t*>(p_pr);
    ws->order = reinterpret_cast<int32_t*>(p_or);
    ws->enc_start = reinterpret_cast<int32_t*>(p_es);
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


__device__ __forceinline__ __half2 as_h2(uint32_t w) { return *reinterpret_cast<__half2*>(&w); }

// One 16-byte half (8 columns: h = 0 low, 1 high) of tile group gi's row r
// (0..127) from a tile in shared memory: two 64-column TMA boxes written with
// the 128-byte swizzle (16-byte chunk c of row r sits at chunk c ^ (r & 7)),
// so 8 consecutive rows of one half hit distinct banks.
__device__ __forceinline__ uint4 tile_half(const uint8_t* buf, int gi, int r, int h) {
  const uint8_t* base = buf + (gi >> 2) * kBoxBytes + r * 128;
  return *reinterpret_cast<const uint4*>(base + (((2 * (gi & 3) + h) ^ (r & 7)) << 4));
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

// Parameters of group g for both precisions (one warp; lanes 0 and 1 write
// them): scale, zero point, outlier threshold, regular flag, and the compact
// copies of the two fp16 scales and regular flags.  The code thresholds are
// left to group_thresholds_warp (later, grid-parallel): finding them is the
// costly part and only encode needs them.
__device__ void group_params_warp(GroupParams* params, uint32_t* gscale, uint8_t* greg, int64_t g,
                                  float mn, float mx, int lane) {
  GroupParams q2, q4;
  group_scalars(mn, mx, 4, q2);
  group_scalars(mn, mx, 16, q4);
  if (lane == 0) {
    gscale[g] = (uint32_t)q2.scale_h | ((uint32_t)q4.scale_h << 16);
    greg[g] = (uint8_t)((q2.flags & kFlagRegular) | ((q4.flags & kFlagRegular) << 1));
  }
  if (lane < 2) {
    const GroupParams& p = lane ? q4 : q2;
    GroupParams* d = params + 2 * g + lane;
    d->gmin = p.gmin;
    d->gmax = p.gmax;
    d->scale = p.scale;
    d->thr = p.thr;
    d->zero = p.zero;
    d->levels = p.levels;
    d->flags = p.flags;
    d->scale_h = p.scale_h;
  }
}

// Code thresholds of group g for both precisions (one warp): lanes 0-2 find
// the 2-bit thresholds, lanes 3-17 the 4-bit ones, from the parameters
// group_params_warp wrote; unused slots and irregular groups get +inf.
__device__ void group_thresholds_warp(GroupParams* params, int64_t g, int lane) {
  GroupParams* p2 = params + 2 * g;
  GroupParams* p4 = p2 + 1;
  if (lane < 18) {
    const bool four = lane >= 3;
    const int L = four ? 16 : 4;
    const int level = four ? lane - 2 : lane + 1;
    const GroupParams* d = four ? p4 : p2;
    const float gmin = __ldcg(&d->gmin), scale = __ldcg(&d->scale);
    const int flags = __ldcg(&d->flags);
    const uint16_t T =
        (flags & kFlagRegular) ? find_threshold(gmin, scale, L, level) : (uint16_t)0x7C00;
    (four ? p4 : p2)->thresh[level - 1] = T;
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

// Prediction of one row chunk of a group from its 16 column sums of w*w and
// the columns' RN(1/h) (1 where nothing is divided): fp64, the products are
// exact; non-finite column sums are left out (the group's flags hold them).
__device__ __forceinline__ double chunk_pred(const float4 (&cc)[4], const float (&rc16)[16]) {
  double part[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float cv[4] = {cc[q].x, cc[q].y, cc[q].z, cc[q].w};
    double t = 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) t = fma((double)cv[e], (double)rc16[4 * q + e], t);
    part[q] = t;
  }
  double v = (part[0] + part[1]) + (part[2] + part[3]);
  if (!isfinite(v)) {
    v = 0.0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float cv[4] = {cc[q].x, cc[q].y, cc[q].z, cc[q].w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (isfinite(cv[e])) v += (double)cv[e] * (double)rc16[4 * q + e];
    }
  }
  return v;
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
  int no_select;       // the combine stops after the per-group totals (row-split slabs)
  int exact_thresholds;  // the exact kernel finds the code thresholds (row-split encode)
  int stats_grid;      // CTAs of the stats kernel (the segment records' layout)
  int comb_smem;       // dynamic shared memory of the combine kernel (selection scratch)
  int enc_grid;        // CTAs of the encode kernel
  int all_pending;     // every group takes its exact serial sum (mb_quantize_exact_sums)
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
};

// Several matrices in one launch: the CTAs [cta0[m], cta0[m + 1]) of a
// kernel serve matrix m exactly as a grid of their own would (CTA index b of
// G); the matrices share nothing.  One matrix is a batch of one.
constexpr int kMaxBatch = 8;
template <int NB>
struct BatchMap {
  int n;
  int cta0[NB + 1];
};
struct CtaSlot {
  int m, b, G;
};
template <int NB>
__device__ __forceinline__ CtaSlot batch_slot(const BatchMap<NB>& bm) {
  const int x = (int)blockIdx.x;
  int m = 0;
#pragma unroll
  for (int i = 1; i < NB; ++i) m += (i < bm.n && x >= bm.cta0[i]) ? 1 : 0;
  return CtaSlot{m, x - bm.cta0[m], bm.cta0[m + 1] - bm.cta0[m]};
}

// combine / exact arguments of a batch
template <int NB>
struct ArgsBatch {
  QArgs a[NB];
  BatchMap<NB> bm;
};

// Transfer function g applied after f: (i0, i1, po) becomes the composite.
// Increments saturate at 2^30 (any sum that large has left its binade).
__device__ __forceinline__ void tf_then(int& i0, int& i1, int& po, int gi0, int gi1, int gpo) {
  const int p0 = po & 1, p1 = (po >> 1) & 1;
  const int n0 = min(i0 + (p0 ? gi1 : gi0), 1 << 30);
  const int n1 = min(i1 + (p1 ? gi1 : gi0), 1 << 30);
  po = ((gpo >> p0) & 1) | (((gpo >> p1) & 1) << 1);
  i0 = n0;
  i1 = n1;
}

// Replay runs [a, b) of group g's chunk rc exactly, starting from s.  Runs go
// 32 at a time (lane = run).  From the exact s in binade e every lane takes
// its run's transfer function in e; an inclusive scan composes them, so
// lane j holds the sum after runs 0..j as if all stayed in e.  The first run
// whose prefix leaves the binade (or holds a term >= 2^e) is added term by
// term from the exact sum before it, and the scan resumes behind it in the
// new binade: one scan per binade crossing instead of one step per run.
// Sums below 2^-103 (where the binade's quantum is subnormal) go term by
// term.  The next batch's rows load while one is processed.
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
    float tmax = 0.0f;
    bool finite = true;
    if (valid) {
      uint64_t X2[8];
      run_squares(v, cmask, X2);
      run_terms(X2, gd.R2, gd.NH2, gd.mode, T2);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float t0, t1;
        f2_unpack(T2[k], t0, t1);
        finite &= isfinite(t0) && isfinite(t1);
        tmax = fmaxf(tmax, fmaxf(t0, t1));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) T2[k] = 0ull;
    }
    const int nrun = min(32, b - j0);
    int cur = 0;  // runs [0, cur) of the batch are in s
    while (cur < nrun) {
      if (!(s >= 0x1p-103f && s < 0x1p127f)) {
        // zero, tiny or huge sum: run cur term by term
        float t = s;
        if (lane == cur) t = serial_add(s, T2);
        s = __shfl_sync(0xffffffffu, t, cur);
        ++cur;
        continue;
      }
      const int e = f32_binade(s);
      int i0 = 0, i1 = 0, po = 2;  // identity
      bool bad = false;
      if (lane >= cur && lane < nrun) {
        if (finite && tmax < pow2f(e)) {
          RunTF tf;
          run_tf(T2, e, tf);
          i0 = tf.inc0;
          i1 = tf.inc1;
          po = tf.pout;
        } else {
          bad = true;
        }
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int u0 = __shfl_up_sync(0xffffffffu, i0, o);
        int u1 = __shfl_up_sync(0xffffffffu, i1, o);
        int up = __shfl_up_sync(0xffffffffu, po, o);
        if (lane >= o) {
          tf_then(u0, u1, up, i0, i1, po);  // the earlier lanes' runs first
          i0 = u0;
          i1 = u1;
          po = up;
        }
      }
      const int m = (int)__fmul_rn(s, pow2f(23 - e));  // s / q, in [2^23, 2^24)
      const int m2 = min(m + ((m & 1) ? i1 : i0), 1 << 30);
      const unsigned cross =
          __ballot_sync(0xffffffffu, lane >= cur && lane < nrun && (bad || m2 >= (1 << 24)));
      const int u = cross ? __ffs(cross) - 1 : nrun;  // first run that leaves binade e
      if (u > cur) {
        // runs [cur, u) stay in e: the sum after them, exactly
        s = __shfl_sync(0xffffffffu, __fmul_rn((float)m2, pow2f(e - 23)), u - 1);
      }
      if (u < nrun) {
        float t = s;
        if (lane == u) t = serial_add(s, T2);
        s = __shfl_sync(0xffffffffu, t, u);
        cur = u + 1;
      } else {
        cur = nrun;
      }
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

__device__ __forceinline__ unsigned lanes_upto(int x) { return (2u << x) - 1u; }  // 0..x

// The exact sensitivity of group g from its chunk programs.  Consecutive
// stretches in one binade compose without the sum (composition is
// associative); the composite is applied to the exact sum when the binade
// changes or a window comes, and replayed if the check in apply_tf fails.
// Chunks come 32 at a time (lane = chunk); runs of chunks whose program is a
// single stretch in one binade are composed at once by a segmented scan over
// the lanes, so the serial walk visits only those runs, the other chunks'
// items and the replays.
__device__ __noinline__ float assemble_group(const QArgs& A, const GroupDiv& gd, int g,
                                             int lane) {
  float S = 0.0f;
  int p_open = 0, p_e = 0, p_i0 = 0, p_i1 = 0, p_po = 2, p_c = 0, p_r = 0;
  auto flush = [&](int c_end, int r_end) {
    if (!p_open) return;
    p_open = 0;
    if (!apply_tf(S, p_e, p_i0, p_i1)) replay_span(A, gd, g, p_c, p_r, c_end, r_end, S, lane);
  };
  // one item: a window [ra, rb) of chunk (replayed), or a stretch in binade e
  // with transfer function (i0, i1, po) from run ra of chunk
  auto item = [&](int chunk, int e, int i0, int i1, int po, int ra, int rb) {
    if (e == kItemWindow) {
      flush(chunk, ra);
      replay_runs(A, gd, g, chunk, ra, rb, S, lane);
    } else if (p_open && p_e == e) {
      tf_then(p_i0, p_i1, p_po, i0, i1, po);
    } else {
      flush(chunk, ra);
      p_open = 1;
      p_e = e;
      p_i0 = i0;
      p_i1 = i1;
      p_po = po;
      p_c = chunk;
      p_r = ra;
    }
  };
  const int nrc = A.nrc;
  for (int cb = 0; cb < nrc && isfinite(S); cb += 32) {
    const size_t rec = (size_t)g * nrc + cb + lane;
    const bool have = cb + lane < nrc;
    // every slot at once (slots past the count are not used)
    uint32_t cw = 0u;
    int4 it[kMaxItems];
#pragma unroll
    for (int k = 0; k < kMaxItems; ++k)
      it[k] = have ? __ldcg(A.ws.items + rec * kMaxItems + k) : make_int4(0, 0, 0, 0);
    if (have) cw = __ldcg(A.ws.icount + rec);
    const bool simple =
        have && !(cw & kCntOverflow) && (cw & 0xFFFFu) == 1u && it[0].x != kItemWindow;
    const unsigned smask = __ballot_sync(0xffffffffu, simple);
    const int e_prev = __shfl_up_sync(0xffffffffu, it[0].x, 1);
    const bool start =
        simple && (lane == 0 || !((smask >> (lane - 1)) & 1u) || e_prev != it[0].x);
    const unsigned stmask = __ballot_sync(0xffffffffu, start);
    // segmented inclusive scan: lane holds the composite from its run's
    // first chunk through itself
    int s0 = it[0].y, s1 = it[0].z, sp = it[0].w & 3;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u0 = __shfl_up_sync(0xffffffffu, s0, o);
      int u1 = __shfl_up_sync(0xffffffffu, s1, o);
      int up = __shfl_up_sync(0xffffffffu, sp, o);
      const bool join =
          simple && lane >= o && (stmask & lanes_upto(lane) & ~lanes_upto(lane - o)) == 0u;
      if (join) {
        tf_then(u0, u1, up, s0, s1, sp);
        s0 = u0;
        s1 = u1;
        sp = up;
      }
    }
    const int nc = min(32, nrc - cb);
    int c = 0;
    while (c < nc && isfinite(S)) {
      const int chunk = cb + c;
      if ((smask >> c) & 1u) {
        const unsigned brk = (stmask | ~smask) & ~lanes_upto(c);
        const int end = min(nc, brk ? __ffs(brk) - 1 : 32);
        const int e = __shfl_sync(0xffffffffu, it[0].x, c);
        const int ra = (__shfl_sync(0xffffffffu, it[0].w, c) >> 2) & 0x7FFF;
        const int i0 = __shfl_sync(0xffffffffu, s0, end - 1);
        const int i1 = __shfl_sync(0xffffffffu, s1, end - 1);
        const int po = __shfl_sync(0xffffffffu, sp, end - 1);
        item(chunk, e, i0, i1, po, ra, 0);
        c = end;
        continue;
      }
      const uint32_t w = __shfl_sync(0xffffffffu, cw, c);
      if (w & kCntOverflow) {
        flush(chunk, 0);
        replay_runs(A, gd, g, chunk, 0, kChunkRows, S, lane);
      } else {
        const int n = (int)(w & 0xFFFFu);
        for (int k = 0; k < n; ++k) {
          int4 v = it[0];
#pragma unroll
          for (int q = 1; q < kMaxItems; ++q)
            if (q == k) v = it[q];
          const int ix = __shfl_sync(0xffffffffu, v.x, c);
          const int iy = __shfl_sync(0xffffffffu, v.y, c);
          const int iz = __shfl_sync(0xffffffffu, v.z, c);
          const int iw = __shfl_sync(0xffffffffu, v.w, c);
          item(chunk, ix, iy, iz, iw & 3, (iw >> 2) & 0x7FFF, (iw >> 17) & 0x7FFF);
        }
      }
      ++c;
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
  const int64_t row0 = (int64_t)rc * kChunkRows;
  // the chunk's rows (lane = run of each 32-run step), loaded up front so
  // the four loads overlap one another and the prefix computation
  Row16 rv[kSteps];
#pragma unroll
  for (int s = 0; s < kSteps; ++s) {
    rv[s].lo = rv[s].hi = make_uint4(0, 0, 0, 0);
    if (row0 + s * 32 + lane < A.M) rv[s] = load_row16(A.W, row0 + s * 32 + lane, A.K, c0, gs, vec);
  }
  // predicted prefix before the chunk, from the column sums of the chunks
  float rc16[16];
#pragma unroll
  for (int k = 0; k < 8; ++k) f2_unpack(gd.R2[k], rc16[2 * k], rc16[2 * k + 1]);
  double pstart = 0.0;
  for (int j = lane; j < rc; j += 32) {
    const float4* src = reinterpret_cast<const float4*>(A.ws.ccol + ((size_t)g * A.nrc + j) * 16);
    float4 cc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) cc[q] = __ldcg(src + q);
    pstart += chunk_pred(cc, rc16);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pstart += __shfl_xor_sync(0xffffffffu, pstart, o);
  int4* items = A.ws.items + rec * kMaxItems;
  ProgBuilder pb;
  pb.open = 0;
  pb.count = 0;
  pb.overflow = false;
  pb.e = pb.inc0 = pb.inc1 = pb.a = pb.b = 0;
  pb.pout = 2;
  double ctot = 0.0;
#pragma unroll
  for (int s = 0; s < kSteps; ++s) {
    const int r = s * 32 + lane;
    const bool rvalid = row0 + r < A.M;
    uint64_t X2[8], T2[8];
    run_squares(rv[s], rvalid ? cmask : 0u, X2);
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

// One radix step (one warp): among the 256 bins (highest first) find the
// bin holding the s2[1]-th largest key; extend the prefix s2[0] with it and
// leave in s2[1] how many keys of that bin are still needed.
__device__ __forceinline__ void radix_pick(const uint32_t* hist, uint32_t* s2, uint32_t prefix,
                                           int shift, int lane) {
  uint32_t c[8], tot = 0;  // lane l owns bins 8l .. 8l+7
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    c[j] = hist[lane * 8 + j];
    tot += c[j];
  }
  uint32_t suf = tot;  // keys in lanes >= lane
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

// hist[bin] += 1 for the lanes with `on`, one shared-memory atomic per
// distinct bin of the warp (keys cluster in few bins in the early passes).
__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin, bool on) {
  const unsigned act = __ballot_sync(0xffffffffu, on);
  if (!act) return;
  const unsigned same = __match_any_sync(0xffffffffu, on ? bin : 0xFFFFFFFFu);
  const int lane = threadIdx.x & 31;
  if (on && (__ffs(same) - 1) == lane) atomicAdd(&hist[bin], (uint32_t)__popc(same));
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
    for (int i0 = 0; i0 < n; i0 += NT) {  // whole warps (match_any)
      const int i = i0 + tid;
      const uint32_t kk = i < n ? key(i) : 0u;
      hist_add(hist, (kk >> shift) & 255u, i < n && (kk & mask) == prefix);
    }
    sync_nt<NT>();
    if (warp == 0) radix_pick(hist, s2, prefix, shift, lane);
    mask |= 0xFFu << shift;
    sync_nt<NT>();
  }
  *need_eq = s2[1];
  const uint32_t T = s2[0];
  sync_nt<NT>();
  return T;
}

// Two order statistics at once over the same indices: the ka-th largest of
// keys a(i) and the kb-th largest of keys b(i) (the passes share the syncs).
template <int NT, typename KeyA, typename KeyB>
__device__ void kth_largest2(int n, int ka, KeyA a, int kb, KeyB b, uint32_t* hist /*512*/,
                             uint32_t* s4, uint32_t& Ta, uint32_t& Tb) {
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  if (tid == 0) {
    s4[0] = 0;
    s4[1] = (uint32_t)ka;
    s4[2] = 0;
    s4[3] = (uint32_t)kb;
  }
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 512; i += NT) hist[i] = 0;
    sync_nt<NT>();
    const uint32_t pa = s4[0], pb = s4[2];
    for (int i0 = 0; i0 < n; i0 += NT) {  // whole warps (match_any)
      const int i = i0 + tid;
      const uint32_t x = i < n ? a(i) : 0u, y = i < n ? b(i) : 0u;
      hist_add(hist, (x >> shift) & 255u, i < n && (x & mask) == pa);
      hist_add(hist, 256 + ((y >> shift) & 255u), i < n && (y & mask) == pb);
    }
    sync_nt<NT>();
    if (warp == 0) radix_pick(hist, s4, pa, shift, lane);
    if (warp == (NT > 32 ? 1 : 0)) radix_pick(hist + 256, s4 + 2, pb, shift, lane);
    mask |= 0xFFu << shift;
    sync_nt<NT>();
  }
  Ta = s4[0];
  Tb = s4[2];
  sync_nt<NT>();
}

// hist[bin] += 1 for the lanes with `on`: the first active lane's bin takes
// one shared-memory atomic for all lanes sharing it (in the early passes
// nearly every key falls in one bin), the other lanes add one each.
__device__ __forceinline__ void hist_add_lead(uint32_t* hist, uint32_t bin, bool on, int lane) {
  const unsigned act = __ballot_sync(0xffffffffu, on);
  if (act == 0u) return;
  const int leader = __ffs(act) - 1;
  const uint32_t lb = __shfl_sync(0xffffffffu, bin, leader);
  const unsigned same = __ballot_sync(0xffffffffu, on && bin == lb);
  if (lane == leader) atomicAdd(&hist[lb], (uint32_t)__popc(same));
  if (on && bin != lb) atomicAdd(&hist[bin], 1u);
}

// kth_largest2 over keys held in registers: thread tid holds keys
// tid + i NT (i < KPT) of both sets; n <= KPT NT.  The histograms are double
// buffered (hist: 1024 words), so a pass takes two block barriers: count
// (and zero the next pass's histograms), then pick.  s4 keeps the results.
template <int NT, int KPT>
__device__ void kth_largest2_reg(const uint32_t (&x)[KPT], const uint32_t (&y)[KPT], int n,
                                 int ka, int kb, uint32_t* hist, uint32_t* s4, uint32_t& Ta,
                                 uint32_t& Tb) {
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  for (int i = tid; i < 512; i += NT) hist[i] = 0;
  if (tid == 0) {
    s4[0] = 0;
    s4[1] = (uint32_t)ka;
    s4[2] = 0;
    s4[3] = (uint32_t)kb;
  }
  sync_nt<NT>();
  uint32_t mask = 0;
  int cur = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    uint32_t* h = hist + cur * 512;
    uint32_t* hn = hist + (cur ^ 1) * 512;
    const uint32_t pa = s4[0], pb = s4[2];
#pragma unroll
    for (int i = 0; i < KPT; ++i) {
      if (i * NT < n) {  // uniform: whole warps take part
        const bool v = tid + i * NT < n;
        hist_add_lead(h, (x[i] >> shift) & 255u, v && (x[i] & mask) == pa, lane);
        hist_add_lead(h + 256, (y[i] >> shift) & 255u, v && (y[i] & mask) == pb, lane);
      }
    }
    // the previous pass's histograms were last read before its final barrier
    for (int i = tid; i < 512; i += NT) hn[i] = 0;
    sync_nt<NT>();
    if (warp == 0) radix_pick(h, s4, pa, shift, lane);
    if (warp == (NT > 32 ? 1 : 0)) radix_pick(h + 256, s4 + 2, pb, shift, lane);
    mask |= 0xFFu << shift;
    cur ^= 1;
    sync_nt<NT>();
  }
  Ta = s4[0];
  Tb = s4[2];
}

// Sortable key of a non-negative float or NaN (NaN above +inf, as the bit
// patterns of the reference's comparisons would order them).
__device__ __forceinline__ uint32_t sens_key(float s) {
  return isnan(s) ? 0xFFFFFFFFu : __float_as_uint(s);
}

// Tile ranges of the encode CTAs, weighted by the work of each column tile
// (once every precision is known; NT threads).  Encode works through a tile
// in items: 64 rows of a 2-bit group cost about 1, 32 rows of a 4-bit group
// about 1.35 and of an irregular group about 4.5, and a tile's write-out
// about 16 (units of 1/10 below).  CTA b gets the tiles [S_b, S_b+1) (in
// column-major order) where the weighted prefix reaches b / G of the total.
// floor(x / d) for 0 <= x < 2^53 and d > 0 without a 64-bit division.
__device__ __forceinline__ int64_t floor_div_small(int64_t x, int64_t d) {
  int64_t q = (int64_t)((double)x / (double)d);
  if (q * d > x)
    --q;
  else if ((q + 1) * d <= x)
    ++q;
  return q;
}

__device__ __forceinline__ int64_t enc_uniform_start(int64_t b, int64_t ntiles, int G) {
  return b * ntiles / G;
}

template <int NT>
__device__ void enc_partition(const QArgs& a, const uint32_t* s_cost /* nct, or null */,
                              long long* s_pref /* nct + 1 */) {
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  constexpr int NWARP = NT / 32;
  __shared__ long long s_part[NWARP];
  const int G = a.enc_grid, nct = a.nct, nrc = a.nrc;
  const int64_t ntiles = (int64_t)nct * nrc;
  if (G <= 0 || G > kMaxEncGrid) return;
  int32_t* S = a.ws.enc_start;
  if (ntiles < 2 * (int64_t)G || s_cost == nullptr || s_pref == nullptr) {
    for (int b = tid; b <= G; b += NT) S[b] = (int32_t)enc_uniform_start(b, ntiles, G);
    return;
  }
  // s_pref[ct] = weighted work of the column tiles before ct (exclusive scan)
  const int per = (nct + NT - 1) / NT;
  const int c0 = min(nct, tid * per), c1 = min(nct, c0 + per);
  long long local = 0;
  for (int ct = c0; ct < c1; ++ct) local += (long long)s_cost[ct] * nrc;
  long long incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_part[warp] = incl;
  sync_nt<NT>();
  long long P = incl - local;
  for (int w = 0; w < warp; ++w) P += s_part[w];
  for (int ct = c0; ct < c1; ++ct) {
    s_pref[ct] = P;
    P += (long long)s_cost[ct] * nrc;
  }
  if (c1 == nct && c0 < c1) s_pref[nct] = P;
  sync_nt<NT>();
  const long long total = s_pref[nct];
  // CTA b starts in the column tile with s_pref[ct] G <= b total <
  // s_pref[ct + 1] G (the prefix grows strictly: every tile costs > 0), at
  // row chunk ceil((b total - s_pref[ct] G) / (G cost)) of it; the products
  // stay below 2^53 (M K < 2^31)
  for (int b = 1 + tid; b < G; b += NT) {
    const long long bt = (long long)b * total;
    int lo = 0, hi = nct - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_pref[mid] * G <= bt)
        lo = mid;
      else
        hi = mid - 1;
    }
    const long long num = bt - s_pref[lo] * G, den = (long long)G * s_cost[lo];
    S[b] = (int32_t)((int64_t)lo * nrc + floor_div_small(num + den - 1, den));
  }
  if (tid == 0) {
    S[0] = 0;
    S[G] = (int32_t)ntiles;
  }
}

// Interval of a group's fp32 serial sum as sortable keys (lo rounded down,
// hi rounded up) from its flags, prediction P and moment (M rows of 16
// terms).  NaN / inf groups are exact.
__device__ __forceinline__ uint2 sens_interval_of(uint32_t f, double P, double mom, int64_t M) {
  if (f & kGrpNaN) return make_uint2(0xFFFFFFFFu, 0xFFFFFFFFu);
  if (f & kGrpInf) return make_uint2(0x7F800000u, 0x7F800000u);
  const double n = 16.0 * (double)M;
  const double dcr = n * kEps24;
  if ((f & kGrpLoose) || dcr >= 0.5) return make_uint2(0u, 0x7F800000u);
  const double eps = 32.0 * kEps24;
  const double D = dcr / (1.0 - dcr);
  const double E = kEps24 * (1.0 + eps) * (1.0 + D) * mom * (1.0 + 1e-6) + n * 0x1p-148;
  const double lo = fmax(P * (1.0 - eps) - E, 0.0), hi = P * (1.0 + eps) + E;
  return make_uint2(__float_as_uint(__double2float_rd(lo)),
                    __float_as_uint(__double2float_ru(hi)));  // +inf past FLT_MAX
}

// The selection from the intervals (the last stats CTA; NT threads).  Group g
// is certainly 4-bit if its lower bound exceeds the (n4+1)-th largest upper
// bound (at most n4 groups, g included, can reach its sum), certainly 2-bit
// if its upper bound is below the n4-th largest lower bound (n4 groups surely
// exceed it).  The rest are pending; if all or none of them must be 4-bit
// the selection is complete, otherwise their exact sums decide.
constexpr int kSelKPT = 8;  // keys per thread held in registers by the selection

// Encode work of a group (units of 1/10; a column tile's write-out is 160).
__device__ __forceinline__ uint32_t enc_group_cost(int pr, uint8_t greg) {
  return !((greg >> pr) & 1) ? 180u : pr ? 54u : 20u;
}

template <int NT>
__device__ void select_from_intervals(const QArgs& a, uint8_t* scratch, size_t scratch_bytes) {
  const int ng = a.ng, n4 = a.n4, nct = a.nct;
  const int tid = threadIdx.x % NT, lane = threadIdx.x & 31, warp = tid >> 5;
  constexpr int NWARP = NT / 32;
  __shared__ uint32_t hist[1024];
  __shared__ uint32_t s4[4];
  __shared__ uint32_t s_wsum[NWARP];
  __shared__ uint32_t s_cnt[2];
  // scratch: the keys (only when they do not fit in registers and do fit
  // here), then the column tiles' encode costs and their prefix
  const bool reg_keys = ng <= kSelKPT * NT;
  const bool keys_in_smem = !reg_keys && (size_t)ng * 8 <= scratch_bytes;
  const size_t cost_off = keys_in_smem ? (size_t)ng * 8 : 0;
  const size_t pref_off = (cost_off + (size_t)nct * 4 + 7) & ~(size_t)7;
  const bool cost_in_smem = pref_off + (size_t)(nct + 1) * 8 <= scratch_bytes;
  uint2* keys = reinterpret_cast<uint2*>(scratch);
  uint32_t* s_cost = reinterpret_cast<uint32_t*>(scratch + cost_off);
  long long* s_pref = reinterpret_cast<long long*>(scratch + pref_off);
  auto key_of = [&](int g) -> uint2 { return keys_in_smem ? keys[g] : __ldcg(a.ws.gkey + g); };
  if (cost_in_smem)
    for (int ct = tid; ct < nct; ct += NT) s_cost[ct] = 160;
  if (tid == 0) s_cnt[0] = s_cnt[1] = 0;
  // adds the encode cost of group g (precision pr) to its column tile; the
  // groups of a column tile are 8 consecutive indices, and with NT a multiple
  // of 8 they sit in 8 consecutive lanes (all lanes call it)
  auto add_cost = [&](int g, bool on, int pr, uint8_t greg) {
    uint32_t c = on ? enc_group_cost(pr, greg) : 0u;
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    c += __shfl_xor_sync(0xffffffffu, c, 2);
    c += __shfl_xor_sync(0xffffffffu, c, 4);
    if ((lane & 7) == 0 && c != 0u && g < ng) atomicAdd(&s_cost[g / kTileGroups], c);
  };
  int pending = 0;
  if (a.select && n4 > 0) {
    const bool all_in = n4 >= ng;
    uint32_t Alo = 0, Bhi = 0;
    uint32_t kx[kSelKPT], ky[kSelKPT];
    uint8_t kg[kSelKPT];
    if (reg_keys) {
#pragma unroll
      for (int i = 0; i < kSelKPT; ++i) {
        const int g = tid + i * NT;
        const uint2 k = g < ng ? __ldcg(a.ws.gkey + g) : make_uint2(0u, 0u);
        kx[i] = k.x;
        ky[i] = k.y;
        kg[i] = g < ng ? a.ws.greg[g] : (uint8_t)0;
      }
      kth_largest2_reg<NT, kSelKPT>(kx, ky, ng, n4, all_in ? n4 : n4 + 1, hist, s4, Alo, Bhi);
    } else {
      if (keys_in_smem)
        for (int g = tid; g < ng; g += NT) keys[g] = __ldcg(a.ws.gkey + g);
      sync_nt<NT>();
      auto lo_of = [&](int g) -> uint32_t { return key_of(g).x; };
      auto hi_of = [&](int g) -> uint32_t { return key_of(g).y; };
      kth_largest2<NT>(ng, n4, lo_of, all_in ? n4 : n4 + 1, hi_of, hist, s4, Alo, Bhi);
    }
    // certainly 4-bit (1), certainly 2-bit (0) or pending (2); the decided
    // groups' encode costs go to their column tiles now
    uint32_t c_in = 0, c_pend = 0;
    auto classify = [&](int g, uint32_t l, uint32_t h, uint8_t greg, bool on) {
      uint8_t p = 0;
      if (on) {
        p = a.all_pending ? 2 : ((all_in || l > Bhi) ? 1 : (h < Alo ? 0 : 2));
        c_in += p == 1;
        c_pend += p == 2;
        a.ws.prec[g] = p;
      }
      if (cost_in_smem) add_cost(g, on && p != 2, p, greg);
    };
    if (reg_keys) {
#pragma unroll
      for (int i = 0; i < kSelKPT; ++i)
        if (i * NT < ng) classify(tid + i * NT, kx[i], ky[i], kg[i], tid + i * NT < ng);
    } else {
      for (int g0 = 0; g0 < ng; g0 += NT) {  // whole warps (add_cost shuffles)
        const int g = g0 + tid;
        const uint2 k = g < ng ? key_of(g) : make_uint2(0u, 0u);
        classify(g, k.x, k.y, g < ng ? a.ws.greg[g] : (uint8_t)0, g < ng);
      }
    }
    c_in = __reduce_add_sync(0xffffffffu, c_in);
    c_pend = __reduce_add_sync(0xffffffffu, c_pend);
    if (lane == 0) {
      atomicAdd(&s_cnt[0], c_in);
      atomicAdd(&s_cnt[1], c_pend);
    }
    sync_nt<NT>();
    const int need = n4 - (int)s_cnt[0], np = (int)s_cnt[1];
    if (tid == 0) a.ws.hdr->n_straddle = (uint32_t)np;
    if (np > 0 && !a.all_pending && (need <= 0 || need >= np)) {
      // all pending groups take the same precision
      const uint8_t to = need > 0 ? 1 : 0;
      for (int g0 = 0; g0 < ng; g0 += NT) {
        const int g = g0 + tid;
        const bool pend = g < ng && a.ws.prec[g] == 2;
        if (pend) a.ws.prec[g] = to;
        if (cost_in_smem) add_cost(g, pend, to, pend ? a.ws.greg[g] : (uint8_t)0);
      }
      sync_nt<NT>();
    } else if (np > 0) {
      pending = 1;
      if (tid == 0) a.ws.hdr->need = (uint32_t)need;
    }
  } else {
    for (int g0 = 0; g0 < ng; g0 += NT) {
      const int g = g0 + tid;
      if (g < ng) a.ws.prec[g] = 0;
      if (cost_in_smem) add_cost(g, g < ng, 0, g < ng ? a.ws.greg[g] : (uint8_t)0);
    }
    sync_nt<NT>();
  }
  if (!pending) {
    // every precision is known: the tile split here; group_precision,
    // any_irregular and the 2nd-order table are written by the CTAs of the
    // next kernel in parallel (tables_grid)
    enc_partition<NT>(a, cost_in_smem ? s_cost : nullptr, cost_in_smem ? s_pref : nullptr);
    if (tid == 0) {
      a.ws.hdr->n_dec = (uint32_t)ng;
      a.ws.hdr->n_pend = 0;
    }
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
// stats kernel: persistent CTAs, each over a contiguous column-major range of
// the 128 x 128 tiles, a three-stage TMA ring so the next tiles' loads
// overlap the current tile's work, one warp per group.
// ---------------------------------------------------------------------------

// w*w of the two fp16 values of `w`, accumulated into a0 / a1 in fp32 (the
// squares are exact in fp32; one rounding per add).
__device__ __forceinline__ void sq_acc2(uint32_t w, float& a0, float& a1) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
      "fma.rn.f32.f16 %0, l, l, %0;\n\tfma.rn.f32.f16 %1, h, h, %1;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "r"(w));
}

// The same swizzled tile layout from plain loads (inputs TMA cannot take);
// `fill` outside the matrix.
__device__ __forceinline__ void tile_fill(const __half* W, int64_t M, int64_t K, uint8_t* dst,
                                          int64_t t, int nct, uint16_t fill) {
  const int rc = (int)(t / nct), ct = (int)(t % nct);
  for (int e = threadIdx.x; e < kChunkRows * kTileCols; e += blockDim.x) {
    const int r = e / kTileCols, c = e % kTileCols;
    const int64_t gr = (int64_t)rc * kChunkRows + r, gc = (int64_t)ct * kTileCols + c;
    const uint16_t v = (gr < M && gc < K) ? __half_as_ushort(W[gr * K + gc]) : fill;
    const int half = c >> 6, cc = c & 63;
    *reinterpret_cast<uint16_t*>(dst + half * kBoxBytes + r * 128 +
                                 (((cc >> 3) ^ (r & 7)) << 4) + (cc & 7) * 2) = v;
  }
}

// Tile u of the stats pass is (column tile u / nrc, row chunk u % nrc); stats
// CTA b takes the tiles [U_b, U_b+1), U_b = floor(b * ntiles / G), G <= ntiles
// (so no range is empty).  A CTA's tiles of one column tile form a segment,
// identified by b + ct (both grow along u, so the ids are distinct).
__device__ __forceinline__ int stats_start(int b, int ntiles, int G) {
  return (int)floor_div_small((int64_t)b * ntiles, G);
}

// The last CTA to finish column tile ct: each group's totals from its
// segments (one warp per group, lanes over the segments in row order), its
// flags, min / max, sensitivity interval and the parameters of both
// precisions.  The prediction P is the sum of the segments' sums; the moment
// sum_j terms_j * P_incl(j) adds, per segment, its own moment and
// (prediction before the segment) * (its terms); any fp64 summation order is
// covered by the interval's slack.
template <bool kSens>
__device__ __noinline__ void ct_combine(const QArgs& A, int ct, int warp, int lane) {
  const int64_t g = (int64_t)ct * kTileGroups + warp;
  if (g >= A.ng) return;
  const int64_t M = A.M;
  const int nrc = A.nrc, G = A.stats_grid, ntiles = A.nct * A.nrc;
  const int64_t u0 = (int64_t)ct * nrc, u1 = u0 + nrc;
  // the CTAs holding the column tile's first and last chunk
  const int b0 = (int)floor_div_small((u0 + 1) * G - 1, ntiles);
  const int b1 = (int)floor_div_small(u1 * G - 1, ntiles);
  float mn = INFINITY, mx = -INFINITY;
  uint32_t flags = 0;
  double carry = 0.0, mom = 0.0;
  for (int bb = b0; bb <= b1; bb += 32) {
    const int b = bb + lane;
    double sum = 0.0, smom = 0.0;
    uint4 w = make_uint4(__float_as_uint(INFINITY), __float_as_uint(-INFINITY), 0u, 0u);
    if (b <= b1) {
      const SegRec* src = A.ws.seg + ((size_t)(b + ct) * kTileGroups + warp);
      const double2 d = __ldcg(reinterpret_cast<const double2*>(src));
      w = __ldcg(reinterpret_cast<const uint4*>(src) + 1);
      sum = d.x;
      smom = d.y;
    }
    mn = fminf(mn, __uint_as_float(w.x));
    mx = fmaxf(mx, __uint_as_float(w.y));
    flags |= w.w;
    if (kSens) {
      double incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      mom += smom + (carry + (incl - sum)) * (16.0 * (double)w.z);
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
    if (lane == 0) {
      A.ws.gpred[g] = carry;
      A.ws.gmom[g] = mom;
      A.ws.gflag[g] = flags;
      A.ws.gkey[g] = sens_interval_of(flags, carry, mom, M);
    }
  }
  if (lane == 0) {
    A.ws.gmin[g] = mn;
    A.ws.gmax[g] = mx;
  }
  group_params_warp(A.ws.params, A.ws.gscale, A.ws.greg, g, mn, mx, lane);
}


// stats: persistent CTAs, each streaming its contiguous range of tiles
// (column-major) through a TMA ring, one warp per group of the current tile.
// Per tile: the per-column sums of w*w (kept for the exact sums of pending
// groups); per segment, in registers: min / max and the prediction sums
// (lane = column: RN(1/h) * column sum, in fp64).  At a segment's end its
// record is written; the CTA completing a column tile combines its groups,
// and the CTA completing the last column tile selects the 4-bit groups
// (torch_ops.cu:149-179) and splits the encode tiles.
template <bool kSens>
__device__ __forceinline__ void stats_body(const CUtensorMap& tmap, const QArgs& A, int use_tma,
                                           int bid, int G) {
  extern __shared__ uint8_t dsm_raw[];
  // 1024-byte aligned for the 128-byte swizzle; offset arithmetic on the
  // shared array keeps the pointer in the shared space (plain LDS)
  uint8_t* dsm = dsm_raw + ((1024u - (smem_u32(dsm_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full[kStages];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t M = A.M, K = A.K;
  const int nrc = A.nrc, nct = A.nct;
  const int ntiles = nct * nrc;  // below 2^31 (checked on the host)
  const int u_begin = stats_start(bid, ntiles, G);
  const int u_end = stats_start(bid + 1, ntiles, G);
  int u_ahead = u_begin;  // thread 0: the next tile to load
  int ct_ahead = u_begin / nrc, rc_ahead = u_begin - ct_ahead * nrc;
  // W stays in L2 for encode's second read where it fits (encode's own
  // loads and stores are evict-first)
  const uint64_t pol = l2_evict_last();
  auto issue = [&](int s) {
    uint8_t* dst = dsm + (size_t)s * kTileBytes;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&full[s], kTileBytes);
    tma_load_2d_hint(dst, &tmap, &full[s], ct_ahead * kTileCols, rc_ahead * kChunkRows, pol);
    tma_load_2d_hint(dst + kBoxBytes, &tmap, &full[s], ct_ahead * kTileCols + 64,
                     rc_ahead * kChunkRows, pol);
    ++u_ahead;
    if (++rc_ahead == nrc) {
      rc_ahead = 0;
      ++ct_ahead;
    }
  };
  if (tid == 0 && use_tma) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    for (int s = 0; s < kStages && u_ahead < u_end; ++s) issue(s);
  }
  __syncthreads();
  bool failed = false;
  uint32_t bad = 0;  // thread 0: stages whose wait ran out
  int st = 0;
  uint32_t ph = 0;  // phase parity of stage st
  // the open segment of this warp's group: min / max, and per lane the
  // prediction sum and moment of its column (even lanes; odd lanes hold 0)
  __half2 smn = __float2half2_rn(INFINITY), smx = __float2half2_rn(-INFINITY);
  double ssum = 0.0, smom = 0.0, rcl = 0.0;
  bool snan = false, sinf = false, sloose = false;
  uint32_t srows = 0;
  int seg_rc0 = 0;
  // lane = row rl (of 16) of each 16-row step and half hh of the group's 16
  // columns (a quarter warp reads 8 rows of one half: 8 distinct swizzle
  // slots); after the column-sum butterfly lane l holds column
  // 8 hh + 4 b3 + 2 b2 + b1 (bits of l)
  const int rl = lane & 15, hh = lane >> 4;
  const bool b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
  const int col = 8 * hh + (b3 ? 4 : 0) + (b2 ? 2 : 0) + (b1 ? 1 : 0);
  const bool even = !(lane & 1);
  int ct = u_begin / nrc, rc = u_begin - ct * nrc;
  for (int u = u_begin; u < u_end; ++u) {
    uint8_t* buf = dsm + (size_t)st * kTileBytes;
    const int64_t row0 = (int64_t)rc * kChunkRows;
    const int gi = warp;
    const int64_t g = (int64_t)ct * kTileGroups + gi;
    const int64_t c0 = g * kGroup1;
    const bool seg_first = u == u_begin || rc == 0;
    const bool seg_last = u == u_end - 1 || rc == nrc - 1;
    const int rows = (int)min64(kChunkRows, M - row0);
    if (seg_first) {
      smn = __float2half2_rn(INFINITY);
      smx = __float2half2_rn(-INFINITY);
      ssum = smom = 0.0;
      snan = sinf = sloose = false;
      srows = 0;
      seg_rc0 = rc;
      if (kSens) {
        float r = 1.0f;
        if (g < A.ng && c0 + col < K) {
          const float h = __ldg(A.hess + c0 + col);
          if (h > 1e-8f) {
            r = __frcp_rn(h);
            sloose = !(h >= 0x1p-60f && h <= 0x1p60f);
          }
        }
        rcl = even ? (double)r : 0.0;
      }
    }
    if (use_tma) {
      const bool ok = mbar_wait(&full[st], ph);
      failed |= !ok;
      if (tid == 0 && !ok) bad |= 1u << st;
    } else {
      tile_fill(A.W, M, K, buf, (int64_t)rc * nct + ct, nct, 0x7E00);
      __syncthreads();
    }
    if (g < A.ng) {
      const int gs = (int)min64(kGroup1, K - c0);
      const uint32_t cmask = gs >= 16 ? 0xFFFFu : ((1u << gs) - 1u);
      const bool edge = (row0 + kChunkRows > M) || gs < kGroup1;
      const size_t rec = (size_t)g * nrc + rc;
      __half2 hmn = smn, hmx = smx;
      float acc[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = 0.0f;
      if (!edge) {  // the whole tile lies inside the matrix (all but the edge tiles)
#pragma unroll
        for (int s = 0; s < kChunkRows / 16; ++s) {
          const uint4 q = tile_half(buf, gi, s * 16 + rl, hh);
          const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            hmn = __hmin2(hmn, as_h2(w4[k]));
            hmx = __hmax2(hmx, as_h2(w4[k]));
            if (kSens) sq_acc2(w4[k], acc[2 * k], acc[2 * k + 1]);
          }
        }
      } else {
        // this half's valid columns
        const uint32_t hmask = (cmask >> (8 * hh)) & 0xFFu;
#pragma unroll 1
        for (int s = 0; s < kChunkRows / 16; ++s) {
          const int r = s * 16 + rl;
          const uint4 q = tile_half(buf, gi, r, hh);
          const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
          const uint32_t vmask = row0 + r < M ? hmask : 0u;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // outside the matrix: NaN for min / max (ignored), 0 for sums
            const uint32_t w = w4[k];
            const uint32_t keep = (((vmask >> (2 * k)) & 1u) ? 0x0000FFFFu : 0u) |
                                  (((vmask >> (2 * k + 1)) & 1u) ? 0xFFFF0000u : 0u);
            const uint32_t ws = w & keep;
            const uint32_t wm = ws | (0x7E007E00u & ~keep);
            hmn = __hmin2(hmn, as_h2(wm));
            hmx = __hmax2(hmx, as_h2(wm));
            if (kSens) sq_acc2(ws, acc[2 * k], acc[2 * k + 1]);
          }
        }
      }
      smn = hmn;
      smx = hmx;
      srows += (uint32_t)rows;
      if (kSens) {
        // per-column sums over the chunk's rows by a transposing butterfly
        // over the row bits 3..1 (each step halves the columns a lane
        // holds), then a plain sum over bit 0
        float a4[4], a2[2];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          a4[j] = __fadd_rn(b3 ? acc[4 + j] : acc[j],
                            __shfl_xor_sync(0xffffffffu, b3 ? acc[j] : acc[4 + j], 8));
#pragma unroll
        for (int j = 0; j < 2; ++j)
          a2[j] = __fadd_rn(b2 ? a4[2 + j] : a4[j],
                            __shfl_xor_sync(0xffffffffu, b2 ? a4[j] : a4[2 + j], 4));
        float a1 = __fadd_rn(b1 ? a2[1] : a2[0], __shfl_xor_sync(0xffffffffu, b1 ? a2[0] : a2[1], 2));
        a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
        if (even) A.ws.ccol[rec * 16 + col] = a1;
        // the chunk's prediction, lane by lane (exact products); a NaN / inf
        // column sum is flagged and left out
        snan |= isnan(a1);
        sinf |= isinf(a1);
        ssum += isfinite(a1) ? (double)a1 * rcl : 0.0;
        smom = fma(16.0 * (double)rows, ssum, smom);
      }
      if (seg_last) {
        float mn = fminf(__half2float(__low2half(smn)), __half2float(__high2half(smn)));
        float mx = fmaxf(__half2float(__low2half(smx)), __half2float(__high2half(smx)));
        mn = warp_min(mn);
        mx = warp_max(mx);
        double sum = ssum, mom = smom;
        uint32_t flags = 0;
        if (kSens) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
            mom += __shfl_xor_sync(0xffffffffu, mom, o);
          }
          flags = (__any_sync(0xffffffffu, snan) ? kGrpNaN : 0u) |
                  (__any_sync(0xffffffffu, sinf) ? kGrpInf : 0u) |
                  (__any_sync(0xffffffffu, sloose) ? kGrpLoose : 0u);
        }
        if (lane == 0) {
          SegRec* dst = A.ws.seg + ((size_t)(bid + ct) * kTileGroups + gi);
          reinterpret_cast<double2*>(dst)[0] = make_double2(sum, mom);
          reinterpret_cast<uint4*>(dst)[1] =
              make_uint4(__float_as_uint(mn), __float_as_uint(mx), srows, flags);
        }
      }
    }
    // zero this tile's share of the per-row outlier counts
    if (ct == 0)
      for (int r = tid; r < kChunkRows; r += kStatsThreads)
        if (row0 + r < M) A.ws.row_counts[row0 + r] = 0;
    __syncthreads();  // the stage is free
    if (tid == 0 && use_tma && u_ahead < u_end) issue(st);
    if (++st == kStages) {
      st = 0;
      ph ^= 1u;
    }
    if (++rc == nrc) {
      rc = 0;
      ++ct;
    }
  }
  grid_launch_dependents();
  failed = __syncthreads_or(failed) != 0;
  if (tid == 0) {
    if (failed) atomicOr(&A.ws.hdr->status, kStatusTimeout);
    // loads whose wait ran out may still be in flight: let them land (the
    // stage's last issued phase, bounded) before the CTA exits
    for (int s = 0; s < kStages; ++s)
      if (bad & (1u << s)) (void)mbar_wait(&full[s], 0u), (void)mbar_wait(&full[s], 1u);
  }
}

template <int NB>
struct __align__(64) StatsBatch {
  CUtensorMap tmap[NB];
  QArgs a[NB];
  int use_tma[NB];
  BatchMap<NB> bm;
};

template <bool kSens, int NB>
__global__ void __launch_bounds__(kStatsThreads, 2)
    stats_kernel(const __grid_constant__ StatsBatch<NB> P) {
  const CtaSlot c = batch_slot(P.bm);
  stats_body<kSens>(P.tmap[c.m], P.a[c.m], P.use_tma[c.m], c.b, c.G);
}

// combine: a warp per group (grid-stride) adds the group's segment records
// in row order (ct_combine): min / max, sensitivity interval, the parameters
// of both precisions and their code thresholds.  The CTA finishing last
// selects the 4-bit groups (torch_ops.cu:149-179) and splits the encode
// tiles.  Launched after stats with programmatic dependent launch.
constexpr int kCombThreads = 256;
template <bool kSens, int NB>
__global__ void __launch_bounds__(kCombThreads, 1)
    combine_kernel(const __grid_constant__ ArgsBatch<NB> P) {
  extern __shared__ uint8_t csm[];
  __shared__ int s_last;
  const CtaSlot c = batch_slot(P.bm);
  const QArgs& A = P.a[c.m];
  const int tid = threadIdx.x, lane = tid & 31;
  grid_dependency_wait();  // every segment record written
  const int64_t nw = (int64_t)c.G * (kCombThreads / 32);
  for (int64_t g = ((int64_t)c.b * kCombThreads + tid) >> 5; g < A.ng; g += nw) {
    ct_combine<kSens>(A, (int)(g / kTileGroups), (int)(g % kTileGroups), lane);
    __syncwarp();  // the parameters lanes 0 and 1 wrote
    group_thresholds_warp(A.ws.params, g, lane);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&A.ws.hdr->ticket_ct, 1u) == (unsigned)c.G - 1u;
  __syncthreads();
  grid_launch_dependents();
  if (!s_last || A.no_select) return;
  __threadfence();
  select_from_intervals<kCombThreads>(A, csm, (size_t)A.comb_smem);
}

// ---------------------------------------------------------------------------
// encode: the outlier test of the reference and the code helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool is_outlier(float x, float scale, int zero, float thr, int q,
                                           int fma_mode) {
  const float qz = (float)(q - zero);
  const float err = fma_mode ? fabsf(__fmaf_rn(-scale, qz, x))
                             : fabsf(__fsub_rn(x, __fmul_rn(scale, qz)));
  return err > thr;
}

// Codes of a regular group's run (16 values of one row) from its code
// thresholds T_j (the smallest fp16 value whose code is >= j; +inf if none):
// code(w) = #{j : w >= T_j}.  The run's words are re-paired so that half-word
// lane 0 of pair k holds element k and lane 1 element k + 8; then every
// packed comparison feeds one output position per lane.

// Lane select: a where the mask is set, b elsewhere.
__device__ __forceinline__ uint32_t lane_sel(uint32_t m, uint32_t a, uint32_t b) {
  return (m & a) | (~m & b);
}

// 2-bit: c_k = [P_k >= T1] + [P_k >= T2] + [P_k >= T3] (fp16 0..3, exact),
// accumulated as 1024 + c_0 + 4 c_1 + 16 c_2 + 64 c_3 (an fp16 integer below
// 2048, so its low mantissa byte is the four codes' 2-bit fields).
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

__device__ __forceinline__ uint32_t enc2_run(const Row16& v, uint32_t t1, uint32_t t2,
                                             uint32_t t3) {
  const uint32_t w[8] = {v.lo.x, v.lo.y, v.lo.z, v.lo.w, v.hi.x, v.hi.y, v.hi.z, v.hi.w};
  const __half2 T1 = as_h2(t1), T2 = as_h2(t2), T3 = as_h2(t3);
  // fp16 bit patterns: 1024, and the weights 1, 4, 16, 64 in both lanes
  constexpr uint32_t kW[4] = {0x3C003C00u, 0x44004400u, 0x4C004C00u, 0x54005400u};
  __half2 acc[2] = {as_h2(0x64006400u), as_h2(0x64006400u)};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const __half2 P = as_h2(__byte_perm(w[k >> 1], w[4 + (k >> 1)], (k & 1) ? 0x7632 : 0x5410));
    const __half2 c = __hadd2(__hadd2(__hge2(P, T1), __hge2(P, T2)), __hge2(P, T3));
    acc[k >> 2] = __hfma2(c, as_h2(kW[k & 3]), acc[k >> 2]);
  }
  // bytes: elements 0-3, 4-7 (low lanes), 8-11, 12-15 (high lanes)
  return __byte_perm(h2_bits(acc[0]), h2_bits(acc[1]), 0x6240);
}

// 4-bit: a two-level search with lane masks.  The coarse level compares with
// T4, T8, T12 (nested masks m4 >= m8 >= m12, c1 = their count); the fine
// level compares with T(4 c1 + 1..3), selected per lane from the masks; the
// code is 4 c1 + c2 with bit 3 = m8, bit 2 = m4 ^ m8 ^ m12, bit 1 = f2 and
// bit 0 = f1 ^ f2 ^ f3.  Lane masks are 0xFFFF per half, so each nibble is
// taken from its lane directly.

__device__ __forceinline__ void enc4_run(const Row16& v, const uint32_t (&t)[16], uint32_t& wa,
                                         uint32_t& wb) {
  const uint32_t w[8] = {v.lo.x, v.lo.y, v.lo.z, v.lo.w, v.hi.x, v.hi.y, v.hi.z, v.hi.w};
  uint32_t X[2] = {0u, 0u};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const __half2 P = as_h2(__byte_perm(w[k >> 1], w[4 + (k >> 1)], (k & 1) ? 0x7632 : 0x5410));
    const uint32_t m4 = __hge2_mask(P, as_h2(t[3]));
    const uint32_t m8 = __hge2_mask(P, as_h2(t[7]));
    const uint32_t m12 = __hge2_mask(P, as_h2(t[11]));
    uint32_t f[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint32_t F = lane_sel(m12, t[12 + i], lane_sel(m8, t[8 + i], lane_sel(m4, t[4 + i], t[i])));
      f[i] = __hge2_mask(P, as_h2(F));
    }
    const uint32_t b2 = m4 ^ m8 ^ m12, b0 = f[0] ^ f[1] ^ f[2];
    const int sh = 4 * (k & 3);
    X[k >> 2] |= (m8 & (0x00080008u << sh)) | (b2 & (0x00040004u << sh)) |
                 (f[1] & (0x00020002u << sh)) | (b0 & (0x00010001u << sh));
  }
  wa = __byte_perm(X[0], X[1], 0x5410);  // elements 0-7
  wb = __byte_perm(X[0], X[1], 0x7632);  // elements 8-15
}

// Irregular groups: the reference formula per element (quantize.cu:178-240),
// reading the run from the swizzled tile: (2-bit word or first 4-bit word,
// second 4-bit word, outlier count).
__device__ __noinline__ uint3 enc_irregular(const GroupParams& gp, const uint8_t* row_base,
                                            int lo_off, int hi_off, int gs) {
  const bool four = gp.levels == 16;
  uint32_t wa = 0, wb = 0, cnt = 0;
#pragma unroll 1
  for (int i = 0; i < gs; ++i) {
    const uint16_t hb =
        *reinterpret_cast<const uint16_t*>(row_base + (i < 8 ? lo_off : hi_off) + (i & 7) * 2);
    const float x = __half2float(__ushort_as_half(hb));
    const int q = code_of(x, gp.gmin, gp.scale, gp.levels);
    cnt += is_outlier(x, gp.scale, gp.zero, gp.thr, q, kOutlierFma);
    if (!four)
      wa |= (uint32_t)(q & 0x3) << (2 * i);
    else if (i < 8)
      wa |= (uint32_t)(q & 0xF) << (4 * i);
    else
      wb |= (uint32_t)(q & 0xF) << (4 * (i - 8));
  }
  return make_uint3(wa, wb, cnt);
}

// Exact sums of the pending groups (the first kExactCtas blocks of the encode
// grid): warps take (pending group, chunk) work items; the last chunk of a
// group assembles its exact sum, the last group completes the selection.
__device__ __noinline__ void exact_ctas(const QArgs& a, int bid, int G) {
  const Header* hdr = a.ws.hdr;
  const uint32_t np = *reinterpret_cast<const volatile uint32_t*>(&hdr->n_pend);
  if (np == 0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t ndec = *reinterpret_cast<const volatile uint32_t*>(&hdr->n_dec);
  __shared__ GroupDiv s_div[8];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s2[2];
  const int64_t nwork = (int64_t)np * a.nrc;
  for (int64_t w = (int64_t)bid * 8 + warp; w < nwork; w += (int64_t)G * 8) {
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
    const uint32_t fl = __ldcg(a.ws.gflag + g);
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
    // the tables follow in tables_kernel, over the whole grid
  }
}

// group_precision, any_irregular and the 2nd-order chunk table
// (quantize.cu:245-272) once every precision is known, by all CTAs of the
// grid: threads over groups, one warp per chunk.  Chunk c's scales are those
// of the groups s0 mod ng, s0 mod ng + 1, ... (cyclic, s0 = 256 c; the
// partial chunk is the last).
__device__ __noinline__ void tables_grid(const QArgs& a, int bid, int G) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = a.ng;
  bool irr = false;
  for (int g = bid * blockDim.x + tid; g < ng; g += G * blockDim.x) {
    const uint8_t pr = a.ws.prec[g];
    a.gp[g] = pr;
    irr |= !((a.ws.greg[g] >> pr) & 1);
  }
  if (__any_sync(0xffffffffu, irr) && lane == 0) atomicOr(&a.ws.hdr->any_irregular, 1u);
  auto scale_of = [&](int g) -> float {
    const uint32_t sh2 = __ldcg(a.ws.gscale + g);
    return __half2float(
        __ushort_as_half((uint16_t)(a.ws.prec[g] ? (sh2 >> 16) : (sh2 & 0xFFFFu))));
  };
  const ChunkLayout& cl = a.cl;
  const int nchunks = cl.ntab_full + cl.has_partial;
  const int64_t step = kGroup2 % ng;  // s0 mod ng advances by this per chunk
  const int nwarps = G * (blockDim.x >> 5);
  for (int ci = bid * (blockDim.x >> 5) + warp; ci < nchunks; ci += nwarps) {
    const bool partial = ci >= cl.ntab_full;
    const int64_t cidx = partial ? cl.nfull : ci;
    const int n = (int)min64(kGroup2, cl.total - cidx * kGroup2);
    float mn = 1e10f, mx = -1e10f;
    if (n >= ng) {  // every group at least once
      for (int g = lane; g < ng; g += 32) {
        const float v = scale_of(g);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
    } else {
      const int g0 = (int)((cidx * step) % ng);
      for (int k = lane; k < n; k += 32) {
        int g = g0 + k;
        if (g >= ng) g -= ng;
        const float v = scale_of(g);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
    }
    mn = warp_min(mn);
    mx = warp_max(mx);
    float sc2 = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
    if (sc2 < 1e-10f) sc2 = 1e-10f;
    if (lane == 0) {
      const int z2 = f2i_rz(roundf(__fdiv_rn(-mn, sc2)));
      if (z2 < -128 || z2 > 127) atomicOr(&a.ws.hdr->status, kStatusZero2Wrap);
      a.ws.chunk_tab[partial ? cl.ntab_full : ci] =
          make_float4(mn, sc2, __int_as_float((int)__half_as_ushort(__float2half_rn(sc2))),
                      __int_as_float((int)(int8_t)z2));
    }
    if (!partial) {
      // the chunk's 256 2nd-order codes (quantize.cu:274-279), in flat order:
      // every full chunk of the same position in the period has them
      const int g0 = (int)((cidx * step) % ng);
      for (int k = lane; k < kGroup2; k += 32) {
        int g = g0 + k % ng;
        if (g >= ng) g -= ng;
        const int q2 = f2i_rz(roundf(__fdiv_rn(__fsub_rn(scale_of(g), mn), sc2)));
        a.ws.sq_pat[ci * kGroup2 + k] = (uint8_t)max(0, min(15, q2));
      }
    }
  }
}

// Between the selection and the tables: the exact sums of the pending groups
// (whose last warp completes the selection); nothing when no group is
// pending.
// Encode is launched only when this kernel is done: its CTAs are large
// (two fill an SM) and, resident early, would hold the SMs that other work
// on other streams can use meanwhile.
template <int NB>
__global__ void __launch_bounds__(256) exact_kernel(const __grid_constant__ ArgsBatch<NB> P) {
  const CtaSlot c = batch_slot(P.bm);
  const QArgs& a = P.a[c.m];
  grid_dependency_wait();  // stats and the selection complete
  // every group's code thresholds for both precisions (a warp per group),
  // when the combine kernel did not find them (row-split slabs)
  if (a.exact_thresholds) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)c.G * (blockDim.x >> 5);
    for (int64_t g = ((int64_t)c.b * blockDim.x + threadIdx.x) >> 5; g < a.ng; g += nw)
      group_thresholds_warp(a.ws.params, g, lane);
  }
  if (*reinterpret_cast<const volatile uint32_t*>(&a.ws.hdr->n_pend) != 0)
    exact_ctas(a, c.b, c.G);
  grid_launch_dependents();
}

// Once every precision is known: group_precision, any_irregular and the
// 2nd-order chunk table over the whole grid; after exact sums (the
// selection's tile split predates them) CTA 0 splits the legacy encode's
// tiles evenly.
template <int NB>
__global__ void __launch_bounds__(256) tables_kernel(const __grid_constant__ ArgsBatch<NB> P) {
  const CtaSlot c = batch_slot(P.bm);
  const QArgs& a = P.a[c.m];
  grid_dependency_wait();  // the selection (and exact sums) complete
  tables_grid(a, c.b, c.G);
  if (c.b == 0 && *reinterpret_cast<const volatile uint32_t*>(&a.ws.hdr->n_pend) != 0)
    enc_partition<256>(a, nullptr, nullptr);
  grid_launch_dependents();
}

// ---------------------------------------------------------------------------
// post: 2nd-order scales / zeros (quantize.cu:245-272 over the flattened
// [M, ng] scales) and the outlier row pointers (torch_ops.cu:210-229), done
// by encode's CTAs.
// ---------------------------------------------------------------------------
// 2nd-order scales / zeros, and the row pointers when no group can hold
// outliers (all CTAs of encode, grid-stride, once the tables are final).
__device__ __forceinline__ void post_prologue(const QArgs& a, int bid, int G) {
  const int64_t M = a.M;
  const int64_t gtid = (int64_t)bid * blockDim.x + threadIdx.x;
  const int64_t gthreads = (int64_t)G * blockDim.x;
  const ChunkLayout& cl = a.cl;
  for (int64_t c = gtid; c < cl.ng2; c += gthreads) {
    const float4 e = a.ws.chunk_tab[c < cl.nfull ? (int)(c % cl.period) : cl.ntab_full];
    a.scales2[c] = __ushort_as_half((uint16_t)__float_as_int(e.z));
    a.zeros2[c] = (int8_t)__float_as_int(e.w);
  }
  if (a.ws.hdr->any_irregular == 0) {
    for (int64_t r = gtid; r <= M; r += gthreads) a.row_ptrs[r] = 0;
    if (gtid == 0) *a.nnz = 0;
  }
}

// When groups may hold outliers: the last encode CTA to finish turns the
// per-row counts into row pointers (all threads of every CTA call it;
// `part`: NT entries of shared scratch the CTA no longer needs).
template <int NT>
__device__ __forceinline__ void post_rowptr_scan(const QArgs& a, int G, long long* part) {
  if (a.ws.hdr->any_irregular == 0) return;
  __shared__ int s_last;
  const int tid = threadIdx.x;
  const int64_t M = a.M;
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&a.ws.hdr->ticket_post, 1u) == (unsigned)G - 1u;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int nt = blockDim.x;
  const int64_t per = ceil_div(M, (int64_t)nt);
  const int64_t q0 = min64(M, tid * per), q1 = min64(M, q0 + per);
  long long sum = 0;
  for (int64_t r = q0; r < q1; ++r) sum += __ldcg(a.ws.row_counts + r);
  part[tid] = sum;
  __syncthreads();
  for (int o = 1; o < nt; o <<= 1) {
    const long long y = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += y;
    __syncthreads();
  }
  long long run = part[tid] - sum;
  if (tid == 0) a.row_ptrs[0] = 0;
  for (int64_t r = q0; r < q1; ++r) {
    run += __ldcg(a.ws.row_counts + r);
    a.row_ptrs[r + 1] = (int32_t)run;
  }
  if (tid == nt - 1) *a.nnz = (int32_t)part[tid];
}

// encode: persistent CTAs over the 128 x 128 tiles of W.  CTA b takes a
// contiguous range of tiles in column-major order (tile u: column tile
// u / nrc, row chunk u % nrc), weighted by work when the selection split the
// tiles (enc_partition), so its tiles mostly share one column tile and
// the per-column-tile context -- kinds and thresholds of the 8 groups, their
// 2nd-order codes and the list of work items sorted by cost -- is built once
// per column tile.  An item is 64 rows of a 2-bit group (a lane codes rows r
// and r + 32) or 32 rows of a 4-bit or irregular group (about 2.7 times
// costlier per row); warps take items from a shared counter, costliest
// first, so the tile's items spread evenly over the warps.  Tiles arrive
// through a two-stage TMA ring and every thread waits on the stage's mbarrier
// itself; codes are
// staged group-major (lane = row; rows padded so the transposing reads are
// conflict-free too) in one of two buffers and leave as whole tile rows:
// 16-byte stores of packed_2bit, packed_4bit, scales_1st and 8-byte stores of
// zeros_1st and scales_1st_quant.  One block barrier per tile.
constexpr int kEncKind2 = 0, kEncKind4 = 1, kEncKindIrr = 2, kEncKindNone = 3;
constexpr int kMaxRowPeriod = kGroup2;           // 256 / gcd(ng, 256) rows

struct __align__(16) EncCtx {
  uint4 thr[kTileGroups][4];                   // T_1..T_15 as broadcast half2, +inf pad
  uint8_t sqrow[kMaxRowPeriod][kTileGroups];   // 2nd-order code by (row mod period, group)
  uint4 shv;                                   // scales_1st of the 8 groups (fp16)
  uint2 zv;                                    // zeros_1st of the 8 groups
  uint8_t kind[kTileGroups];
  uint8_t gs[kTileGroups];                     // columns of the group inside K
  uint8_t pr[kTileGroups];                     // precision (1 = 4-bit)
  uint8_t items[kTileGroups * kSteps];         // group | step << 3 | (64 rows) << 5
  int nitems;
};

// Output words of (group, row) of one tile, exactly as stored: packed_2bit
// (0 for a 4-bit group) and packed_4bit (0 for a 2-bit group).
constexpr int kCodePitch = kChunkRows + 4;
struct __align__(16) EncCodes {
  uint32_t p2[kTileGroups][kCodePitch];
  uint2 p4[kTileGroups][kCodePitch];
};

// The context of column tile ct (all threads; ends with a block barrier).
// rp = 256 / gcd(ng, 256): the flat index r * ng + g of scales_1st advances
// by a whole number of 256-long 2nd-order chunks every rp rows, so row r's
// codes depend on r mod rp only (full chunks; rows that reach the partial
// last chunk are coded directly in the write-out).
__device__ __forceinline__ void enc_build_ctx(const QArgs& a, EncCtx& cx, int ct, int rp) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = a.ng;
  const int64_t g = (int64_t)ct * kTileGroups + warp;
  uint32_t t = 0x7C007C00u;  // +inf: never reached
  int kind = kEncKindNone, pr = 0, gs = 0;
  uint16_t sh = 0;
  int8_t z = 0;
  if (warp < kTileGroups && g < ng) {
    pr = a.ws.prec[g];
    const GroupParams& p = a.ws.params[2 * g + pr];
    if (lane < 15) t = (uint32_t)p.thresh[lane] * 0x00010001u;
    kind = (p.flags & kFlagRegular) ? (pr ? kEncKind4 : kEncKind2) : kEncKindIrr;
    gs = (int)min64(kGroup1, a.K - g * kGroup1);
    sh = (uint16_t)p.scale_h;
    z = (int8_t)p.zero;
  }
  if (warp < kTileGroups && lane < 16) (&cx.thr[warp][0].x)[lane] = t;
  if (warp < kTileGroups && lane == 0) {
    cx.kind[warp] = (uint8_t)kind;
    cx.gs[warp] = (uint8_t)gs;
    cx.pr[warp] = (uint8_t)pr;
    reinterpret_cast<uint16_t*>(&cx.shv)[warp] = sh;
    reinterpret_cast<int8_t*>(&cx.zv)[warp] = z;
  }
  __syncthreads();
  if (warp == 0) {
    // the item list, costliest items first: irregular groups (4 items of 32
    // rows), 2-bit groups (2 items of 64 rows), 4-bit groups (4 items of 32
    // rows), each kind in group order
    const int kd = lane < kTileGroups ? cx.kind[lane] : kEncKindNone;
    const int n = kd == kEncKind2 ? 2 : kd == kEncKindNone ? 0 : 4;
    const unsigned below = (1u << lane) - 1u;
    int pos = 0;
    const int order[3] = {kEncKindIrr, kEncKind2, kEncKind4};
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const unsigned m = __ballot_sync(0xffffffffu, kd == order[q]);
      const int per = order[q] == kEncKind2 ? 2 : 4;
      if (kd == order[q]) pos += per * __popc(m & below);
      else if ((kd == kEncKind2 && q == 0) || (kd == kEncKind4 && q < 2)) pos += per * __popc(m);
    }
    for (int k = 0; k < n; ++k)
      cx.items[pos + k] = (uint8_t)(n == 2 ? (lane | ((2 * k) << 3) | (1 << 5)) : (lane | (k << 3)));
    int tot = n;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (lane == 0) cx.nitems = tot;
  }
  // 2nd-order codes by (row mod rp, group) from the final chunk table
  const ChunkLayout& cl = a.cl;
  const int P256 = cl.period * kGroup2;
  for (int e = tid; e < rp * kTileGroups; e += blockDim.x) {
    const int rho = e >> 3, gw = e & 7;
    const int64_t gg = (int64_t)ct * kTileGroups + gw;
    uint8_t q = 0;
    if (gg < ng) {
      const int u = (int)(((int64_t)rho * ng + gg) % P256);
      const float4 ch = a.ws.chunk_tab[min(u >> 8, cl.ntab_full)];
      const float s1f =
          __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(&cx.shv)[gw]));
      const int q2 = f2i_rz(roundf(__fdiv_rn(__fsub_rn(s1f, ch.x), ch.y)));
      q = (uint8_t)max(0, min(15, q2));
    }
    cx.sqrow[rho][gw] = q;
  }
  __syncthreads();
}

// 2nd-order code of scales_1st[r, g] (quantize.cu:274-280) computed directly.
__device__ __forceinline__ uint8_t sq_direct(const QArgs& a, float s1f, int64_t r, int64_t g) {
  const ChunkLayout& cl = a.cl;
  const int64_t si = r * a.ng + g;
  const int idx = si < cl.nfull * kGroup2 ? (int)((si % ((int64_t)cl.period * kGroup2)) >> 8)
                                          : cl.ntab_full;
  const float4 ch = a.ws.chunk_tab[idx];
  const int q2 = f2i_rz(roundf(__fdiv_rn(__fsub_rn(s1f, ch.x), ch.y)));
  return (uint8_t)max(0, min(15, q2));
}

__global__ void __launch_bounds__(kEncThreads, 2)
    encode_kernel(const __grid_constant__ CUtensorMap tmap, const QArgs a, int use_tma,
                  int vec_out) {
  extern __shared__ uint8_t dsm_raw[];
  // 1024-byte aligned for the 128-byte swizzle; offset arithmetic on the
  // shared array keeps the pointer in the shared space (plain LDS)
  uint8_t* dsm = dsm_raw + ((1024u - (smem_u32(dsm_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full[kEncStages];
  __shared__ EncCtx cx;
  __shared__ EncCodes cbuf[2];
  __shared__ int item_next[2];  // next item of the tiles using code buffer 0 / 1
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t M = a.M;
  const int ng = a.ng, nrc = a.nrc;
  // The CTA's tiles [S0, S1) come from the selection (weighted by work);
  // tile u = ct * nrc + rc, and (ct, rc) advance without divisions.
  struct Seq {
    int ct, rc;
  };
  auto seq_next = [&](Seq& q) {
    if (++q.rc == nrc) {
      q.rc = 0;
      ++q.ct;
    }
  };
  auto issue = [&](const Seq& q, int s) {
    uint8_t* dst = dsm + (size_t)s * kTileBytes;
    mbar_arrive_expect_tx(&full[s], kTileBytes);
    tma_load_2d(dst, &tmap, &full[s], q.ct * kTileCols, q.rc * kChunkRows);
    tma_load_2d(dst + kBoxBytes, &tmap, &full[s], q.ct * kTileCols + 64, q.rc * kChunkRows);
  };
  if (tid == 0 && use_tma) {
    for (int s = 0; s < kEncStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  if (tid < 2) item_next[tid] = 0;  // visible after the context's barriers
  grid_dependency_wait();  // the selection, parameters, 2nd-order table and ranges are final
  post_prologue(a, (int)blockIdx.x, (int)gridDim.x);
  // the tile range, clamped into the matrix whatever the split wrote
  const int64_t ntiles_all = (int64_t)a.nct * nrc;
  const int64_t S0 = max64(0, min64(ntiles_all, a.ws.enc_start[blockIdx.x]));
  const int64_t S1 = max64(S0, min64(ntiles_all, a.ws.enc_start[blockIdx.x + 1]));
  const int64_t ntile_cta = S1 - S0;
  Seq ahead{(int)(S0 / nrc), (int)(S0 % nrc)};  // thread 0: the next tile to load
  if (tid == 0 && use_tma)
    for (int s = 0; s < kEncStages && s < ntile_cta; ++s) {
      issue(ahead, s);
      seq_next(ahead);
    }
  const int P256 = a.cl.period * kGroup2;
  const int rp = P256 / ng;  // a power of two, at most 256
  const int64_t row_full_end = a.cl.nfull * kGroup2;
  const int64_t full_rows = row_full_end / ng;  // rows whose scales lie in full 2nd-order chunks
  // write-out offsets of thread tid < 256 in a full tile (elements / words
  // from the tile's first output): packed_2bit row tid/2, half tid%2;
  // packed_4bit rows tid/4 and tid/4 + 64, quarter tid%4 (the per-row arrays
  // go to the threads from kRowWriter0)
  const int wo_r2 = tid >> 1, wo_h2 = tid & 1;
  const int64_t wo_o2 = (int64_t)wo_r2 * ng + 4 * wo_h2;
  const int wo_r4 = tid >> 2, wo_q4 = tid & 3;
  const int64_t wo_o4 = 2 * (int64_t)wo_r4 * ng + 4 * wo_q4;
  bool failed = false;
  uint32_t bad = 0;  // thread 0: stages whose wait ran out
  int cur_ct = -1;
  Seq cur{(int)(S0 / nrc), (int)(S0 % nrc)};
  for (int64_t i = 0; i < ntile_cta; ++i, seq_next(cur)) {
    const int ct = cur.ct, rc = cur.rc;
    const int s = (int)(i & 1);
    if (ct != cur_ct) {
      if (cur_ct >= 0) __syncthreads();  // the previous write-out is done with the context
      enc_build_ctx(a, cx, ct, rp);
      cur_ct = ct;
    }
    uint8_t* buf = dsm + (size_t)s * kTileBytes;
    if (use_tma) {
      const bool ok = mbar_wait(&full[s], (uint32_t)((i >> 1) & 1));
      failed |= !ok;
      if (tid == 0 && !ok) bad |= 1u << s;
    } else {
      tile_fill(a.W, M, a.K, buf, (int64_t)rc * a.nct + ct, a.nct, 0);
      __syncthreads();
    }
    const int64_t row0 = (int64_t)rc * kChunkRows;
    const int nr = (int)min64(kChunkRows, M - row0);
    EncCodes& cb = cbuf[i & 1];
    const int nitems = cx.nitems;
    int* next_item = &item_next[i & 1];
    int grab = lane == 0 ? atomicAdd(next_item, 1) : 0;
#pragma unroll 1
    for (;;) {
      const int j = __shfl_sync(0xffffffffu, grab, 0);
      if (j >= nitems) break;
      if (lane == 0) grab = atomicAdd(next_item, 1);  // the next item, in flight meanwhile
      const int it = cx.items[j];
      const int gw = it & 7, st = (it >> 3) & 3;
      if (st * 32 >= nr) continue;
      const int r0 = st * 32 + lane;  // rows r0 (and r0 + 32 for 2-bit; same swizzle phase)
      const uint8_t* rb = buf + (gw >> 2) * kBoxBytes + r0 * 128;
      const int c0 = 2 * (gw & 3), sw = lane & 7;
      const int lo_off = (c0 ^ sw) << 4, hi_off = ((c0 + 1) ^ sw) << 4;
      auto run_at = [&](int h) {
        Row16 v;
        v.lo = *reinterpret_cast<const uint4*>(rb + 32 * 128 * h + lo_off);
        v.hi = *reinterpret_cast<const uint4*>(rb + 32 * 128 * h + hi_off);
        return v;
      };
      const int kind = cx.kind[gw];
      const int gs = cx.gs[gw];
      if (kind == kEncKind2) {
        const Row16 v0 = run_at(0), v1 = run_at(1);
        const uint4 T = cx.thr[gw][0];
        uint32_t w0 = enc2_run(v0, T.x, T.y, T.z), w1 = enc2_run(v1, T.x, T.y, T.z);
        if (gs < kGroup1) {  // columns past K hold code 0
          w0 &= (1u << (2 * gs)) - 1u;
          w1 &= (1u << (2 * gs)) - 1u;
        }
        cb.p2[gw][r0] = w0;
        cb.p2[gw][r0 + 32] = w1;
        cb.p4[gw][r0] = make_uint2(0u, 0u);
        cb.p4[gw][r0 + 32] = make_uint2(0u, 0u);
      } else if (kind == kEncKind4) {
        uint32_t t[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 T = cx.thr[gw][q];
          t[4 * q] = T.x;
          t[4 * q + 1] = T.y;
          t[4 * q + 2] = T.z;
          t[4 * q + 3] = T.w;
        }
        const uint32_t ma = gs >= 8 ? 0xFFFFFFFFu : ((1u << (4 * gs)) - 1u);
        const uint32_t mb = gs <= 8 ? 0u : gs >= 16 ? 0xFFFFFFFFu : ((1u << (4 * (gs - 8))) - 1u);
        uint2 c;
        enc4_run(run_at(0), t, c.x, c.y);
        cb.p2[gw][r0] = 0u;
        cb.p4[gw][r0] = make_uint2(c.x & ma, c.y & mb);  // columns past K: code 0
      } else {
        const int64_t g = (int64_t)ct * kTileGroups + gw;
        const GroupParams& gp = a.ws.params[2 * g + cx.pr[gw]];
        const bool four = cx.pr[gw] != 0;
        const uint3 c = enc_irregular(gp, rb, lo_off, hi_off, gs);
        if (c.z && r0 < nr) atomicAdd(a.ws.row_counts + row0 + r0, (int)c.z);
        cb.p2[gw][r0] = four ? 0u : c.x;
        cb.p4[gw][r0] = four ? make_uint2(c.x, c.y) : make_uint2(0u, 0u);
      }
    }
    __syncthreads();  // codes staged; the tile buffer is free
    if (tid == 32) item_next[i & 1] = 0;  // its next user starts after the next barrier
    if (tid == 0 && use_tma && i + kEncStages < ntile_cta) {
      fence_proxy_async_smem();
      issue(ahead, s);
      seq_next(ahead);
    }
    const int gb = ct * kTileGroups;
    const int64_t obase = row0 * ng + gb;  // flat index of (row0, gb)
    if (vec_out && gb + kTileGroups <= ng && nr == kChunkRows && row0 + kChunkRows <= full_rows) {
      // a full tile: fixed trip counts, per-thread offsets from the prologue
      if (tid < 256) {
        const uint4 x2 = make_uint4(cb.p2[wo_h2 * 4][wo_r2], cb.p2[wo_h2 * 4 + 1][wo_r2],
                                    cb.p2[wo_h2 * 4 + 2][wo_r2], cb.p2[wo_h2 * 4 + 3][wo_r2]);
        *reinterpret_cast<uint4*>(a.packed2 + obase + wo_o2) = x2;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int r = wo_r4 + 64 * k;
          const uint2 x = cb.p4[2 * wo_q4][r], y = cb.p4[2 * wo_q4 + 1][r];
          *reinterpret_cast<uint4*>(a.packed4 + 2 * obase + wo_o4 + (int64_t)k * 128 * ng) =
              make_uint4(x.x, x.y, y.x, y.y);
        }
      }
      if (tid >= kRowWriter0 && tid < kRowWriter0 + kRowWriters) {
        for (int r = tid - kRowWriter0; r < kChunkRows; r += kRowWriters) {
          const int64_t o = obase + (int64_t)r * ng;
          *reinterpret_cast<uint4*>(a.scales1 + o) = cx.shv;
          *reinterpret_cast<uint2*>(a.zeros1 + o) = cx.zv;
          *reinterpret_cast<uint2*>(a.sq + o) =
              *reinterpret_cast<const uint2*>(&cx.sqrow[(rc * kChunkRows + r) & (rp - 1)][0]);
        }
      }
    } else if (vec_out && gb + kTileGroups <= ng) {
      for (int k = tid; k < nr * 2; k += blockDim.x) {
        const int r = k >> 1, h = k & 1;
        const uint4 x = make_uint4(cb.p2[4 * h][r], cb.p2[4 * h + 1][r], cb.p2[4 * h + 2][r],
                                   cb.p2[4 * h + 3][r]);
        reinterpret_cast<uint4*>(a.packed2 + obase + r * ng)[h] = x;
      }
      for (int k = tid; k < nr * 4; k += blockDim.x) {
        const int r = k >> 2, q = k & 3;
        const uint2 x = cb.p4[2 * q][r], y = cb.p4[2 * q + 1][r];
        reinterpret_cast<uint4*>(a.packed4 + 2 * (obase + r * ng))[q] =
            make_uint4(x.x, x.y, y.x, y.y);
      }
      const uint4 shv = cx.shv;
      const uint2 zv = cx.zv;
      // rows before nfast take their 2nd-order codes from the table
      const int nfast = (int)max64(0, min64(nr, full_rows - row0));
      for (int r = tid; r < nr; r += blockDim.x) {
        const int64_t o = obase + r * ng;
        *reinterpret_cast<uint4*>(a.scales1 + o) = shv;
        *reinterpret_cast<uint2*>(a.zeros1 + o) = zv;
        uint2 q;
        if (r < nfast) {
          q = *reinterpret_cast<const uint2*>(&cx.sqrow[(rc * kChunkRows + r) & (rp - 1)][0]);
        } else {
          uint8_t b[kTileGroups];
#pragma unroll
          for (int w = 0; w < kTileGroups; ++w)
            b[w] = sq_direct(a, __half2float(__ushort_as_half(
                                    reinterpret_cast<const uint16_t*>(&cx.shv)[w])),
                             row0 + r, gb + w);
          q.x = b[0] | (b[1] << 8) | (b[2] << 16) | ((uint32_t)b[3] << 24);
          q.y = b[4] | (b[5] << 8) | (b[6] << 16) | ((uint32_t)b[7] << 24);
        }
        *reinterpret_cast<uint2*>(a.sq + o) = q;
      }
    } else {
      for (int k = tid; k < nr * kTileGroups; k += blockDim.x) {
        const int r = k >> 3, w = k & 7;
        const int g = gb + w;
        if (g >= ng) continue;
        const int64_t row = row0 + r;
        const int64_t si = row * ng + g;
        a.packed2[si] = (int32_t)cb.p2[w][r];
        reinterpret_cast<uint2*>(a.packed4)[si] = cb.p4[w][r];
        const uint16_t shb = reinterpret_cast<const uint16_t*>(&cx.shv)[w];
        a.scales1[si] = __ushort_as_half(shb);
        a.zeros1[si] = reinterpret_cast<const int8_t*>(&cx.zv)[w];
        a.sq[si] = (row + 1) * ng <= row_full_end
                       ? cx.sqrow[row & (rp - 1)][w]
                       : sq_direct(a, __half2float(__ushort_as_half(shb)), row, g);
      }
    }
  }
  grid_launch_dependents();
  failed = __syncthreads_or(failed) != 0;
  if (tid == 0) {
    if (failed) atomicOr(&a.ws.hdr->status, kStatusTimeout);
    // loads whose wait ran out may still be in flight: let them land
    for (int s = 0; s < kEncStages; ++s)
      if (bad & (1u << s)) (void)mbar_wait(&full[s], 0u), (void)mbar_wait(&full[s], 1u);
  }
  post_rowptr_scan<kEncThreads>(a, (int)gridDim.x, reinterpret_cast<long long*>(dsm));
}


// scales_1st, zeros_1st and scales_1st_quant of rows [M b / G, M (b + 1) / G)
// (CTA b of G), each a contiguous stretch of its array written with 16-byte
// stores.  scales_1st and zeros_1st are the same in every row (the column
// group's parameters); the 2nd-order code of (r, g) takes the chunk table
// entry of its flat index r ng + g (quantize.cu:245-272), which for rows in
// full chunks repeats every rp = 256 / gcd(ng, 256) rows: those rows copy
// one of the rp pattern rows the tables kernel wrote once per matrix (each
// CTA computing them, rp * ng codes, had cost the 4096x11008 encode ~5 M
// warp instructions), the rows of the partial chunk compute theirs.  Needs
// ng % 16 == 0 and 16-byte aligned arrays; `scratch` is shared memory the CTA
// no longer needs (3 ng bytes).
__device__ __noinline__ void fill_row_arrays(const QArgs& a, int bid, int G, uint8_t* scratch,
                                             size_t scratch_bytes) {
  const int ng = a.ng, tid = threadIdx.x, nt = blockDim.x;
  const int64_t r0 = a.M * bid / G, r1 = a.M * (bid + 1) / G;
  uint16_t* sc = reinterpret_cast<uint16_t*>(scratch);  // [ng] fp16 bits
  int8_t* zr = reinterpret_cast<int8_t*>(scratch + 2 * ng);
  (void)scratch_bytes;  // 3 ng bytes are used
  const int rp = (int)((int64_t)a.cl.period * kGroup2 / ng);
  const int64_t full_rows = a.cl.nfull * kGroup2 / ng;  // rows whose scales lie in full chunks
  for (int g = tid; g < ng; g += nt) {
    const GroupParams& p = a.ws.params[2 * g + a.ws.prec[g]];
    sc[g] = (uint16_t)p.scale_h;
    zr[g] = (int8_t)p.zero;
  }
  __syncthreads();
  const int n = (int)((r1 - r0) * ng);  // elements of the CTA's stretch (below 2^31)
  const int64_t e0 = r0 * ng;
  uint4* sc_out = reinterpret_cast<uint4*>(a.scales1 + e0);
  for (int j = tid; j < n / 8; j += nt)
    sc_out[j] = *reinterpret_cast<const uint4*>(sc + (j * 8) % ng);
  uint4* z_out = reinterpret_cast<uint4*>(a.zeros1 + e0);
  uint4* q_out = reinterpret_cast<uint4*>(a.sq + e0);
  for (int j = tid; j < n / 16; j += nt) {
    const int l = j * 16, rl = l / ng, g = l - rl * ng;
    z_out[j] = *reinterpret_cast<const uint4*>(zr + g);
    const int64_t r = r0 + rl;
    uint4 q;
    if (r < full_rows) {
      // row r's codes are those of row r mod rp of the period: the tables
      // kernel's per-chunk codes in flat order
      q = __ldg(reinterpret_cast<const uint4*>(a.ws.sq_pat + (int)(r % rp) * ng + g));
    } else {
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int k = 0; k < 16; ++k)
        w[k >> 2] |= (uint32_t)sq_direct(a, __half2float(__ushort_as_half(sc[g + k])), r, g + k)
                     << (8 * (k & 3));
      q = make_uint4(w[0], w[1], w[2], w[3]);
    }
    q_out[j] = q;
  }
}

// ---------------------------------------------------------------------------
// encode, wide-tile form: tiles of 128 rows x 256 columns (16 groups), lane =
// row, packed words written whole by TMA.  Compute warp w takes the 32 rows
// [32 (w & 3), 32 (w & 3) + 32) of the tile and four of its groups, the
// quarter ((w >> 2) + i) & 3 on the CTA's i-th tile, so every warp carries
// the same mix of 2-bit / 4-bit groups over any four tiles and no work queue
// is needed.  A lane codes its row's four runs in registers (straight-line
// code per 2/4-bit pattern of the quarter) and writes the words to a staging
// tile laid out as the output rows (packed_2bit with the 64-byte swizzle,
// packed_4bit with the 128-byte swizzle: conflict-free).  The per-row arrays
// (scales_1st, zeros_1st, 2nd-order codes: 16 or 32 bytes per row and tile,
// too narrow for efficient stores) are written after the tiles, row by row
// (fill_row_arrays).
//
// Warp specialisation: the 16 compute warps never wait on one another inside
// the tile loop.  A producer warp (warp 16, one thread) issues the TMA loads
// of a three-stage tile ring and the two TMA stores of each staged tile, and
// hands buffers over through mbarriers: full[s] (tile landed), empty[s]
// (16 warps done reading it), stg_full (16 warps wrote the staging tile),
// stg_empty (the stores have read it).  A warp codes tile i + 1 in registers
// while tile i's stores drain.  Needs ng % 16 == 0 and 16-byte aligned
// outputs; other shapes take encode_kernel.  CTA b takes the tiles
// [floor(b T / G), floor((b + 1) T / G)) of the T tiles in column-major order.
// ---------------------------------------------------------------------------
constexpr int kE3Cols = 256;
constexpr int kE3Groups = kE3Cols / kGroup1;        // 16
constexpr int kE3Compute = 512;                     // 16 compute warps
constexpr int kE3Threads = kE3Compute + 32;         // + the producer warp
constexpr int kE3Stages = 3;
constexpr int kE3Tile = kChunkRows * kE3Cols * 2;   // 64 KB: four 64-column boxes
constexpr int kE3P2 = kChunkRows * 64;              // 128 rows x 16 words
constexpr int kE3P4 = kChunkRows * 128;             // 128 rows x 32 words
constexpr int kE3Out = kE3P2 + kE3P4;               // the staging buffer: 24 KB
constexpr int kE3OffOut = kE3Stages * kE3Tile;
constexpr int kE3Smem = kE3OffOut + kE3Out + 1024;  // + alignment slack
static_assert(kE3OffOut % 1024 == 0 && kE3Out % 1024 == 0 && kE3P2 % 1024 == 0,
              "staging alignment");

struct __align__(16) Enc3Ctx {
  uint4 thr[kE3Groups][4];                    // T_1..T_15 as broadcast half2, +inf pad
  uint8_t kind[kE3Groups];
  uint8_t gs[kE3Groups];
  uint8_t pr[kE3Groups];
};

struct Enc3Maps {
  CUtensorMap p2, p4;  // packed_2bit (box 128 x 16, 64B swizzle), packed_4bit (128 x 32,
                       // 128B swizzle)
};

// Barrier among the compute warps only (named barrier 1).
__device__ __forceinline__ void enc3_compute_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kE3Compute) : "memory");
}

// Codes of one row's four runs of a quarter whose groups are all regular and
// 16 columns wide; bit q of P: group q of the quarter is 4-bit.  The run of
// group q lies at chunks 2q, 2q + 1 of the row in its 64-column box.
template <int P>
__device__ __forceinline__ void enc3_quarter(const uint8_t* __restrict__ rb, int sw,
                                             const uint4 (*__restrict__ thr)[4],
                                             uint32_t (&w2)[4], uint32_t (&w4)[8]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    Row16 v;
    v.lo = *reinterpret_cast<const uint4*>(rb + (((2 * q) ^ sw) << 4));
    v.hi = *reinterpret_cast<const uint4*>(rb + (((2 * q + 1) ^ sw) << 4));
    if ((P >> q) & 1) {
      uint32_t t[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint4 T = thr[q][k];
        t[4 * k] = T.x;
        t[4 * k + 1] = T.y;
        t[4 * k + 2] = T.z;
        t[4 * k + 3] = T.w;
      }
      enc4_run(v, t, w4[2 * q], w4[2 * q + 1]);
      w2[q] = 0u;
    } else {
      const uint4 T = thr[q][0];
      w2[q] = enc2_run(v, T.x, T.y, T.z);
      w4[2 * q] = w4[2 * q + 1] = 0u;
    }
  }
}

// The producer: TMA loads into the ring, TMA stores of each staged tile.
// One thread.  Returns false if a wait ran out (it then stops issuing).
__device__ __forceinline__ bool enc3_producer(const CUtensorMap& tmap, const Enc3Maps& om,
                                              uint8_t* dsm, uint64_t* full, uint64_t* empty,
                                              uint64_t* stg_full, uint64_t* stg_empty,
                                              int64_t S0, int64_t n, int nrc, int use_tma,
                                              uint32_t& issued_mask) {
  int l_ct = (int)(S0 / nrc), l_rc = (int)(S0 % nrc);  // the next tile to load
  int s_ct = l_ct, s_rc = l_rc;                        // the next tile to store
  const uint64_t pol_in = l2_evict_first(), pol_out = l2_evict_first();
  auto issue = [&](int s) {
    uint8_t* dst = dsm + (size_t)s * kE3Tile;
    mbar_arrive_expect_tx(&full[s], kE3Tile);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      tma_load_2d_hint(dst + j * kBoxBytes, &tmap, &full[s], l_ct * kE3Cols + 64 * j,
                       l_rc * kChunkRows, pol_in);
    issued_mask |= 1u << s;
    if (++l_rc == nrc) {
      l_rc = 0;
      ++l_ct;
    }
  };
  if (use_tma)
    for (int s = 0; s < kE3Stages && s < n; ++s) issue(s);
  uint8_t* s2 = dsm + kE3OffOut;
  uint8_t* s4 = s2 + kE3P2;
  for (int64_t i = 0; i < n; ++i) {
    // the warps release tile i's stage before they write its staging tile:
    // the refill goes out first
    if (use_tma && i + kE3Stages < n) {
      const int s = (int)(i % kE3Stages);
      if (!mbar_wait(&empty[s], (uint32_t)((i / kE3Stages) & 1))) return false;
      fence_proxy_async_smem();
      issue(s);
    }
    if (!mbar_wait(stg_full, (uint32_t)(i & 1))) return false;
    const int x = s_ct * kE3Groups, y = s_rc * kChunkRows;
    tma_store_2d_hint(&om.p2, s2, x, y, pol_out);
    tma_store_2d_hint(&om.p4, s4, 2 * x, y, pol_out);
    bulk_commit();
    if (++s_rc == nrc) {
      s_rc = 0;
      ++s_ct;
    }
    bulk_wait_read<0>();  // the staging tile is read: the warps may refill it
    mbar_arrive(stg_empty);
  }
  return true;
}

__device__ __forceinline__ void encode3_body(const CUtensorMap& tmap, const Enc3Maps& om,
                                             const QArgs& a, int use_tma, int bid, int G) {
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = dsm_raw + ((1024u - (smem_u32(dsm_raw) & 1023u)) & 1023u);
  __shared__ uint64_t full[kE3Stages], empty[kE3Stages], stg_bar[2];
  __shared__ Enc3Ctx cxs[2];  // contexts of consecutive column tiles
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t M = a.M;
  const int ng = a.ng, nrc = a.nrc;
  const int nct3 = ng / kE3Groups;
  if (tid == 0) {
    for (int s = 0; s < kE3Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kE3Compute / 32);
    }
    mbar_init(&stg_bar[0], kE3Compute / 32);  // stg_full: the 16 warps wrote the staging tile
    mbar_init(&stg_bar[1], 1);                // stg_empty: the stores have read it
    fence_mbar_init();
  }
  grid_dependency_wait();  // the selection, parameters and 2nd-order table are final
  post_prologue(a, bid, G);
  const int64_t ntiles = (int64_t)nct3 * nrc;
  const int64_t S0 = ntiles * bid / G, S1 = ntiles * (bid + 1) / G;
  const int64_t ntile_cta = S1 - S0;
  __syncthreads();  // barrier initialisation visible
  bool failed = false;
  uint32_t issued = 0;  // producer: stages that received a load
  if (warp == kE3Compute / 32) {
    if (lane == 0)
      failed = !enc3_producer(tmap, om, dsm, full, empty, &stg_bar[0], &stg_bar[1], S0,
                              ntile_cta, nrc, use_tma, issued);
  } else {
    const int slab = warp & 3, qsel = warp >> 2;
    const int rr = slab * 32 + lane;  // this lane's row in the tile
    const int sw = rr & 7;            // its 128-byte swizzle phase
    uint8_t* s2 = dsm + kE3OffOut;
    uint8_t* s4 = s2 + kE3P2;
    int cur_ct = -1, pats = 0;  // pats: the 4 quarters' patterns, 5 bits each
    const Enc3Ctx* cx = &cxs[0];
    int ct = (int)(S0 / nrc), rc = (int)(S0 % nrc);
    for (int64_t i = 0; i < ntile_cta; ++i) {
      const int s = (int)(i % kE3Stages);
      const uint32_t ph = (uint32_t)((i / kE3Stages) & 1);
      if (ct != cur_ct) {
        // a new column tile: its context goes to the other slot (before the
        // last barrier every warp finished the tiles of the column tile
        // that used it); warp w builds group w
        Enc3Ctx* nx = &cxs[ct & 1];
        const int64_t g = (int64_t)ct * kE3Groups + warp;
        uint32_t t = 0x7C007C00u;  // +inf: never reached
        int kind = kEncKindNone, pr = 0, gs = 0;
        if (g < ng) {
          pr = a.ws.prec[g];
          const GroupParams& p = a.ws.params[2 * g + pr];
          if (lane < 15) t = (uint32_t)p.thresh[lane] * 0x00010001u;
          kind = (p.flags & kFlagRegular) ? (pr ? kEncKind4 : kEncKind2) : kEncKindIrr;
          gs = (int)min64(kGroup1, a.K - g * kGroup1);
        }
        if (lane < 16) (&nx->thr[warp][0].x)[lane] = t;
        if (lane == 0) {
          nx->kind[warp] = (uint8_t)kind;
          nx->gs[warp] = (uint8_t)gs;
          nx->pr[warp] = (uint8_t)pr;
        }
        enc3_compute_sync();
        int pat = 0;
        if (lane < 4) {
          for (int q = 0; q < 4; ++q) {
            const int gi = 4 * lane + q;
            const int kd = nx->kind[gi];
            if (nx->gs[gi] != kGroup1 || (kd != kEncKind2 && kd != kEncKind4)) pat = 16;
            if (pat < 16 && kd == kEncKind4) pat |= 1 << q;
          }
        }
        pats = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) pats |= __shfl_sync(0xffffffffu, pat, q) << (5 * q);
        cx = nx;
        cur_ct = ct;
      }
      uint8_t* buf = dsm + (size_t)s * kE3Tile;
      if (use_tma) {
        // after a wait ran out the thread stops waiting (outputs are flagged
        // invalid), so a failed pipeline ends in bounded time
        if (!failed && !mbar_wait(&full[s], ph)) failed = true;
      } else {
        enc3_compute_sync();  // every compute warp is done with the stage
        for (int j = 0; j < 2; ++j) {
          uint8_t* dst = buf + j * kTileBytes;
          for (int e = tid; e < kChunkRows * kTileCols; e += kE3Compute) {
            const int r = e / kTileCols, c = e % kTileCols;
            const int64_t gr = (int64_t)rc * kChunkRows + r,
                          gc = (2 * (int64_t)ct + j) * kTileCols + c;
            const uint16_t v = (gr < M && gc < a.K) ? __half_as_ushort(a.W[gr * a.K + gc]) : 0;
            const int half = c >> 6, cc = c & 63;
            *reinterpret_cast<uint16_t*>(dst + half * kBoxBytes + r * 128 +
                                         (((cc >> 3) ^ (r & 7)) << 4) + (cc & 7) * 2) = v;
          }
        }
        enc3_compute_sync();
      }
      const int64_t row0 = (int64_t)rc * kChunkRows;
      const int qq = (qsel + (int)(i & 3)) & 3;  // this warp's quarter of the tile
      // codes of this lane's row, groups 4 qq .. 4 qq + 3 (box qq of the tile)
      const uint8_t* rb = buf + qq * kBoxBytes + rr * 128;
      uint32_t w2[4], w4[8];
      uint32_t cnt = 0;
      const uint4(*thr)[4] = &cx->thr[4 * qq];
      switch ((pats >> (5 * qq)) & 31) {
#define MB_ENC3_CASE(P) \
  case P:               \
    enc3_quarter<P>(rb, sw, thr, w2, w4); \
    break;
        MB_ENC3_CASE(0) MB_ENC3_CASE(1) MB_ENC3_CASE(2) MB_ENC3_CASE(3)
        MB_ENC3_CASE(4) MB_ENC3_CASE(5) MB_ENC3_CASE(6) MB_ENC3_CASE(7)
        MB_ENC3_CASE(8) MB_ENC3_CASE(9) MB_ENC3_CASE(10) MB_ENC3_CASE(11)
        MB_ENC3_CASE(12) MB_ENC3_CASE(13) MB_ENC3_CASE(14) MB_ENC3_CASE(15)
#undef MB_ENC3_CASE
        default:
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int gi = 4 * qq + q;
            const int kind = cx->kind[gi];
            const int lo_off = ((2 * q) ^ sw) << 4, hi_off = ((2 * q + 1) ^ sw) << 4;
            w2[q] = 0u;
            w4[2 * q] = w4[2 * q + 1] = 0u;
            if (kind == kEncKind2) {
              Row16 v;
              v.lo = *reinterpret_cast<const uint4*>(rb + lo_off);
              v.hi = *reinterpret_cast<const uint4*>(rb + hi_off);
              const uint4 T = cx->thr[gi][0];
              uint32_t w = enc2_run(v, T.x, T.y, T.z);
              const int gs = cx->gs[gi];
              if (gs < kGroup1) w &= (1u << (2 * gs)) - 1u;  // columns past K hold code 0
              w2[q] = w;
            } else if (kind == kEncKind4) {
              Row16 v;
              v.lo = *reinterpret_cast<const uint4*>(rb + lo_off);
              v.hi = *reinterpret_cast<const uint4*>(rb + hi_off);
              uint32_t t[16];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint4 T = cx->thr[gi][k];
                t[4 * k] = T.x;
                t[4 * k + 1] = T.y;
                t[4 * k + 2] = T.z;
                t[4 * k + 3] = T.w;
              }
              uint32_t x, y;
              enc4_run(v, t, x, y);
              const int gs = cx->gs[gi];
              if (gs < kGroup1) {
                x &= gs >= 8 ? 0xFFFFFFFFu : ((1u << (4 * gs)) - 1u);
                y &= gs <= 8 ? 0u : ((1u << (4 * (gs - 8))) - 1u);
              }
              w4[2 * q] = x;
              w4[2 * q + 1] = y;
            } else if (kind == kEncKindIrr) {
              const int64_t g = (int64_t)ct * kE3Groups + gi;
              const GroupParams& gp = a.ws.params[2 * g + cx->pr[gi]];
              const uint3 c = enc_irregular(gp, rb, lo_off, hi_off, cx->gs[gi]);
              if (cx->pr[gi]) {
                w4[2 * q] = c.x;
                w4[2 * q + 1] = c.y;
              } else {
                w2[q] = c.x;
              }
              cnt += c.z;
            }
          }
      }
      // this warp is done reading the stage
      __syncwarp();
      if (lane == 0 && use_tma) mbar_arrive(&empty[s]);
      const int64_t row = row0 + rr;
      if (cnt && row < M) atomicAdd(a.ws.row_counts + row, (int)cnt);
      // the staging tile: the previous tile's stores have read it
      if (i > 0 && !failed && !mbar_wait(&stg_bar[1], (uint32_t)((i - 1) & 1))) failed = true;
      *reinterpret_cast<uint4*>(s2 + rr * 64 + ((qq ^ ((rr >> 1) & 3)) << 4)) =
          make_uint4(w2[0], w2[1], w2[2], w2[3]);
      *reinterpret_cast<uint4*>(s4 + rr * 128 + (((2 * qq) ^ sw) << 4)) =
          make_uint4(w4[0], w4[1], w4[2], w4[3]);
      *reinterpret_cast<uint4*>(s4 + rr * 128 + (((2 * qq + 1) ^ sw) << 4)) =
          make_uint4(w4[4], w4[5], w4[6], w4[7]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&stg_bar[0]);
      if (++rc == nrc) {
        rc = 0;
        ++ct;
      }
    }
  }
  grid_launch_dependents();
  if (warp == kE3Compute / 32 && lane == 0) bulk_wait<0>();  // the CTA's stores are complete
  failed = __syncthreads_or(failed) != 0;
  if (tid == kE3Compute && failed) {
    atomicOr(&a.ws.hdr->status, kStatusTimeout);
    // loads still in flight land before the shared memory is reused
    for (int s = 0; s < kE3Stages; ++s)
      if (issued & (1u << s)) (void)mbar_wait(&full[s], 0u), (void)mbar_wait(&full[s], 1u);
  }
  __syncthreads();
  // the tiles and the staging buffer are free: the per-row arrays
  fill_row_arrays(a, bid, G, dsm, (size_t)(kE3Smem - 1024));
  post_rowptr_scan<kE3Threads>(a, G, reinterpret_cast<long long*>(dsm));
}

template <int NB>
struct __align__(64) Enc3Batch {
  CUtensorMap tmap[NB];
  Enc3Maps om[NB];
  QArgs a[NB];
  int use_tma[NB];
  BatchMap<NB> bm;
};

template <int NB>
__global__ void __launch_bounds__(kE3Threads, 1)
    encode3_kernel(const __grid_constant__ Enc3Batch<NB> P) {
  const CtaSlot c = batch_slot(P.bm);
  encode3_body(P.tmap[c.m], P.om[c.m], P.a[c.m], P.use_tma[c.m], c.b, c.G);
}


// extract: one warp per row with outliers; only non-regular groups can hold
// them.  Lanes 0-15 take the group's 16 columns; the ballot order is the
// column order.
__device__ __forceinline__ void extract_row(const __half* __restrict__ W, int64_t r, int64_t K,
                                            int ng, const GroupParams* __restrict__ params,
                                            const uint8_t* __restrict__ prec,
                                            const int32_t* __restrict__ row_ptrs,
                                            __half* __restrict__ vals, int32_t* __restrict__ cols,
                                            int fma_mode, int lane) {
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

__global__ void __launch_bounds__(256)
    extract_kernel(const __half* __restrict__ W, int64_t M, int64_t K, int ng,
                   const GroupParams* __restrict__ params, const uint8_t* __restrict__ prec,
                   const int32_t* __restrict__ row_ptrs, __half* __restrict__ vals,
                   int32_t* __restrict__ cols, int fma_mode) {
  const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (r >= M) return;
  extract_row(W, r, K, ng, params, prec, row_ptrs, vals, cols, fma_mode, threadIdx.x & 31);
}

// The CSR extraction chained to encode (programmatic dependent launch): the
// outlier count is read on the device, so no host round trip sits between
// the kernels (mb_quantize_csr).  Nothing to do without outliers; more
// outliers than `capacity` set kStatusCsrOverflow and write nothing.  Warps
// stride over the rows.
template <int NB>
struct CsrBatch {
  QArgs a[NB];
  int64_t capacity[NB];
  __half* vals[NB];
  int32_t* cols[NB];
  BatchMap<NB> bm;
};

template <int NB>
__global__ void __launch_bounds__(256) extract_cap_kernel(const __grid_constant__ CsrBatch<NB> P) {
  const CtaSlot c = batch_slot(P.bm);
  const QArgs& a = P.a[c.m];
  grid_dependency_wait();  // encode and its row-pointer scan complete
  const int32_t n = *reinterpret_cast<const volatile int32_t*>(a.nnz);
  if (n <= 0) return;
  if ((int64_t)n > P.capacity[c.m]) {
    if (c.b == 0 && threadIdx.x == 0) atomicOr(&a.ws.hdr->status, kStatusCsrOverflow);
    return;
  }
  const int64_t nw = (int64_t)c.G * (blockDim.x >> 5);
  for (int64_t r = ((int64_t)c.b * blockDim.x + threadIdx.x) >> 5; r < a.M; r += nw)
    extract_row(a.W, r, a.K, a.ng, a.ws.params, a.ws.prec, a.row_ptrs, P.vals[c.m],
                P.cols[c.m], kOutlierFma, threadIdx.x & 31);
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

// Everything a quantize call launches, prepared on the host: arguments,
// tensor maps and grids.
struct QuantizeLaunch {
  QArgs qa;
  CUtensorMap tmap;
  Enc3Maps omaps;
  bool tma, enc3, sens;
  int vec_out;
  int64_t stats_grid, comb_grid, enc_grid, enc3_grid;
  int64_t stats_full, enc3_full;  // every SM's resident CTAs (a batch's grids)
  size_t hdr_bytes;
};

int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return sms;
  static std::atomic<int> sm_cache[64];
  if (dev < 64 && sm_cache[dev].load(std::memory_order_acquire) > 0)
    return sm_cache[dev].load(std::memory_order_acquire);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
  if (dev < 64) sm_cache[dev].store(sms, std::memory_order_release);
  return sms;
}

// CTAs of encode_kernel (persistent: every CTA resident); the selection
// splits the tiles among them.
mb_status legacy_enc_grid(int64_t ntiles, int sms, int64_t* grid) {
  static std::atomic<int> occ[64];
  int per_sm = 1;
  MB_CUDA_TRY(blocks_per_sm_once(encode_kernel, kEncThreads, kEncSmem, occ, 64, &per_sm));
  *grid = std::max<int64_t>(
      1, std::min<int64_t>({ntiles, (int64_t)sms * std::max(per_sm, 1), (int64_t)kMaxEncGrid}));
  return MB_OK;
}

// Validation and set-up shared by mb_quantize and the row-split entry points.
// With stats_only the outputs are not needed (may be null).
mb_status quantize_prepare(const void* weights_fp16, int64_t M, int64_t K, double ratio_4bit,
                           const float* hessian_diag, int64_t hessian_numel, int32_t* packed_2bit,
                           int32_t* packed_4bit, void* scales_1st_fp16, int8_t* zeros_1st,
                           void* scales_2nd_fp16, int8_t* zeros_2nd, uint8_t* scales_1st_quant,
                           uint8_t* group_precision, int32_t* outlier_row_ptrs,
                           int32_t* nnz_device, void* workspace, size_t workspace_bytes,
                           bool stats_only, QuantizeLaunch& L) {
  if (mb_status st = check_common(weights_fp16, M, K)) return st;
  if (!stats_only)
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
  L.sens = selecting && n4 > 0;
  const bool w_aligned = (reinterpret_cast<uintptr_t>(weights_fp16) & 15u) == 0;
  L.hdr_bytes = sizeof(Header) + sizeof(uint32_t) * nct;

  QArgs& qa = L.qa;
  std::memset(&qa, 0, sizeof(qa));
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
  qa.select = L.sens;
  qa.w_aligned = w_aligned;
  qa.no_select = 0;
  qa.packed2 = packed_2bit;
  qa.packed4 = packed_4bit;
  qa.scales1 = static_cast<__half*>(scales_1st_fp16);
  qa.zeros1 = zeros_1st;
  qa.scales2 = static_cast<__half*>(scales_2nd_fp16);
  qa.zeros2 = zeros_2nd;
  qa.sq = scales_1st_quant;
  qa.row_ptrs = outlier_row_ptrs;
  qa.nnz = nnz_device;

  // TMA needs a 16-byte aligned base and a row pitch that is a multiple of 16
  // bytes; other inputs fill the same shared-memory layout with plain loads.
  std::memset(&L.tmap, 0, sizeof(L.tmap));
  L.tma = w_aligned && (K % 8 == 0) &&
          make_tensor_map_2d_16bit_sw128(&L.tmap, weights_fp16, false, (uint64_t)M, (uint64_t)K,
                                         kChunkRows, 64);
  const int sms = device_sms();
  const int64_t ntiles = nct * nrc;
  // the encode grid (persistent: every CTA resident), known to the selection,
  // which splits the tiles among its CTAs
  if (mb_status st = legacy_enc_grid(ntiles, sms, &L.enc_grid)) return st;
  qa.enc_grid = (int)L.enc_grid;
  {
    auto kern = L.sens ? stats_kernel<true, 1> : stats_kernel<false, 1>;
    static std::atomic<int> occ[2][64];
    int per_sm = 1;
    MB_CUDA_TRY(blocks_per_sm_once(kern, kStatsThreads, kStatsSmem, occ[L.sens ? 1 : 0], 64,
                                   &per_sm));
    // at most one CTA per tile (no empty tile range) and the records' cap
    L.stats_full = (int64_t)sms * std::max(per_sm, 1);
    L.stats_grid = std::max<int64_t>(1, std::min<int64_t>(stats_grid_cap(ntiles), L.stats_full));
  }
  qa.stats_grid = (int)L.stats_grid;
  qa.exact_thresholds = 0;
  L.comb_grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(ng, kCombThreads / 32), sms));
  {
    // the selection's scratch: keys when they do not fit in registers, then
    // the column tiles' encode costs and their prefix (small CTAs let other
    // matrices' kernels share the SMs)
    size_t need = (ng > (int64_t)kSelKPT * kCombThreads) ? (size_t)ng * 8 : 0;
    need = ((need + (size_t)nct * 4 + 7) & ~(size_t)7) + (size_t)(nct + 1) * 8 + 256;
    qa.comb_smem = (int)std::min<size_t>(need, (size_t)kCombSmem);
  }
  L.enc3 = false;
  L.enc3_grid = 1;
  L.enc3_full = sms;
  L.vec_out = 0;
  std::memset(&L.omaps, 0, sizeof(L.omaps));
  if (stats_only) return MB_OK;
  // the wide-tile encode with whole-tile TMA stores: ng % 16 == 0 and 16-byte
  // aligned outputs
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const uint64_t um = (uint64_t)M, ung = (uint64_t)ng;
  L.enc3 =
      (ng % kE3Groups == 0) && al16(packed_2bit) && al16(packed_4bit) &&
      al16(scales_1st_fp16) && al16(zeros_1st) && al16(scales_1st_quant) &&
      make_tensor_map_2d(&L.omaps.p2, packed_2bit, 4, um, ung, kChunkRows, 16, 64) &&
      make_tensor_map_2d(&L.omaps.p4, packed_4bit, 4, um, 2 * ung, kChunkRows, 32, 128);
  if (L.enc3) {
    static std::atomic<int> occ3[64];
    int per_sm = 1;
    MB_CUDA_TRY(blocks_per_sm_once(encode3_kernel<1>, kE3Threads, kE3Smem, occ3, 64, &per_sm));
    L.enc3_full = (int64_t)sms * std::max(per_sm, 1);
    L.enc3_grid = std::max<int64_t>(1, std::min<int64_t>((ng / kE3Groups) * nrc, L.enc3_full));
  }
  const auto al = [](const void* p, unsigned m) {
    return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0;
  };
  L.vec_out = (ng % 8 == 0) && al(packed_2bit, 16) && al(packed_4bit, 16) &&
              al(scales_1st_fp16, 16) && al(zeros_1st, 8) && al(scales_1st_quant, 8);
  return MB_OK;
}

// Grid shares of a batch: matrix i gets about total * w[i] / sum(w) CTAs, at
// least 1 and at most cap[i].
void split_grid(int n, const int64_t* w, const int64_t* cap, int64_t total, int64_t* out) {
  double sw = 0.0;
  for (int i = 0; i < n; ++i) sw += (double)w[i];
  for (int i = 0; i < n; ++i) {
    const int64_t g = (int64_t)std::llround((double)total * (double)w[i] / std::max(sw, 1.0));
    out[i] = std::max<int64_t>(1, std::min<int64_t>(g, cap[i]));
  }
}

template <int NB>
void fill_map(BatchMap<NB>& bm, int n, const int64_t* grid) {
  bm.n = n;
  bm.cta0[0] = 0;
  for (int i = 0; i < n; ++i) bm.cta0[i + 1] = bm.cta0[i] + (int)grid[i];
}

// The CSR arrays of mb_quantize_csr (one per matrix of a batch).
struct CsrOut {
  __half* vals;
  int32_t* cols;
  int64_t capacity;
};

// The header memsets, then one stats and one combine launch for n <= NB
// matrices (all with or all without the sensitivity pass).  One matrix keeps
// its own grids; in a batch the stats kernel's full grid is split by tile
// count and each matrix's combine keeps its grid.
template <int NB>
mb_status launch_stats_batch(QuantizeLaunch* const* Ls, int n, cudaStream_t stream) {
  const bool sens = Ls[0]->sens;
  int64_t sg[NB], cg[NB];
  if (n == 1) {
    sg[0] = Ls[0]->stats_grid;
  } else {
    int64_t w[NB], cap[NB];
    for (int i = 0; i < n; ++i) {
      w[i] = (int64_t)Ls[i]->qa.nct * Ls[i]->qa.nrc;
      cap[i] = stats_grid_cap(w[i]);
    }
    split_grid(n, w, cap, Ls[0]->stats_full, sg);
  }
  StatsBatch<NB> P;
  ArgsBatch<NB> C;
  std::memset(&P, 0, sizeof(P));
  std::memset(&C, 0, sizeof(C));
  int comb_smem = 0;
  for (int i = 0; i < n; ++i) {
    QuantizeLaunch& L = *Ls[i];
    L.qa.stats_grid = (int)sg[i];  // the segment records' layout
    MB_CUDA_TRY(cudaMemsetAsync(L.qa.ws.hdr, 0, L.hdr_bytes, stream));
    P.tmap[i] = L.tmap;
    P.a[i] = L.qa;
    P.use_tma[i] = L.tma ? 1 : 0;
    C.a[i] = L.qa;
    cg[i] = L.comb_grid;
    comb_smem = std::max(comb_smem, L.qa.comb_smem);
  }
  fill_map(P.bm, n, sg);
  fill_map(C.bm, n, cg);
  auto kern = sens ? stats_kernel<true, NB> : stats_kernel<false, NB>;
  static std::atomic<uint64_t> sattr[2];
  MB_CUDA_TRY(set_smem_limit_once(kern, kStatsSmem, sattr[sens ? 1 : 0]));
  kern<<<(unsigned)P.bm.cta0[n], kStatsThreads, kStatsSmem, stream>>>(P);
  MB_LAUNCH_CHECK("stats_kernel");
  auto comb = sens ? combine_kernel<true, NB> : combine_kernel<false, NB>;
  static std::atomic<uint64_t> cattr[2];
  MB_CUDA_TRY(set_smem_limit_once(comb, kCombSmem, cattr[sens ? 1 : 0]));
  return launch_pdl(comb, dim3((unsigned)C.bm.cta0[n]), dim3(kCombThreads), (size_t)comb_smem,
                    stream, C);
}

// The tables kernel for n <= NB matrices: a thread per group, a warp per
// distinct 2nd-order chunk.
template <int NB>
mb_status launch_tables(QuantizeLaunch* const* Ls, int n, cudaStream_t stream) {
  ArgsBatch<NB> T;
  std::memset(&T, 0, sizeof(T));
  int64_t tg[NB];
  for (int i = 0; i < n; ++i) {
    const QArgs& qa = Ls[i]->qa;
    T.a[i] = qa;
    const int64_t nchunks = qa.cl.ntab_full + qa.cl.has_partial;
    tg[i] = std::max<int64_t>(
        1, std::min<int64_t>(32, ceil_div(std::max<int64_t>(qa.ng, nchunks * 32), 256)));
  }
  fill_map(T.bm, n, tg);
  return launch_pdl(tables_kernel<NB>, dim3((unsigned)T.bm.cta0[n]), dim3(256), 0, stream, T);
}

// The exact-sum kernel, the tables, encode and (with csr) the CSR extraction
// for n <= NB matrices, chained with PDL.  A batch (n > 1) needs every
// matrix on the wide-tile encode; its full grid is split by tile count.
template <int NB>
mb_status launch_tables_encode_batch(QuantizeLaunch* const* Ls, int n, cudaStream_t stream,
                                     const CsrOut* csr) {
  ArgsBatch<NB> X;
  std::memset(&X, 0, sizeof(X));
  int64_t xg[NB];
  for (int i = 0; i < n; ++i) {
    X.a[i] = Ls[i]->qa;
    // one matrix: the whole GPU; in a batch enough warps for the chunk
    // programs of four pending groups at once
    xg[i] = n == 1 ? kExactCtas
                   : std::max<int64_t>(16, std::min<int64_t>(kExactCtas, (Ls[i]->qa.nrc + 1) / 2));
  }
  fill_map(X.bm, n, xg);
  if (mb_status st = launch_pdl(exact_kernel<NB>, dim3((unsigned)X.bm.cta0[n]), dim3(256), 0,
                                stream, X))
    return st;
  if (mb_status st = launch_tables<NB>(Ls, n, stream)) return st;
  if (n == 1 && !Ls[0]->enc3) {
    const QuantizeLaunch& L = *Ls[0];
    if (mb_status st = launch_pdl(encode_kernel, dim3((unsigned)L.enc_grid), dim3(kEncThreads),
                                  kEncSmem, stream, L.tmap, L.qa, L.tma ? 1 : 0, L.vec_out))
      return st;
  } else {
    int64_t eg[NB];
    if (n == 1) {
      eg[0] = Ls[0]->enc3_grid;
    } else {
      int64_t w[NB], cap[NB];
      for (int i = 0; i < n; ++i) {
        MB_REQUIRE(Ls[i]->enc3, "a batch needs the wide-tile encode for every matrix");
        w[i] = cap[i] = (int64_t)(Ls[i]->qa.ng / kE3Groups) * Ls[i]->qa.nrc;
      }
      split_grid(n, w, cap, Ls[0]->enc3_full, eg);
    }
    Enc3Batch<NB> E;
    std::memset(&E, 0, sizeof(E));
    for (int i = 0; i < n; ++i) {
      E.tmap[i] = Ls[i]->tmap;
      E.om[i] = Ls[i]->omaps;
      E.a[i] = Ls[i]->qa;
      E.use_tma[i] = Ls[i]->tma ? 1 : 0;
    }
    fill_map(E.bm, n, eg);
    static std::atomic<uint64_t> eattr{0};
    MB_CUDA_TRY(set_smem_limit_once(encode3_kernel<NB>, kE3Smem, eattr));
    if (mb_status st = launch_pdl(encode3_kernel<NB>, dim3((unsigned)E.bm.cta0[n]),
                                  dim3(kE3Threads), kE3Smem, stream, E))
      return st;
  }
  if (csr == nullptr) return MB_OK;
  CsrBatch<NB> B;
  std::memset(&B, 0, sizeof(B));
  int64_t bg[NB];
  for (int i = 0; i < n; ++i) {
    B.a[i] = Ls[i]->qa;
    B.capacity[i] = csr[i].capacity;
    B.vals[i] = csr[i].vals;
    B.cols[i] = csr[i].cols;
    bg[i] = std::max<int64_t>(1, std::min<int64_t>(ceil_div(Ls[i]->qa.M, 8), 1184 / n));
  }
  fill_map(B.bm, n, bg);
  return launch_pdl(extract_cap_kernel<NB>, dim3((unsigned)B.bm.cta0[n]), dim3(256), 0, stream,
                    B);
}

mb_status launch_stats(QuantizeLaunch& L, cudaStream_t stream) {
  QuantizeLaunch* p = &L;
  return launch_stats_batch<1>(&p, 1, stream);
}

mb_status launch_tables_encode(QuantizeLaunch& L, cudaStream_t stream, const CsrOut* csr) {
  QuantizeLaunch* p = &L;
  return launch_tables_encode_batch<1>(&p, 1, stream, csr);
}

// ---------------------------------------------------------------------------
// Row-split quantize: one matrix's rows over several processes (GPUs).  Each
// rank streams its slab of rows (stats without the selection) and exports one
// 32-byte record per group: min / max, the prediction and moment of the
// slab's serial-sum terms, the slab's rows and flags.  The records of all
// ranks, in rank (row) order, give every rank the same group parameters and
// the same sensitivity intervals as one pass over the whole matrix, so every
// rank takes the same selection (rows_select_kernel).  Groups left pending
// are settled by their exact serial sums over all rows (the caller gathers
// their column strips and quantizes them; mb_rows_set_precision), then each
// rank builds the 2nd-order tables and encodes its slab.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rows_pack_kernel(const QArgs a, SegRec* __restrict__ rec) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= a.ng) return;
  SegRec r;
  r.sum = a.select ? a.ws.gpred[g] : 0.0;
  r.mom = a.select ? a.ws.gmom[g] : 0.0;
  r.mn = a.ws.gmin[g];
  r.mx = a.ws.gmax[g];
  r.rows = (uint32_t)a.M;
  r.flags = a.select ? a.ws.gflag[g] : 0u;
  rec[g] = r;
}

// One CTA.  Group totals over the P slabs in row order (warp per group, lanes
// over slabs: the combine of ct_combine with slabs as segments), parameters
// of both precisions, intervals over all M_total rows, then the selection.
__global__ void __launch_bounds__(kStatsThreads, 1)
    rows_select_kernel(const QArgs A, const SegRec* __restrict__ rec, int P, int64_t M_total,
                       int32_t* __restrict__ pending, int32_t* __restrict__ counts) {
  extern __shared__ uint8_t dsm_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ng = A.ng;
  for (int g = warp; g < ng; g += kStatsThreads / 32) {
    float mn = INFINITY, mx = -INFINITY;
    uint32_t flags = 0;
    double carry = 0.0, mom = 0.0;
    for (int pp = 0; pp < P; pp += 32) {
      const int p = pp + lane;
      double sum = 0.0, smom = 0.0;
      uint32_t rows = 0;
      if (p < P) {
        const SegRec r = rec[(size_t)p * ng + g];
        sum = r.sum;
        smom = r.mom;
        rows = r.rows;
        mn = fminf(mn, r.mn);
        mx = fmaxf(mx, r.mx);
        flags |= r.flags;
      }
      double incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      mom += smom + (carry + (incl - sum)) * (16.0 * (double)rows);
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    mn = warp_min(mn);
    mx = warp_max(mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mom += __shfl_xor_sync(0xffffffffu, mom, o);
    flags = __reduce_or_sync(0xffffffffu, flags);
    if (lane == 0) {
      A.ws.gmin[g] = mn;
      A.ws.gmax[g] = mx;
      if (A.select) {
        A.ws.gpred[g] = carry;
        A.ws.gmom[g] = mom;
        A.ws.gflag[g] = flags;
        A.ws.gkey[g] = sens_interval_of(flags, carry, mom, M_total);
      }
    }
    group_params_warp(A.ws.params, A.ws.gscale, A.ws.greg, g, mn, mx, lane);
  }
  __threadfence();
  __syncthreads();
  select_from_intervals<kStatsThreads>(A, dsm_raw, (size_t)kStages * kTileBytes);
  __syncthreads();
  const Header* h = A.ws.hdr;
  const uint32_t np = *reinterpret_cast<const volatile uint32_t*>(&h->n_pend);
  const uint32_t nd = *reinterpret_cast<const volatile uint32_t*>(&h->n_dec);
  for (uint32_t i = tid; i < np; i += kStatsThreads) pending[i] = A.ws.order[nd + i];
  if (tid == 0) {
    counts[0] = (int32_t)np;
    counts[1] = np ? (int32_t)*reinterpret_cast<const volatile uint32_t*>(&h->need) : 0;
  }
}

// The precisions of the pending groups, decided by the caller; nothing stays
// pending afterwards.
__global__ void rows_set_kernel(const QArgs a, const int32_t* __restrict__ groups,
                                const uint8_t* __restrict__ prec, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t g = groups[i];
    if (g >= 0 && g < a.ng) a.ws.prec[g] = prec[i] ? 1 : 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    a.ws.hdr->n_pend = 0;
    a.ws.hdr->n_dec = (uint32_t)a.ng;
  }
  // the tile split of encode_kernel (uniform), which the selection leaves
  // open while groups are pending
  if (blockIdx.x == 0) enc_partition<256>(a, nullptr, nullptr);
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
  QuantizeLaunch L;
  if (mb_status st = quantize_prepare(weights_fp16, M, K, ratio_4bit, hessian_diag,
                                      hessian_numel, packed_2bit, packed_4bit, scales_1st_fp16,
                                      zeros_1st, scales_2nd_fp16, zeros_2nd, scales_1st_quant,
                                      group_precision, outlier_row_ptrs, nnz_device, workspace,
                                      workspace_bytes, false, L))
    return st;
  if (mb_status st = launch_stats(L, stream)) return st;
  return launch_tables_encode(L, stream, nullptr);
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

extern "C" mb_status mb_quantize_csr(const void* weights_fp16, int64_t M, int64_t K,
                                     double ratio_4bit, const float* hessian_diag,
                                     int64_t hessian_numel, int32_t* packed_2bit,
                                     int32_t* packed_4bit, void* scales_1st_fp16,
                                     int8_t* zeros_1st, void* scales_2nd_fp16, int8_t* zeros_2nd,
                                     uint8_t* scales_1st_quant, uint8_t* group_precision,
                                     int32_t* outlier_row_ptrs, int32_t* nnz_device,
                                     void* outlier_values_fp16, int32_t* outlier_col_indices,
                                     int64_t outlier_capacity, void* workspace,
                                     size_t workspace_bytes, mb_stream_t stream_) {
  mb_quantize_job job;
  job.weights_fp16 = weights_fp16;
  job.M = M;
  job.K = K;
  job.ratio_4bit = ratio_4bit;
  job.hessian_diag = hessian_diag;
  job.hessian_numel = hessian_numel;
  job.packed_2bit = packed_2bit;
  job.packed_4bit = packed_4bit;
  job.scales_1st_fp16 = scales_1st_fp16;
  job.zeros_1st = zeros_1st;
  job.scales_2nd_fp16 = scales_2nd_fp16;
  job.zeros_2nd = zeros_2nd;
  job.scales_1st_quant = scales_1st_quant;
  job.group_precision = group_precision;
  job.outlier_row_ptrs = outlier_row_ptrs;
  job.nnz_device = nnz_device;
  job.outlier_values_fp16 = outlier_values_fp16;
  job.outlier_col_indices = outlier_col_indices;
  job.outlier_capacity = outlier_capacity;
  job.workspace = workspace;
  job.workspace_bytes = workspace_bytes;
  return mb_quantize_csr_many(&job, 1, stream_);
}

extern "C" mb_status mb_quantize_csr_many(const mb_quantize_job* jobs, int64_t n,
                                          mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(n >= 0, "the job count must not be negative");
  MB_REQUIRE(n == 0 || jobs != nullptr, "jobs must not be null");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  // every job is checked before anything is launched
  std::vector<QuantizeLaunch> Ls((size_t)n);
  std::vector<CsrOut> csr((size_t)n);
  for (int64_t i = 0; i < n; ++i) {
    const mb_quantize_job& j = jobs[i];
    MB_REQUIRE(j.outlier_capacity >= 0, "outlier_capacity must not be negative");
    MB_REQUIRE(j.outlier_capacity == 0 || (j.outlier_values_fp16 && j.outlier_col_indices),
               "CSR pointers must not be null when outlier_capacity > 0");
    if (mb_status st = quantize_prepare(
            j.weights_fp16, j.M, j.K, j.ratio_4bit, j.hessian_diag, j.hessian_numel,
            j.packed_2bit, j.packed_4bit, j.scales_1st_fp16, j.zeros_1st, j.scales_2nd_fp16,
            j.zeros_2nd, j.scales_1st_quant, j.group_precision, j.outlier_row_ptrs,
            j.nnz_device, j.workspace, j.workspace_bytes, false, Ls[(size_t)i]))
      return st;
    csr[(size_t)i] = CsrOut{static_cast<__half*>(j.outlier_values_fp16),
                            j.outlier_col_indices, j.outlier_capacity};
  }
  // consecutive jobs on the wide-tile encode with the same sensitivity pass
  // share launches, kMaxBatch at a time
  int64_t i = 0;
  while (i < n) {
    QuantizeLaunch* grp[kMaxBatch];
    int k = 0;
    int64_t e = i;
    if (Ls[(size_t)i].enc3)
      while (e < n && k < kMaxBatch && Ls[(size_t)e].enc3 && Ls[(size_t)e].sens == Ls[(size_t)i].sens)
        grp[k++] = &Ls[(size_t)e++];
    if (k <= 1) {
      if (mb_status st = launch_stats(Ls[(size_t)i], stream)) return st;
      if (mb_status st = launch_tables_encode(Ls[(size_t)i], stream, &csr[(size_t)i])) return st;
      ++i;
      continue;
    }
    if (mb_status st = launch_stats_batch<kMaxBatch>(grp, k, stream)) return st;
    if (mb_status st = launch_tables_encode_batch<kMaxBatch>(grp, k, stream, &csr[(size_t)i]))
      return st;
    i = e;
  }
  return MB_OK;
}

extern "C" mb_status mb_quantize_exact_sums(const void* weights_fp16, int64_t M, int64_t K,
                                            double ratio_4bit, const float* hessian_diag,
                                            int64_t hessian_numel, float* sums,
                                            uint8_t* group_precision, void* workspace,
                                            size_t workspace_bytes, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(sums != nullptr && group_precision != nullptr, "output pointers must not be null");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  QuantizeLaunch L;
  if (mb_status st = quantize_prepare(weights_fp16, M, K, ratio_4bit, hessian_diag,
                                      hessian_numel, nullptr, nullptr, nullptr, nullptr, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, workspace,
                                      workspace_bytes, true, L))
    return st;
  MB_REQUIRE(L.sens && L.qa.n4 < L.qa.ng,
             "the exact sums need a hessian and a ratio_4bit selecting some but not all groups");
  L.qa.gp = group_precision;
  L.qa.all_pending = 1;
  if (mb_status st = launch_stats(L, stream)) return st;
  ArgsBatch<1> X;
  std::memset(&X, 0, sizeof(X));
  X.a[0] = L.qa;
  X.bm.n = 1;
  X.bm.cta0[0] = 0;
  X.bm.cta0[1] = kExactCtas;
  if (mb_status st = launch_pdl(exact_kernel<1>, dim3(kExactCtas), dim3(256), 0, stream, X))
    return st;
  QuantizeLaunch* p = &L;
  if (mb_status st = launch_tables<1>(&p, 1, stream)) return st;
  MB_CUDA_TRY(cudaMemcpyAsync(sums, L.qa.ws.sens, sizeof(float) * (size_t)L.qa.ng,
                              cudaMemcpyDeviceToDevice, stream));
  return MB_OK;
}

extern "C" mb_status mb_quantize_info(const void* workspace, size_t workspace_bytes, int64_t M,
                                      int64_t K, uint32_t* info, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(workspace && info, "null argument");
  MB_REQUIRE(M > 0 && K > 0, "M and K must be positive");
  const size_t need = workspace_layout(M, K, nullptr, nullptr);
  if (workspace_bytes < need) return set_error(MB_ERR_WORKSPACE, "workspace too small");
  Workspace ws;
  workspace_layout(M, K, static_cast<char*>(const_cast<void*>(workspace)), &ws);
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  Header h;
  MB_CUDA_TRY(cudaMemcpyAsync(&h, ws.hdr, sizeof(Header), cudaMemcpyDeviceToHost, stream));
  MB_CUDA_TRY(cudaStreamSynchronize(stream));
  info[0] = h.status;
  info[1] = h.n_straddle;
  info[2] = h.n_pend;
  info[3] = h.any_irregular;
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

// ---- row-split quantize ----

extern "C" size_t mb_rows_record_bytes(int64_t K) {
  return K > 0 ? (size_t)ceil_div(K, kGroup1) * sizeof(SegRec) : 0;
}

extern "C" mb_status mb_rows_stats(const void* weights_slab, int64_t M_slab, int64_t K,
                                   double ratio_4bit, const float* hessian_diag,
                                   int64_t hessian_numel, void* records, void* workspace,
                                   size_t workspace_bytes, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(records != nullptr, "records must not be null");
  MB_REQUIRE((reinterpret_cast<uintptr_t>(records) & 15u) == 0,
             "records must be 16-byte aligned");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  QuantizeLaunch L;
  if (mb_status st = quantize_prepare(weights_slab, M_slab, K, ratio_4bit, hessian_diag,
                                      hessian_numel, nullptr, nullptr, nullptr, nullptr, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, workspace,
                                      workspace_bytes, true, L))
    return st;
  L.qa.no_select = 1;
  if (mb_status st = launch_stats(L, stream)) return st;
  rows_pack_kernel<<<(unsigned)ceil_div(L.qa.ng, 256), 256, 0, stream>>>(
      L.qa, static_cast<SegRec*>(records));
  MB_LAUNCH_CHECK("rows_pack_kernel");
  return MB_OK;
}

extern "C" mb_status mb_rows_select(const void* records_all, int n_ranks, int64_t M_total,
                                    const void* weights_slab, int64_t M_slab, int64_t K,
                                    double ratio_4bit, const float* hessian_diag,
                                    int64_t hessian_numel, void* workspace,
                                    size_t workspace_bytes, int32_t* pending_groups,
                                    int32_t* counts, mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(records_all && pending_groups && counts, "null argument");
  MB_REQUIRE(n_ranks >= 1, "n_ranks must be >= 1");
  MB_REQUIRE(M_total >= M_slab, "M_total must cover the slab");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  QuantizeLaunch L;
  if (mb_status st = quantize_prepare(weights_slab, M_slab, K, ratio_4bit, hessian_diag,
                                      hessian_numel, nullptr, nullptr, nullptr, nullptr, nullptr,
                                      nullptr, nullptr, nullptr, nullptr, nullptr, workspace,
                                      workspace_bytes, true, L))
    return st;
  const int smem = kStages * kTileBytes;
  static std::atomic<uint64_t> attr_done{0};
  MB_CUDA_TRY(set_smem_limit_once(rows_select_kernel, smem, attr_done));
  rows_select_kernel<<<1, kStatsThreads, smem, stream>>>(
      L.qa, static_cast<const SegRec*>(records_all), n_ranks, M_total, pending_groups, counts);
  MB_LAUNCH_CHECK("rows_select_kernel");
  return MB_OK;
}

extern "C" mb_status mb_rows_set_precision(void* workspace, size_t workspace_bytes,
                                           int64_t M_slab, int64_t K, const int32_t* groups,
                                           const uint8_t* precision, int64_t n,
                                           mb_stream_t stream_) {
  clear_error();
  MB_REQUIRE(workspace != nullptr, "workspace must not be null");
  MB_REQUIRE(n == 0 || (groups && precision), "null argument");
  MB_REQUIRE(M_slab > 0 && K > 0, "M and K must be positive");
  if (workspace_bytes < workspace_layout(M_slab, K, nullptr, nullptr))
    return set_error(MB_ERR_WORKSPACE, "workspace too small");
  QArgs qa;
  std::memset(&qa, 0, sizeof(qa));
  workspace_layout(M_slab, K, static_cast<char*>(workspace), &qa.ws);
  qa.ng = (int)ceil_div(K, kGroup1);
  qa.nct = (int)ceil_div(K, kTileCols);
  qa.nrc = (int)ceil_div(M_slab, kChunkRows);
  int64_t eg = 1;
  if (mb_status st = legacy_enc_grid((int64_t)qa.nct * qa.nrc, device_sms(), &eg)) return st;
  qa.enc_grid = (int)eg;
  rows_set_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(qa, groups, precision,
                                                                           n);
  MB_LAUNCH_CHECK("rows_set_kernel");
  return MB_OK;
}

extern "C" mb_status mb_rows_encode(const void* weights_slab, int64_t M_slab, int64_t K,
                                    double ratio_4bit, const float* hessian_diag,
                                    int64_t hessian_numel, int32_t* packed_2bit,
                                    int32_t* packed_4bit, void* scales_1st_fp16,
                                    int8_t* zeros_1st, void* scales_2nd_fp16, int8_t* zeros_2nd,
                                    uint8_t* scales_1st_quant, uint8_t* group_precision,
                                    int32_t* outlier_row_ptrs, int32_t* nnz_device,
                                    void* workspace, size_t workspace_bytes,
                                    mb_stream_t stream_) {
  clear_error();
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  QuantizeLaunch L;
  if (mb_status st = quantize_prepare(weights_slab, M_slab, K, ratio_4bit, hessian_diag,
                                      hessian_numel, packed_2bit, packed_4bit, scales_1st_fp16,
                                      zeros_1st, scales_2nd_fp16, zeros_2nd, scales_1st_quant,
                                      group_precision, outlier_row_ptrs, nnz_device, workspace,
                                      workspace_bytes, false, L))
    return st;
  L.qa.exact_thresholds = 1;  // the selection took the parameters from all slabs' records
  return launch_tables_encode(L, stream, nullptr);
}
