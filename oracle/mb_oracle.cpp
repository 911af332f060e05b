// memboost oracle -- TEST INFRASTRUCTURE ONLY.
//
// A CPU restatement of memboost's quantization pipeline, written to reproduce
// the reference CUDA kernels bit for bit.  It is the checker for the sm_100a
// kernels in memboost_b200/csrc and the timed CPU baseline in bench.py; it is
// never linked into, loaded by, or called from the product path.
//
// Every step follows the reference operation by operation (same fp32 ops in
// the same order, same casts).  Citations are to the reference project:
//   core/quantize.cu      -- the CUDA kernels
//   core/torch_ops.cu     -- the host orchestration (allocation, host top-k,
//                            host prefix sum)
//
// Device semantics that C leaves undefined are emulated explicitly:
//   * float -> int32 conversion is `cvt.rzi.s32.f32`: truncate toward zero,
//     saturate at INT32_MIN/INT32_MAX, NaN -> 0            (f2i_rz_sat)
//   * int32 -> int8 keeps the low byte (two's complement)  (low_byte_i8)
//   * __float2half is round-to-nearest-even with overflow to inf
//                                                           (f32_to_f16_rn)
//
// The one open question about the reference's compiled code -- whether nvcc
// contracted `w - scale * (q - zero)` in the outlier test into a single fused
// multiply-add (quantize.cu:192-194, 217-219, 232-235) -- is a parameter
// (`fma_mode`); the GPU parity tests decide it against the reference kernels.
//
// Build: oracle/Makefile (g++ -O2 -ffp-contract=off, std::thread for the
// parallel loops).
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>
#include <thread>

namespace {

constexpr int kGroup1 = 16;   // core/quantize.cuh:9  GROUP_SIZE_1ST
constexpr int kGroup2 = 256;  // core/quantize.cuh:10 GROUP_SIZE_2ND

// ---- fp16 helpers (IEEE 754 binary16, written from the format definition) ----

inline float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t ex = (h >> 10) & 0x1F;
  const uint32_t man = h & 0x3FF;
  uint32_t bits;
  if (ex == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      float v = (float)man * 0x1p-24f;  // exact
      std::memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (ex == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((ex - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Round-to-nearest-even conversion (the behaviour of cvt.rn.f16.f32).
inline uint16_t f32_to_f16_rn(float f) {
  uint32_t bits;
  std::memcpy(&bits, &f, 4);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
  if (std::isnan(f)) return (uint16_t)0x7FFF;  // canonical NaN
  double v = std::fabs((double)f);
  if (std::isinf(f)) return sign | 0x7C00;
  if (v == 0.0) return sign;
  if (v < 0x1p-14) {  // half subnormal range: multiples of 2^-24
    double r = std::nearbyint(v * 0x1p24);  // default mode is to-nearest-even
    return sign | (uint16_t)r;              // r == 1024 is the smallest normal
  }
  int ex;
  std::frexp(v, &ex);  // v = m * 2^ex, m in [0.5, 1)
  int e = ex - 1;      // v in [2^e, 2^(e+1))
  double r = std::nearbyint(std::ldexp(v, 10 - e));  // in [1024, 2048]
  if (r == 2048.0) {
    r = 1024.0;
    e += 1;
  }
  if (e > 15) return sign | 0x7C00;
  return sign | (uint16_t)(((e + 15) << 10) | ((int)r - 1024));
}

// cvt.rzi.s32.f32 semantics.
inline int f2i_rz_sat(float x) {
  if (std::isnan(x)) return 0;
  if (x >= 2147483648.0f) return INT_MAX;
  if (x <= -2147483648.0f) return INT_MIN;
  return (int)x;
}

inline int8_t low_byte_i8(int v) { return (int8_t)(uint8_t)((uint32_t)v & 0xFFu); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Static-partition parallel loop over [0, n) on `nthreads` host threads
// (<= 0: all hardware threads).  Each index is handled by exactly one thread
// and every result depends only on its own index, so the output does not
// depend on the thread count.
template <class F>
void parallel_for(int64_t n, int nthreads, F&& body) {
  int nt = nthreads > 0 ? nthreads : (int)std::thread::hardware_concurrency();
  if (nt < 1) nt = 1;
  if ((int64_t)nt > n) nt = (int)std::max<int64_t>(n, 1);
  if (nt == 1) {
    for (int64_t i = 0; i < n; ++i) body(i);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve((size_t)nt);
  for (int t = 0; t < nt; ++t) {
    const int64_t lo = n * t / nt, hi = n * (t + 1) / nt;
    pool.emplace_back([lo, hi, &body] {
      for (int64_t i = lo; i < hi; ++i) body(i);
    });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// Group min/max -- core/quantize.cu:103-128.  Per 16-column group, fminf /
// fmaxf over all rows starting from +-1e10f.
void mbo_group_stats(const uint16_t* w, int64_t M, int64_t K, float* gmin, float* gmax,
                     int nthreads) {
  const int64_t ng = ceil_div(K, kGroup1);
  parallel_for(ng, nthreads, [&](int64_t g) {
    const int64_t c0 = g * kGroup1, c1 = std::min<int64_t>(c0 + kGroup1, K);
    float mn = 1e10f, mx = -1e10f;
    for (int64_t r = 0; r < M; ++r)
      for (int64_t c = c0; c < c1; ++c) {
        const float v = f16_to_f32(w[r * K + c]);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
      }
    gmin[g] = mn;
    gmax[g] = mx;
  });
}

// Group sensitivity -- core/quantize.cu:72-98.  A serial fp32 sum over the
// group in row-major order: for each row, for each column of the group,
//   s = (h > 1e-8f) ? (w*w / h) : (w*w);  sum += s;
// w*w of an fp16 value is exact in fp32, so whether the compiler fuses the
// `sum += w*w` branch into an FMA cannot change the result.
void mbo_sensitivity(const uint16_t* w, int64_t M, int64_t K, const float* h, float* sens,
                     int nthreads) {
  const int64_t ng = ceil_div(K, kGroup1);
  parallel_for(ng, nthreads, [&](int64_t g) {
    const int64_t c0 = g * kGroup1, c1 = std::min<int64_t>(c0 + kGroup1, K);
    float sum = 0.0f;
    for (int64_t r = 0; r < M; ++r)
      for (int64_t c = c0; c < c1; ++c) {
        const float v = f16_to_f32(w[r * K + c]);
        const float hv = h[c];
        const float s = (hv > 1e-8f) ? (v * v / hv) : (v * v);
        sum += s;
      }
    sens[g] = sum;
  });
}

// Host top-k -- core/torch_ops.cu:149-179: indices sorted by descending
// sensitivity with std::sort (the same standard-library call, so the order of
// equal keys is whatever libstdc++'s introsort gives), the first
// (int)(ratio * ng) marked 4-bit.  The count is clamped to ng (the reference
// indexes past the end when ratio > 1).
void mbo_select(const float* sens, int64_t ng, double ratio, uint8_t* gp) {
  std::vector<int> idx((size_t)ng);
  std::iota(idx.begin(), idx.end(), 0);
  std::sort(idx.begin(), idx.end(), [&](int a, int b) { return sens[a] > sens[b]; });
  int64_t n4 = (int64_t)(int)(ratio * (double)(int)ng);
  if (n4 > ng) n4 = ng;
  std::memset(gp, 0, (size_t)ng);
  for (int64_t i = 0; i < n4; ++i) gp[idx[(size_t)i]] = 1;
}

// Full quantize pipeline -- core/torch_ops.cu:105-264 calling the kernels of
// core/quantize.cu.  Output layout is the reference's 11-tensor list.
// Returns 0 on success, 1 if out_cap < nnz (then *nnz_out holds the needed
// size and every output except the CSR values/columns is valid), -1 on bad
// arguments.
int mbo_quantize(const uint16_t* w, int64_t M, int64_t K, double ratio, const float* hess,
                 int64_t hess_numel, int fma_mode, int nthreads, int32_t* packed2,
                 int32_t* packed4, uint16_t* scales1, int8_t* zeros1, uint16_t* scales2,
                 int8_t* zeros2, uint8_t* sq, uint8_t* gp, int32_t* row_ptrs,
                 uint16_t* out_vals, int32_t* out_cols, int64_t out_cap, int64_t* nnz_out,
                 float* dbg_gmin, float* dbg_gmax, float* dbg_sens) {
  if (M <= 0 || K <= 0) return -1;
  const int64_t ng = ceil_div(K, kGroup1);
  const int64_t ng2 = ceil_div(M * ng, kGroup2);

  // Step 1: group statistics (torch_ops.cu:139-146).
  std::vector<float> gmin((size_t)ng), gmax((size_t)ng);
  mbo_group_stats(w, M, K, gmin.data(), gmax.data(), nthreads);
  if (dbg_gmin) std::memcpy(dbg_gmin, gmin.data(), sizeof(float) * ng);
  if (dbg_gmax) std::memcpy(dbg_gmax, gmax.data(), sizeof(float) * ng);

  // Step 2: optional sensitivity-based precision (torch_ops.cu:148-179).
  std::memset(gp, 0, (size_t)ng);
  if (hess != nullptr && hess_numel > 0 && ratio > 0.0) {
    std::vector<float> sens((size_t)ng);
    mbo_sensitivity(w, M, K, hess, sens.data(), nthreads);
    if (dbg_sens) std::memcpy(dbg_sens, sens.data(), sizeof(float) * ng);
    mbo_select(sens.data(), ng, ratio, gp);
  }

  // Step 3: quantize weights -- quantize.cu:132-242.  Both packed arrays are
  // zero-filled (torch_ops.cu:131-132); only the selected one is written.
  std::memset(packed2, 0, sizeof(int32_t) * M * ng);
  std::memset(packed4, 0, sizeof(int32_t) * M * ng * 2);
  std::vector<uint8_t> mask((size_t)(M * K), 0);
  parallel_for(M, nthreads, [&](int64_t r) {
    for (int64_t g = 0; g < ng; ++g) {
      const int64_t c0 = g * kGroup1, c1 = std::min<int64_t>(c0 + kGroup1, K);
      const int gs = (int)(c1 - c0);
      const float mn = gmin[(size_t)g], mx = gmax[(size_t)g];
      const int prec = gp[g];
      const int L = (prec == 0) ? 4 : 16;
      float scale = (mx - mn) / (float)(L - 1);
      if (scale < 1e-8f) scale = 1e-8f;
      int zero = f2i_rz_sat(roundf(-mn / scale));
      zero = std::max(0, std::min(L - 1, zero));
      const int64_t si = r * ng + g;
      scales1[si] = f32_to_f16_rn(scale);
      zeros1[si] = (int8_t)zero;
      const float range = mx - mn;
      const float thr = (prec == 0) ? 0.4f * range : 0.15f * range;
      uint32_t words[2] = {0u, 0u};
      for (int i = 0; i < gs; ++i) {
        const int64_t c = c0 + i;
        const float v = f16_to_f32(w[r * K + c]);
        int q = f2i_rz_sat(roundf((v - mn) / scale));
        q = std::max(0, std::min(L - 1, q));
        const float qz = (float)(q - zero);
        float err;
        if (fma_mode)
          err = std::fabs(std::fma(-scale, qz, v));
        else {
          const float deq = scale * qz;
          err = std::fabs(v - deq);
        }
        if (err > thr) mask[(size_t)(r * K + c)] = 1;
        if (prec == 0)
          words[0] |= ((uint32_t)(q & 0x3)) << (i * 2);
        else
          words[i >> 3] |= ((uint32_t)(q & 0xF)) << ((i & 7) * 4);
      }
      if (prec == 0) {
        packed2[si] = (int32_t)words[0];
      } else {
        packed4[r * ng * 2 + g * 2] = (int32_t)words[0];
        packed4[r * ng * 2 + g * 2 + 1] = (int32_t)words[1];
      }
    }
  });

  // Step 4: 2nd-order scale quantization -- quantize.cu:245-281.
  const int64_t total = M * ng;
  parallel_for(ng2, nthreads, [&](int64_t c) {
    const int64_t s0 = c * kGroup2, s1 = std::min<int64_t>(s0 + kGroup2, total);
    float mn = 1e10f, mx = -1e10f;
    for (int64_t i = s0; i < s1; ++i) {
      const float s = f16_to_f32(scales1[i]);
      mn = fminf(mn, s);
      mx = fmaxf(mx, s);
    }
    float sc2 = (mx - mn) / 15.0f;
    if (sc2 < 1e-10f) sc2 = 1e-10f;
    const int z2 = f2i_rz_sat(roundf(-mn / sc2));
    scales2[c] = f32_to_f16_rn(sc2);
    zeros2[c] = low_byte_i8(z2);
    for (int64_t i = s0; i < s1; ++i) {
      const float s = f16_to_f32(scales1[i]);
      int q = f2i_rz_sat(roundf((s - mn) / sc2));
      q = std::max(0, std::min(15, q));
      sq[i] = (uint8_t)q;
    }
  });

  // Steps 5-6: outlier CSR -- quantize.cu:284-321, torch_ops.cu:210-248.
  // Row counts, host exclusive prefix sum, ascending-column extraction of the
  // original fp16 values.
  std::vector<int64_t> counts((size_t)M, 0);
  parallel_for(M, nthreads, [&](int64_t r) {
    int64_t n = 0;
    for (int64_t c = 0; c < K; ++c) n += mask[(size_t)(r * K + c)];
    counts[(size_t)r] = n;
  });
  row_ptrs[0] = 0;
  int64_t acc = 0;
  for (int64_t r = 0; r < M; ++r) {
    acc += counts[(size_t)r];
    row_ptrs[r + 1] = (int32_t)acc;
  }
  *nnz_out = acc;
  if (acc > out_cap) return 1;
  parallel_for(M, nthreads, [&](int64_t r) {
    int64_t o = row_ptrs[r];
    for (int64_t c = 0; c < K; ++c)
      if (mask[(size_t)(r * K + c)]) {
        out_vals[o] = w[r * K + c];
        out_cols[o] = (int32_t)c;
        ++o;
      }
  });
  return 0;
}

// Dequantize -- quantize.cu:386-444 / torch_ops.cu:267-301:
//   out = __float2half(float(scale_half) * ((float)q - zero)), no outlier add-back.
int mbo_dequantize(const int32_t* packed2, const int32_t* packed4, const uint16_t* scales1,
                   const int8_t* zeros1, const uint8_t* gp, int64_t M, int64_t K, uint16_t* out,
                   int nthreads) {
  if (M <= 0 || K <= 0) return -1;
  const int64_t ng = ceil_div(K, kGroup1);
  parallel_for(M, nthreads, [&](int64_t r) {
    for (int64_t g = 0; g < ng; ++g) {
      const int64_t c0 = g * kGroup1;
      const int64_t si = r * ng + g;
      const float scale = f16_to_f32(scales1[si]);
      const int zero = zeros1[si];
      for (int i = 0; i < kGroup1; ++i) {
        if (c0 + i >= K) break;
        uint32_t q;
        if (gp[g] == 0)
          q = ((uint32_t)packed2[si] >> (i * 2)) & 0x3u;
        else
          q = ((uint32_t)packed4[r * ng * 2 + g * 2 + (i >> 3)] >> ((i & 7) * 4)) & 0xFu;
        const float v = scale * ((float)q - (float)zero);
        out[r * K + c0 + i] = f32_to_f16_rn(v);
      }
    }
  });
  return 0;
}

// Pack / unpack -- core/torch_ops.cu:20-102.  Element j of word i sits at
// bits [2j, 2j+2) (2-bit, 16 per word) or [4j, 4j+4) (4-bit, 8 per word).
void mbo_pack_2bit(const uint8_t* v, int64_t n_words, int32_t* out) {
  for (int64_t i = 0; i < n_words; ++i) {
    uint32_t word = 0;
    for (int j = 0; j < 16; ++j) word |= ((uint32_t)(v[i * 16 + j] & 0x3)) << (j * 2);
    out[i] = (int32_t)word;
  }
}

void mbo_unpack_2bit(const int32_t* p, int64_t n_words, int64_t num_elements, uint8_t* out) {
  std::memset(out, 0, (size_t)num_elements);
  for (int64_t i = 0; i < n_words; ++i) {
    const uint32_t word = (uint32_t)p[i];
    for (int j = 0; j < 16 && i * 16 + j < num_elements; ++j) out[i * 16 + j] = (word >> (j * 2)) & 0x3;
  }
}

void mbo_pack_4bit(const uint8_t* v, int64_t n_words, int32_t* out) {
  for (int64_t i = 0; i < n_words; ++i) {
    uint32_t word = 0;
    for (int j = 0; j < 8; ++j) word |= ((uint32_t)(v[i * 8 + j] & 0xF)) << (j * 4);
    out[i] = (int32_t)word;
  }
}

void mbo_unpack_4bit(const int32_t* p, int64_t n_words, int64_t num_elements, uint8_t* out) {
  std::memset(out, 0, (size_t)num_elements);
  for (int64_t i = 0; i < n_words; ++i) {
    const uint32_t word = (uint32_t)p[i];
    for (int j = 0; j < 8 && i * 8 + j < num_elements; ++j) out[i * 8 + j] = (word >> (j * 4)) & 0xF;
  }
}

// gptq_quantize -- models/llama.py:234-294 (torch fp32 tensor arithmetic
// with Python-float scalars), operation by operation:
//   :252-263  gmin/gmax = W[:, 16g:16g+16].min()/.max() (.item(): NaN
//             propagates), group_min[g] = gmin (fp32), group_scale[g] =
//             (gmax - gmin) / (L - 1) in double stored as fp32, 0.0 unless
//             gmax > gmin; L = 16 where gp[g] == 1 else 4
//   :265-268  blocks of `blocksize` columns; W_block = a copy of the
//             original W block (no column of a block is written before it
//             is copied), Err per column
//   :277-281  sc > 0: q_int = ((w - gmin) / sc).round().clamp(0, L - 1),
//             zero = round(-gmin / sc) (Python: double, half-even),
//             q = sc * (q_int - zero); else q = gmin
//   :283      Err = (w - q) / Hinv_cho[col, col]
//   :286-289  W_block[:, j+1:] -= Err[:, j] * Hinv_cho[col, j+1:block_end]
// (w - gmin) / sc divides a tensor by a Python float: PyTorch evaluates that
// as the IEEE quotient on CPU tensors (div_mode 0) and as a multiplication by
// the fp32 reciprocal 1.0f / sc on CUDA tensors (div_mode 1).  Rows are
// independent; they are split over host threads.
void mbo_gptq_quantize(const float* W, int64_t M, int64_t K, const float* Hc, const uint8_t* gp,
                       int64_t blocksize, int div_mode, float* Q, int nthreads) {
  const int64_t ng = K / 16;
  std::vector<float> gmin(ng), sc(ng), rsc(ng), zero_f(ng), lmax(ng);
  for (int64_t g = 0; g < ng; ++g) {
    float mn = INFINITY, mx = -INFINITY;
    bool nan = false;
    for (int64_t r = 0; r < M; ++r)
      for (int64_t c = 16 * g; c < 16 * g + 16; ++c) {
        const float v = W[r * K + c];
        if (std::isnan(v)) nan = true;
        mn = std::min(mn, v);
        mx = std::max(mx, v);
      }
    if (nan) mn = mx = NAN;
    const int L = gp[g] == 1 ? 16 : 4;
    const double d = ((double)mx > (double)mn) ? ((double)mx - (double)mn) / (double)(L - 1) : 0.0;
    gmin[g] = mn;
    sc[g] = (float)d;
    rsc[g] = sc[g] > 0.0f ? 1.0f / sc[g] : 0.0f;
    zero_f[g] = sc[g] > 0.0f ? (float)std::nearbyint(-(double)mn / (double)sc[g]) : 0.0f;
    lmax[g] = (float)(L - 1);
  }
  parallel_for(M, nthreads, [&](int64_t r) {
    std::vector<float> wb((size_t)blocksize);
    for (int64_t bs = 0; bs < K; bs += blocksize) {
      const int64_t be = std::min(bs + blocksize, K);
      const int64_t n = be - bs;
      for (int64_t c = 0; c < n; ++c) wb[c] = W[r * K + bs + c];
      for (int64_t j = 0; j < n; ++j) {
        const int64_t col = bs + j, g = col / 16;
        const float x = wb[j];
        float q;
        if (sc[g] > 0.0f) {
          const float dlt = x - gmin[g];
          float qi = std::nearbyint(div_mode == 1 ? dlt * rsc[g] : dlt / sc[g]);
          if (!std::isnan(qi)) qi = std::min(std::max(qi, 0.0f), lmax[g]);
          q = sc[g] * (qi - zero_f[g]);
        } else {
          q = gmin[g];
        }
        const float err = (x - q) / Hc[col * K + col];
        Q[r * K + col] = q;
        for (int64_t c = j + 1; c < n; ++c) wb[c] = wb[c] - err * Hc[col * K + bs + c];
      }
    }
  });
}

// Conversion helpers exported for the tests.
float mbo_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t mbo_f32_to_f16(float f) { return f32_to_f16_rn(f); }

}  // extern "C"
