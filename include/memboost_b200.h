/*
 * memboost_b200 -- C ABI of the B200-native (sm_100a) memboost quantization
 * hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream; no
 * torch types cross this boundary.  All work is enqueued on `stream` (may be
 * NULL for the legacy default stream); entry points return without a device
 * synchronisation unless stated otherwise.  The caller owns every buffer.
 *
 * Each function names the reference interface it replaces (paths are inside
 * the reference project: core/torch_ops.h, core/bindings.cpp,
 * core/torch_ops.cu).  Data layouts are the reference's QuantizedTensor
 * layout (memboost/formats.py:20-42):
 *   ng  = ceil(K / 16)            1st-order groups per row
 *   ng2 = ceil(M * ng / 256)      2nd-order groups
 *   packed_2bit       int32 [M, ng]     element j of a group at bits [2j, 2j+2)
 *   packed_4bit       int32 [M, 2*ng]   word 2g = cols 0-7, 2g+1 = cols 8-15,
 *                                       element j at bits [4j, 4j+4)
 *   scales_1st        fp16  [M, ng]
 *   zeros_1st         int8  [M, ng]
 *   scales_2nd        fp16  [ng2]
 *   zeros_2nd         int8  [ng2]
 *   scales_1st_quant  uint8 [M, ng]
 *   group_precision   uint8 [ng]        0 = 2-bit, 1 = 4-bit
 *   outlier_values    fp16  [nnz]       CSR, ascending column within a row
 *   outlier_col_indices int32 [nnz]
 *   outlier_row_ptrs  int32 [M + 1]
 */
#ifndef MEMBOOST_B200_H_
#define MEMBOOST_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mb_stream_t; /* == cudaStream_t */

typedef enum {
  MB_OK = 0,
  MB_ERR_INVALID_ARGUMENT = 1, /* a TORCH_CHECK of the reference would fire */
  MB_ERR_CUDA = 2,             /* a CUDA runtime call or launch failed */
  MB_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  MB_ERR_DEVICE_STATUS = 4     /* a kernel reported an error status */
} mb_status;

/* Text of the last error raised on the calling host thread ("" if none). */
const char* mb_last_error(void);

/* Library version string ("memboost_b200 <version> sm_100a"). */
const char* mb_version(void);

/* ---------------------------------------------------------------------------
 * quantize -- replaces memboost::quantize_op (core/torch_ops.h:18-22,
 * core/torch_ops.cu:105-264; bound as _C.quantize in core/bindings.cpp:25-29).
 *
 * Two calls, because the CSR outputs are sized by the outlier count:
 *   1. mb_quantize() writes every output except outlier_values /
 *      outlier_col_indices, writes outlier_row_ptrs [M+1] and the outlier
 *      count to *nnz_device (int32, device memory).
 *   2. When nnz > 0 the caller allocates the CSR arrays and calls
 *      mb_quantize_extract_outliers() with the same weights and workspace.
 * ratio_4bit, hessian_diag: as the reference -- sensitivity-based 4-bit
 * selection runs only when hessian_diag != NULL, hessian_numel > 0 and
 * ratio_4bit > 0; hessian_diag must then hold >= K fp32 values.
 * The workspace (device memory, any contents) must hold
 * mb_quantize_workspace_size(M, K) bytes and stay untouched between the two
 * calls.  Scratch use: per-group statistics, sensitivities, selection,
 * per-group parameters, 2nd-order tables and per-row outlier counts.
 * ------------------------------------------------------------------------- */
size_t mb_quantize_workspace_size(int64_t M, int64_t K);

mb_status mb_quantize(const void* weights_fp16, int64_t M, int64_t K, double ratio_4bit,
                      const float* hessian_diag, int64_t hessian_numel,
                      int32_t* packed_2bit, int32_t* packed_4bit, void* scales_1st_fp16,
                      int8_t* zeros_1st, void* scales_2nd_fp16, int8_t* zeros_2nd,
                      uint8_t* scales_1st_quant, uint8_t* group_precision,
                      int32_t* outlier_row_ptrs, int32_t* nnz_device, void* workspace,
                      size_t workspace_bytes, mb_stream_t stream);

/* Phase 2 of quantize -- core/torch_ops.cu:231-248 (extract_outliers). */
mb_status mb_quantize_extract_outliers(const void* weights_fp16, int64_t M, int64_t K,
                                       const int32_t* outlier_row_ptrs,
                                       void* outlier_values_fp16,
                                       int32_t* outlier_col_indices, const void* workspace,
                                       size_t workspace_bytes, mb_stream_t stream);

/* Both phases of quantize in one enqueue, with no host round trip --
 * core/torch_ops.cu:105-264 (quantize_op including extract_outliers,
 * :231-248).  Same inputs and outputs as mb_quantize, plus caller-sized CSR
 * arrays with room for outlier_capacity outliers: the extraction kernel is
 * chained to the quantize kernels on `stream` and reads the outlier count on
 * the device.  After the stream reaches this point, *nnz_device holds the
 * count; if it exceeds outlier_capacity the CSR values / columns were not
 * written and flag bit 3 (mb_quantize_flags) is set -- call
 * mb_quantize_extract_outliers with larger arrays (same workspace).  No host
 * synchronisation and no allocation inside: a sequence of these calls can
 * be recorded once and replayed (whole-model loops). */
mb_status mb_quantize_csr(const void* weights_fp16, int64_t M, int64_t K, double ratio_4bit,
                          const float* hessian_diag, int64_t hessian_numel,
                          int32_t* packed_2bit, int32_t* packed_4bit, void* scales_1st_fp16,
                          int8_t* zeros_1st, void* scales_2nd_fp16, int8_t* zeros_2nd,
                          uint8_t* scales_1st_quant, uint8_t* group_precision,
                          int32_t* outlier_row_ptrs, int32_t* nnz_device,
                          void* outlier_values_fp16, int32_t* outlier_col_indices,
                          int64_t outlier_capacity, void* workspace, size_t workspace_bytes,
                          mb_stream_t stream);

/* The arguments of one mb_quantize_csr call. */
typedef struct mb_quantize_job {
  const void* weights_fp16;
  int64_t M, K;
  double ratio_4bit;
  const float* hessian_diag;
  int64_t hessian_numel;
  int32_t* packed_2bit;
  int32_t* packed_4bit;
  void* scales_1st_fp16;
  int8_t* zeros_1st;
  void* scales_2nd_fp16;
  int8_t* zeros_2nd;
  uint8_t* scales_1st_quant;
  uint8_t* group_precision;
  int32_t* outlier_row_ptrs;
  int32_t* nnz_device;
  void* outlier_values_fp16;
  int32_t* outlier_col_indices;
  int64_t outlier_capacity;
  void* workspace;
  size_t workspace_bytes;
} mb_quantize_job;

/* n mb_quantize_csr calls in one enqueue, with the same results as n
 * separate calls -- the reference quantizes a model matrix by matrix
 * (models/llama.py:553-600, one _make_quantized_linear, hence one
 * quantize_op, each).  Up to 8 consecutive jobs
 * (same sensitivity pass, i.e. all with or all without a hessian, and
 * column groups a multiple of 16) run as one launch of each kernel, their
 * CTAs split among the matrices by size, so the launch and pipeline start-up
 * costs are paid once per 8 matrices.  Every job is validated before
 * anything is enqueued; the jobs must not share outputs or workspaces. */
mb_status mb_quantize_csr_many(const mb_quantize_job* jobs, int64_t n, mb_stream_t stream);

/* Diagnostics: every group's sensitivity, the reference's serial fp32 sum
 * of its M * 16 terms (core/quantize.cu:72-98), computed by the exact-sum
 * path that mb_quantize uses for the groups straddling the 4-bit boundary
 * -- here for all groups -- into sums[ceil(K / 16)], and the selection made
 * from them into group_precision (the same as mb_quantize's).  Needs a
 * hessian and a ratio_4bit that selects some but not all groups. */
mb_status mb_quantize_exact_sums(const void* weights_fp16, int64_t M, int64_t K,
                                 double ratio_4bit, const float* hessian_diag,
                                 int64_t hessian_numel, float* sums, uint8_t* group_precision,
                                 void* workspace, size_t workspace_bytes, mb_stream_t stream);

/* Host-side flags of the last mb_quantize on `workspace` (synchronises the
 * stream).  Bit 0: the 4-bit selection met a tie of equal sensitivities at
 * the selection boundary and broke it by lowest group index (the reference
 * breaks such ties by std::sort's unspecified order).  Bit 1: a pipeline
 * wait inside a kernel ran out (outputs invalid).  Bit 2: a 2nd-order zero
 * point round(-min / scales_2nd) of some 256-scale chunk lay outside
 * [-128, 127]; zeros_2nd keeps the reference's int8 cast of it
 * (core/quantize.cu:267-272), which wraps, so scales rebuilt from
 * scales_1st_quant / scales_2nd / zeros_2nd (mb_dequantize_2nd) are wrong
 * for that chunk -- a limit of the reference format.  It happens when a
 * chunk's 256 scales are tightly clustered (max / min below about 1.12).
 * Bit 3: mb_quantize_csr found more outliers than its CSR capacity. */
mb_status mb_quantize_flags(const void* workspace, size_t workspace_bytes, int64_t M, int64_t K,
                            uint32_t* flags, mb_stream_t stream);

/* Diagnostics of the last mb_quantize on `workspace` (synchronises the
 * stream; no counterpart in the reference).  info[0] = the flags of
 * mb_quantize_flags; info[1] = groups whose sensitivity interval straddled
 * the 4-bit selection boundary; info[2] = groups among them whose exact
 * serial fp32 sensitivity sums (the order of core/quantize.cu:72-98) were
 * computed to settle the selection; info[3] = 1 if a group of its selected
 * precision may hold outliers (the per-element reference formula ran). */
mb_status mb_quantize_info(const void* workspace, size_t workspace_bytes, int64_t M, int64_t K,
                           uint32_t info[4], mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * quantize without allocation -- no counterpart in the reference.
 *
 * For callers that cannot provide or allocate device memory for the
 * workspace: a C/C++ host linking only this library whose device memory is
 * owned entirely by its own fixed arena, or a latency path that must never
 * reach cudaMalloc/cudaFree (they can synchronise the device).  The scratch
 * is one static device array of MB_NOALLOC_SCRATCH_BYTES per GPU, held for
 * as long as the library is loaded; matrices whose workspace
 * (mb_quantize_workspace_size) exceeds it are rejected.
 *
 * Runs both phases of mb_quantize: same inputs and outputs, plus the CSR
 * arrays with room for outlier_capacity outliers.  Synchronises `stream`
 * once to read the outlier count into *nnz_host; if it exceeds the
 * capacity, MB_ERR_INVALID_ARGUMENT is returned and every output except the
 * CSR values/columns is valid.  All calls share the array: calls whose GPU
 * work overlaps race and corrupt each other -- order them.  The first call
 * on a device looks up the array's device address; make it before any
 * stream capture.
 * ------------------------------------------------------------------------- */
#define MB_NOALLOC_SCRATCH_BYTES (4u << 20) /* 4 MiB */

mb_status mb_quantize_noalloc(const void* weights_fp16, int64_t M, int64_t K, double ratio_4bit,
                              const float* hessian_diag, int64_t hessian_numel,
                              int32_t* packed_2bit, int32_t* packed_4bit, void* scales_1st_fp16,
                              int8_t* zeros_1st, void* scales_2nd_fp16, int8_t* zeros_2nd,
                              uint8_t* scales_1st_quant, uint8_t* group_precision,
                              int32_t* outlier_row_ptrs, int32_t* nnz_device,
                              void* outlier_values_fp16, int32_t* outlier_col_indices,
                              int64_t outlier_capacity, int64_t* nnz_host, mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * Row-split quantize -- one matrix's rows over several processes (GPUs); no
 * counterpart in the reference, which quantizes a matrix on one device
 * (core/torch_ops.cu:105-264).  The results equal mb_quantize on the whole
 * matrix bit for bit.  Rank p holds the row slab [r0_p, r1_p) of W (slab
 * boundaries multiples of 256 / gcd(ceil(K / 16), 256) rows, so no 2nd-order
 * chunk of 256 scales spans two ranks) and a workspace of
 * mb_quantize_workspace_size(M_slab, K) bytes.  Sequence per rank:
 *   1. mb_rows_stats: stream the slab, write one 32-byte record per group
 *      (mb_rows_record_bytes(K) bytes: min, max, prediction and moment of
 *      the slab's sensitivity terms, rows, flags);
 *   2. all-gather the records of all ranks in rank order (the caller's
 *      collective; P * mb_rows_record_bytes(K) bytes);
 *   3. mb_rows_select: group parameters and the 4-bit selection from the
 *      gathered records -- identical on every rank.  counts[0] = groups left
 *      pending (their sensitivity intervals straddle the boundary), counts[1]
 *      = how many of them are 4-bit; pending_groups[0 .. counts[0]) lists
 *      them (device memory, ascending);
 *   4. if counts[0] > 0: the caller settles them by their exact serial sums
 *      over all M_total rows -- e.g. gathers their column strips from every
 *      rank, quantizes the strip matrix with ratio (counts[1] + 0.5) /
 *      counts[0] and reads its group_precision -- and passes the result to
 *      mb_rows_set_precision (always required before step 5 when counts[0]
 *      > 0);
 *   5. mb_rows_encode: the slab's outputs (as mb_quantize on the slab: its
 *      rows of every [M, *] output, its ceil(M_slab * ng / 256) 2nd-order
 *      entries, outlier row pointers local to the slab -- add the outlier
 *      counts of the earlier ranks -- and *nnz_device); CSR values / columns
 *      by mb_quantize_extract_outliers on the slab.
 * ------------------------------------------------------------------------- */
size_t mb_rows_record_bytes(int64_t K);

mb_status mb_rows_stats(const void* weights_slab, int64_t M_slab, int64_t K, double ratio_4bit,
                        const float* hessian_diag, int64_t hessian_numel, void* records,
                        void* workspace, size_t workspace_bytes, mb_stream_t stream);

mb_status mb_rows_select(const void* records_all, int n_ranks, int64_t M_total,
                         const void* weights_slab, int64_t M_slab, int64_t K, double ratio_4bit,
                         const float* hessian_diag, int64_t hessian_numel, void* workspace,
                         size_t workspace_bytes, int32_t* pending_groups, int32_t* counts,
                         mb_stream_t stream);

mb_status mb_rows_set_precision(void* workspace, size_t workspace_bytes, int64_t M_slab,
                                int64_t K, const int32_t* groups, const uint8_t* precision,
                                int64_t n, mb_stream_t stream);

mb_status mb_rows_encode(const void* weights_slab, int64_t M_slab, int64_t K, double ratio_4bit,
                         const float* hessian_diag, int64_t hessian_numel, int32_t* packed_2bit,
                         int32_t* packed_4bit, void* scales_1st_fp16, int8_t* zeros_1st,
                         void* scales_2nd_fp16, int8_t* zeros_2nd, uint8_t* scales_1st_quant,
                         uint8_t* group_precision, int32_t* outlier_row_ptrs,
                         int32_t* nnz_device, void* workspace, size_t workspace_bytes,
                         mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * dequantize -- replaces memboost::dequantize_op (core/torch_ops.h:24-29,
 * core/torch_ops.cu:267-301; bound as _C.dequantize, core/bindings.cpp:31-38).
 * out[r, c] = fp16(float(scales_1st[r, g]) * (q - zeros_1st[r, g])), no
 * outlier add-back.
 * ------------------------------------------------------------------------- */
mb_status mb_dequantize(const int32_t* packed_2bit, const int32_t* packed_4bit,
                        const void* scales_1st_fp16, const int8_t* zeros_1st,
                        const uint8_t* group_precision, int64_t M, int64_t K, void* out_fp16,
                        mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * dequantize from the compact scales -- no counterpart in the reference,
 * which computes scales_1st_quant / scales_2nd / zeros_2nd
 * (core/quantize.cu:245-280) but never reads them back.  Every group's scale
 * is rebuilt from its 4-bit code by the reference's dequantize rule one level
 * up: s = fp16(float(scales_2nd[c]) * (q2 - zeros_2nd[c])), q2 =
 * scales_1st_quant[r, g], c = (r * ng + g) / 256; then out[r, col] =
 * fp16(float(s) * (q - zeros_1st[r, g])).  With nnz > 0 the CSR outliers
 * (row_ptrs [M + 1], col_indices / values [nnz]) are written back as their
 * exact fp16 values; entries past nnz or outside [0, K) are skipped.
 * ------------------------------------------------------------------------- */
mb_status mb_dequantize_2nd(const int32_t* packed_2bit, const int32_t* packed_4bit,
                            const uint8_t* scales_1st_quant, const void* scales_2nd_fp16,
                            const int8_t* zeros_2nd, const int8_t* zeros_1st,
                            const uint8_t* group_precision, const int32_t* outlier_row_ptrs,
                            const int32_t* outlier_col_indices, const void* outlier_values_fp16,
                            int64_t nnz, int64_t M, int64_t K, void* out_fp16,
                            mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * quantized GEMV -- no counterpart in the reference (it has no matmul over
 * its format).  y[r] = sum_c W[r, c] * x[c] in fp32 (y: M floats, x: K fp16),
 * W the reference dequantization of the codes (as mb_dequantize, per-element
 * fp16 rounding) with each CSR outlier's exact value in place of its code's.
 * outlier_row_ptrs [M + 1] is always read; col_indices / values [nnz] when
 * nnz > 0 (entries past nnz or outside [0, K) are skipped).
 * ------------------------------------------------------------------------- */
mb_status mb_qgemv(const int32_t* packed_2bit, const int32_t* packed_4bit,
                   const void* scales_1st_fp16, const int8_t* zeros_1st,
                   const uint8_t* group_precision, const int32_t* outlier_row_ptrs,
                   const int32_t* outlier_col_indices, const void* outlier_values_fp16,
                   int64_t nnz, int64_t M, int64_t K, const void* x_fp16, float* y,
                   mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * pack / unpack -- replace memboost::pack_2bit_op, unpack_2bit_op,
 * pack_4bit_op, unpack_4bit_op (core/torch_ops.h:10-15,
 * core/torch_ops.cu:20-102; bound in core/bindings.cpp:9-22).
 * Device buffers.  pack: n_values % 16 == 0 (2-bit) or % 8 == 0 (4-bit).
 * unpack: num_elements <= 16 * n_words (2-bit) or 8 * n_words (4-bit).
 * ------------------------------------------------------------------------- */
mb_status mb_pack_2bit(const uint8_t* values, int64_t n_values, int32_t* packed,
                       mb_stream_t stream);
mb_status mb_unpack_2bit(const int32_t* packed, int64_t n_words, int64_t num_elements,
                         uint8_t* values, mb_stream_t stream);
mb_status mb_pack_4bit(const uint8_t* values, int64_t n_values, int32_t* packed,
                       mb_stream_t stream);
mb_status mb_unpack_4bit(const int32_t* packed, int64_t n_words, int64_t num_elements,
                         uint8_t* values, mb_stream_t stream);

/* ---------------------------------------------------------------------------
 * GPTQ calibration (models/llama.py; the reference does these steps with
 * torch inside its layer loop, so there is no native interface to replace).
 * ------------------------------------------------------------------------- */

/* Hessian -- replaces the forward-hook accumulation H_acc.add_(x.T @ x)
 * (models/llama.py:523-528) and the normalisation H.div_(total_tokens)
 * (models/llama.py:547-551):
 *   H = alpha * X^T X            (accumulate == 0)
 *   H = H + alpha * X^T X        (accumulate != 0)
 * X: [N, K] row-major fp16 (x_is_bf16 == 0) or bf16, 16-byte aligned, K a
 * multiple of 8.  H: [K, K] fp32 row-major, 16-byte aligned; both triangles
 * are written.  Products of 16-bit inputs are exact in fp32; the sums run on
 * the tensor cores in fp32 in an order of their own, so H matches an fp32
 * GEMM to rounding, not bit for bit.  status_device (optional, device uint32)
 * gets bit 0 set if a pipeline wait ran out (the output is then invalid). */
mb_status mb_hessian(const void* X, int64_t N, int64_t K, int x_is_bf16, float alpha,
                     int accumulate, float* H, uint32_t* status_device, mb_stream_t stream);

/* How gptq_quantize's (w - gmin) / sc (a tensor divided by a Python float,
 * models/llama.py:278) is evaluated: PyTorch computes the IEEE quotient for
 * CPU tensors and multiplies by the fp32 reciprocal of the scalar for CUDA
 * tensors. */
#define MB_GPTQ_DIV_TRUE 0
#define MB_GPTQ_DIV_RECIPROCAL 1

/* Workspace bytes of mb_gptq_quantize (per-group parameters). */
size_t mb_gptq_workspace_size(int64_t M, int64_t K);

/* gptq_quantize -- replaces models/llama.py:234-294: per-group min/max of W
 * (L = 16 levels where group_precision[g] == 1, else 4), then per 128-column
 * block and column the rounding, Err = (w - q) / Hinv_cho[c, c] and the
 * intra-block update W_block[:, j+1:] -= Err * Hinv_cho[c, j+1:], all in the
 * reference's fp32 operation order: Q is bit-identical to the reference run
 * on the same device kind (scalar_division).  W, Q: [M, K] fp32 row-major,
 * 16-byte aligned, not aliased; K a multiple of 16; hinv_cho: [K, K] fp32
 * (upper Cholesky factor of H^-1, models/llama.py:177-203); blocksize 128. */
mb_status mb_gptq_quantize(const float* W, int64_t M, int64_t K, const float* hinv_cho,
                           const uint8_t* group_precision, int blocksize, int scalar_division,
                           float* Q, void* workspace, size_t workspace_bytes,
                           mb_stream_t stream);

/* Rows [row0, row1) of gptq_quantize's Q (written to Q_rows, [row1 - row0,
 * K]), with each group's min / max and scale over all M rows of W as the
 * reference computes them (models/llama.py:248-263) -- the per-rank part of
 * GPTQ with W's rows split over GPUs (rows are independent given Hinv_cho and
 * the group parameters).  Q_rows equals rows [row0, row1) of mb_gptq_quantize
 * bit for bit. */
mb_status mb_gptq_quantize_rows(const float* W, int64_t M, int64_t K, int64_t row0, int64_t row1,
                                const float* hinv_cho, const uint8_t* group_precision,
                                int blocksize, int scalar_division, float* Q_rows,
                                void* workspace, size_t workspace_bytes, mb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MEMBOOST_B200_H_ */
