/*
 * g2ptq_b200 -- C ABI of the B200 (sm_100a) quantization hot path.
 *
 * Every entry point takes raw device pointers, sizes, leading dimensions and a
 * cudaStream_t passed as void*, enqueues its kernels on that stream and
 * returns an int status (G2Q_OK, or a negative G2Q_ERR_* code for an invalid
 * argument or a failed launch).  Entry points never allocate or free device
 * memory and never synchronise the device: callers pass the scratch space a
 * call needs (the *_workspace_bytes queries give its size).  Conditions that
 * are only known on the device (a non-positive Cholesky pivot, a NaN, a zero
 * quantization scale, a tensor-core pipeline wait that gave up) are written
 * to caller-provided device int words (`status`, `info`); a status word is
 * only ever changed from 0 to the first code recorded, so one word can collect
 * the outcome of many calls, and a NULL status discards it.
 *
 * Matrices are row-major fp32 unless stated.  "Token-major" activations are
 * [T, C] with the channel index contiguous, exactly as a linear layer's input
 * arrives in the reference's forward hooks.
 *
 * Each declaration names the reference interface it replaces (paths are
 * relative to the G2PTQ project root).
 */
#ifndef G2PTQ_B200_H
#define G2PTQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G2Q_OK 0
#define G2Q_ERR_INVALID_ARG (-1)
#define G2Q_ERR_CUDA (-2)
#define G2Q_ERR_UNSUPPORTED (-3)
#define G2Q_ERR_NONFINITE (-4)
#define G2Q_ERR_TIMEOUT (-5)
#define G2Q_ERR_BAD_SCALE (-6)
/* the request needs more scratch than the library-owned array of
 * g2q_gram_update_noalloc holds */
#define G2Q_ERR_SCRATCH_LIMIT (-7)

/* element types of activation inputs */
#define G2Q_DTYPE_BF16 0
#define G2Q_DTYPE_F32 1
#define G2Q_DTYPE_F16 2

/* compensation methods */
#define G2Q_METHOD_GPTQ 0
#define G2Q_METHOD_G2PTQ 1
#define G2Q_METHOD_GPTAQ 2

/* block-loss heads of the G2PTQ refresh step */
#define G2Q_LOSS_KL 0  /* sum of KL(softmax(target) || softmax(x)) over rows */
#define G2Q_LOSS_NLL 1 /* sum of cross entropy of x against int64 labels */
#define G2Q_LOSS_MSE 2 /* sum over rows of mean((x - target)^2) / 2 */

/* output masks of g2q_gemm */
#define G2Q_MASK_FULL 0
#define G2Q_MASK_LOWER 1        /* i >= j */
#define G2Q_MASK_UPPER 2        /* i <= j */
#define G2Q_MASK_STRICT_UPPER 3 /* i <  j, others set to zero */

/* ABI version; bumped on any signature change. */
int g2q_abi_version(void);

/* Bound, in SM clock cycles, of every pipeline wait of the tensor-core
 * kernels launched after this call (cycles <= 0 restores the default of
 * 4e9, about two seconds); returns the previous bound.  A wait that runs out
 * records G2Q_ERR_TIMEOUT in the call's status word and the kernel winds down
 * without trapping, so the CUDA context stays usable.  No counterpart in the
 * reference, whose products run in cuBLAS. */
int64_t g2q_set_wait_limit(int64_t cycles);

/* Number of kernels this library has launched in the process so far
 * (host-side count of successful launch calls). */
int64_t g2q_launch_count(void);

/* Human-readable text for a status code (static storage). */
const char* g2q_status_string(int status);

/* Copies `t` token rows of `src` ([t, C], row stride src_ld, element type
 * src_dtype) into rows [row0, row0 + t) of a staging buffer `dst`
 * ([*, dst_ld], element type dst_dtype: BF16 only for a BF16 source, else
 * F32), converting the element type.  When `sub` is non-NULL the staged value
 * is src - sub (same layout and type as src), which is how GPTAQ's
 * (X_fp - X) operand is formed.
 * Replaces the input handling of GPTQ.add_batch, gptq_utils/gptq_utils.py:115-125,
 * and GPTAQ.add_batch, gptq_utils/gptaq_utils.py:130-146. */
int g2q_stage_tokens(void* dst, int dst_dtype, int64_t dst_ld, int64_t row0,
                     const void* src, const void* sub, int src_dtype, int64_t src_ld,
                     int64_t t, int64_t C, void* stream);

/* Gram-matrix update over staged tokens:
 *   D[i, j] <- alpha * D[i, j] + beta * sum_t A[t, i] * s[t] * B[t, j]
 * A is [T, M] (lda), B is [T, N] (ldb), both token-major with element type
 * G2Q_DTYPE_BF16 or G2Q_DTYPE_F32; s[t] = row_scale[t * scale_stride] when
 * row_scale is non-NULL, else 1.  symmetric != 0 (A == B, M == N, no row
 * scale asymmetry needed) computes the upper triangle and mirrors it, leaving
 * a full symmetric D.  precision: 0 = fp32 CUDA cores, 1 = tensor cores
 * (bf16 operands exact for BF16 input; FP32 input split into bf16 hi/lo
 * pairs), which needs `workspace` of g2q_gram_workspace_bytes bytes.
 * `status` (device int, may be NULL) receives G2Q_ERR_TIMEOUT when a
 * tensor-core pipeline wait gives up (D is then incomplete).
 * Replaces the Hessian products of GPTQ.add_batch (gptq_utils/gptq_utils.py:123-126),
 * G2PTQ.add_batch (gptq_utils/g2ptq_utils.py:193-200), GPTAQ.add_batch
 * (gptq_utils/gptaq_utils.py:139-146) and GPTQGuided.add_batch
 * (gptq_utils/gptq_guided_utils.py:78-80). */
int g2q_gram_update(float* D, int64_t ldd, int64_t M, int64_t N,
                    const void* A, int a_dtype, int64_t lda,
                    const void* B, int b_dtype, int64_t ldb,
                    const float* row_scale, int64_t scale_stride,
                    int64_t T, int symmetric, float alpha, float beta, int precision,
                    void* workspace, size_t workspace_bytes, int* status, void* stream);
size_t g2q_gram_workspace_bytes(int64_t M, int64_t N, int64_t T, int precision);

/* Row-scaled Gram updates of G row groups in one call, for g < G:
 *   D[g] <- alpha * D[g] + beta * X^T diag(s[:, g]) X
 * D[g] at D + g * d_gstride (C x C, row stride ldd, left full symmetric),
 * X [T, C] token-major (row stride ldx, G2Q_DTYPE_BF16 or G2Q_DTYPE_F32),
 * s[t, g] = s[t * sstride + g].  Each group's result is that of
 * g2q_gram_update(..., row_scale = s + g, symmetric = 1); at precision 1 BF16
 * tokens are split for all groups in one pass and the G products run as one
 * launch (workspace: g2q_gram_grouped_workspace_bytes).  `status` as for
 * g2q_gram_update.
 * Replaces the per-group saliency-weighted products of G2PTQ.add_batch
 * (gptq_utils/g2ptq_utils.py:193-200) and GPTQGuided.add_batch
 * (gptq_utils/gptq_guided_utils.py:78-80). */
int g2q_gram_update_grouped(float* D, int64_t ldd, int64_t d_gstride, int64_t C,
                            const void* X, int x_dtype, int64_t ldx,
                            const float* s, int64_t sstride, int G, int64_t T,
                            float alpha, float beta, int precision,
                            void* workspace, size_t workspace_bytes, int* status,
                            void* stream);
size_t g2q_gram_grouped_workspace_bytes(int64_t C, int64_t T, int G, int precision);

/* g2q_gram_update at precision 1 (tensor cores) without caller-provided
 * scratch: the bf16 splits of FP32 or row-scaled operands go to a file-scope
 * device array of G2Q_GRAM_STATIC_SCRATCH_BYTES (40 MiB) owned by the library,
 * so neither the caller nor the call allocates device memory.  Requests with
 * g2q_gram_workspace_bytes(M, N, T, 1) above that size return
 * G2Q_ERR_SCRATCH_LIMIT (e.g. T = 1024 tokens at C = 4096 fits; split longer
 * token runs into several calls with alpha = 1 after the first).  BF16 inputs
 * without row scale use no scratch.  The array used is the one of `stream`'s
 * device, which must be the current device (a stream of another device
 * returns G2Q_ERR_INVALID_ARG).  The first call on a device looks the array
 * up (set-up; make it before any stream capture).  One array per device:
 * calls that overlap in time (several streams or host threads) race on it;
 * calls on one stream are safe.  `status` as for g2q_gram_update.  No
 * counterpart in the reference, whose add_batch products allocate through
 * torch. */
#define G2Q_GRAM_STATIC_SCRATCH_BYTES (40u << 20)
int g2q_gram_update_noalloc(float* D, int64_t ldd, int64_t M, int64_t N,
                            const void* A, int a_dtype, int64_t lda,
                            const void* B, int b_dtype, int64_t ldb,
                            const float* row_scale, int64_t scale_stride,
                            int64_t T, int symmetric, float alpha, float beta, int* status,
                            void* stream);
size_t g2q_gram_static_scratch_bytes(void);

/* Adds sum_t x[t, c]^2 * scale to acc[c] after acc *= keep: the running mean
 * of squared activations kept by G2PTQ/GPTQGuided.add_batch
 * (gptq_utils/g2ptq_utils.py:195,201; gptq_utils/gptq_guided_utils.py:81). */
int g2q_sq_colsum(float* acc, float keep, float scale, const void* X, int x_dtype,
                  int64_t ldx, int64_t T, int64_t C, void* stream);

/* Batched fp32 GEMM  C <- alpha * C + beta * op(A) op(B)  with an output mask.
 * op(A) is M x K (A stored K x M when transA), op(B) is K x N (B stored N x K
 * when transB).  Replaces the torch.bmm / baddbmm_ products of fasterquant:
 * gptq_utils/g2ptq_utils.py:462,475-476 (G2PTQ Z and GHinv) and
 * gptq_utils/gptaq_utils.py:350-352 (GPTAQ P). */
int g2q_gemm(float* C, int64_t ldc, int64_t strideC,
             const float* A, int64_t lda, int64_t strideA, int transA,
             const float* B, int64_t ldb, int64_t strideB, int transB,
             int64_t M, int64_t N, int64_t K, int64_t batch,
             float alpha, float beta, int out_mask, void* stream);

/* g2q_gemm on tensor cores with fp32-level accuracy: both operands carried as
 * fp16 hi/lo pairs (22 significant bits), every output row / column scaled by
 * a power of two, three products per K step, fp32 accumulation.  out_mask
 * G2Q_MASK_UPPER falls back to the CUDA-core kernel.  Needs
 * g2q_gemm_tc_workspace_bytes(M, N, K, batch, strideA != 0, strideB != 0)
 * bytes of workspace.  `status` as for g2q_gram_update.  Replaces the same
 * fasterquant products as g2q_gemm. */
int g2q_gemm_tc(float* C, int64_t ldc, int64_t strideC,
                const float* A, int64_t lda, int64_t strideA, int transA,
                const float* B, int64_t ldb, int64_t strideB, int transB,
                int64_t M, int64_t N, int64_t K, int64_t batch,
                float alpha, float beta, int out_mask,
                void* workspace, size_t workspace_bytes, int* status, void* stream);
size_t g2q_gemm_tc_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t batch,
                                   int a_batched, int b_batched);

/* Damped inverse-Cholesky factor.  For each of `batch` matrices H[b] (C x C,
 * symmetric, row stride ldh, batch stride C*ldh) computes upper-triangular
 * U[b] with U^T U = (H + d I)^-1, d = damp_percent[b] * mean(diag H[b]).
 * info[b] (device int) receives 0, the 1-based index of the first
 * non-positive pivot, -1 when the factor holds a NaN, or G2Q_ERR_TIMEOUT when
 * a tensor-core pipeline wait of the chain gave up.  Route: UL
 * factorization H + dI = V V^T (V upper), U = V^-1 -- potrf + trtri, half the
 * work of potrf + potri + potrf.  precision: 0 = fp32 CUDA cores, 1 = trailing
 * updates on tensor cores over scaled fp16 hi/lo operand pairs (three
 * products, fp32-level accuracy).
 * Needs g2q_chol_workspace_bytes(C) bytes.  With precision 1 and batch >= 2, a
 * workspace of k times that (plus 4 KiB) factors the batch in chains of
 * min(k, batch) matrices that advance panel by panel together, every launch
 * of a step covering the whole chain (the layer-batched objects' one launch
 * sequence; results equal those of one-by-one calls bit for bit).  With
 * precision 0, up to four of the batch's factorizations run side by side on
 * library-owned streams forked from and joined back to `stream`.  A timeout
 * in a batched chain is reported in the info word of the chain's first
 * matrix.
 * Replaces the damped Cholesky chain of gptq_utils/gptq_utils.py:291-311
 * (and its copies g2ptq_utils.py:430-450, gptaq_utils.py:323-343,
 * gptq_guided_utils.py:145-165); the damp auto-increment retry stays with the
 * caller, which reads `info`. */
int g2q_chol_upper_inverse(float* U, const float* H, int64_t C, int64_t ldh, int64_t batch,
                           const float* damp_percent_host, int* info, int precision,
                           void* workspace, size_t workspace_bytes, void* stream);
size_t g2q_chol_workspace_bytes(int64_t C);

/* Upper triangle (i <= j) of `batch` C x C matrices H[b] (row stride ldh,
 * batch stride h_bstride), packed row by row and multiplied by `scale`:
 * element (i, j) of matrix b goes to dst[b * C(C+1)/2 + i C - i(i-1)/2 + j - i].
 * g2q_unpack_upper writes H back from that layout: the lower triangle
 * mirrored (mirror != 0) or set to zero (an upper-triangular factor).  The
 * symmetric Hessians and the triangular factors cross NCCL in this form
 * (half the bytes), with the sample-share rescale folded into the pack.
 * Replaces the full-matrix dist.reduce / dist.broadcast of
 * gptq_utils/gptq_utils.py:369-387 and the per-method copies
 * (g2ptq_utils.py:530-575, gptaq_utils.py:393-439, gptq_guided_utils.py:213-249). */
int g2q_pack_upper(float* dst, const float* H, int64_t C, int64_t ldh, int64_t h_bstride,
                   int64_t batch, float scale, void* stream);
int g2q_unpack_upper(float* H, const float* src, int64_t C, int64_t ldh, int64_t h_bstride,
                     int64_t batch, int mirror, void* stream);

/* Per-row quantization parameters over `cols` columns of W (row stride ldw):
 * xmin = min(min(x), 0), xmax = max(max(x), 0); symmetric:
 * scale = max(|xmin|, xmax) / ((2^bits - 1) / 2), zero = 0; asymmetric:
 * scale = (xmax - xmin) / (2^bits - 1), zero = clamp(round(minq - xmin/scale)).
 * Results go to scale[r * param_ld] / zero[r * param_ld].  A non-positive
 * scale sets *status to G2Q_ERR_BAD_SCALE.
 * Replaces WeightQuantizer.find_params without clip search,
 * utils/quant_utils.py:377-433. */
int g2q_find_params(float* scale, float* zero, int64_t param_ld,
                    const float* W, int64_t rows, int64_t cols, int64_t ldw,
                    int bits, int sym, int* status, void* stream);

/* g2q_find_params for `count` consecutive weight groups in one launch: group g
 * covers columns first + g * groupsize .. (clipped at C) of W [rows, C]
 * (row stride ldw) and writes column first / groupsize + g of scale / zero
 * [rows, param_ld]; first is a multiple of groupsize.  Each group's result is
 * that of g2q_find_params on its columns.
 * Replaces the per-group WeightQuantizer.find_params loop of fasterquant's
 * static-group set-up, gptq_utils/gptq_utils.py:259-270. */
int g2q_find_params_groups(float* scale, float* zero, int64_t param_ld,
                           const float* W, int64_t rows, int64_t C, int64_t ldw,
                           int bits, int sym, int64_t first, int count, int groupsize,
                           int* status, void* stream);

/* Clip search of WeightQuantizer.find_params (--w_clip / --w_hclip).  The
 * range [xmin, xmax] is shrunk on a grid, xmin * (1 - i/grid) and
 * xmax * (1 - j/grid) for i, j < maxshrink * grid, and the first (i, j) with
 * the smallest error over the row's columns is kept: sum |fq - x|^norm, or,
 * with hdiag, sum (fq - x)^2 * hdiag[(r / rows_per_block) * hdiag_ld + c]
 * (the Hessian diagonal of the row's block).  Defaults of the reference:
 * grid 50, maxshrink 0.5, norm 2.4. */
typedef struct {
  int grid;
  float maxshrink;
  float norm;
  const float* hdiag;      /* NULL: the |fq - x|^norm error */
  int64_t hdiag_ld;
  int64_t rows_per_block;  /* rows sharing one hdiag row */
} g2q_clip_t;

/* g2q_find_params with the clip search above.
 * Replaces WeightQuantizer.find_params with mse=True (and hclip),
 * utils/quant_utils.py:373-425 (_mse_step_sym/_asym :106-133). */
int g2q_find_params_clip(float* scale, float* zero, int64_t param_ld, const float* W,
                         int64_t rows, int64_t cols, int64_t ldw, int bits, int sym,
                         const g2q_clip_t* clip, int* status, void* stream);

/* Fake quantization  q = clamp(round(w / s) + z, -(maxq+1), maxq),
 * out = s * (q - z)  with per-element parameters s = scale[r*param_ld + colmap[c]].
 * Writes out (fp32, row stride ldo) and, when codes is non-NULL, int8 codes.
 * Replaces WeightQuantizer.fake_quantize (utils/quant_utils.py:435-459) and
 * common_utils.fake_quantize_grouped (gptq_utils/common_utils.py:33-45). */
int g2q_fake_quantize(float* out, int64_t ldo, int8_t* codes, int64_t ldq,
                      const float* W, int64_t ldw, int64_t rows, int64_t cols,
                      const float* scale, const float* zero, int64_t param_ld,
                      const int* colmap, int maxq, void* stream);

/* One lazy-batch compensation block (the reference's kernel boundary).
 * W[b] is rows x ncols (row stride ldw, batch stride w_bstride), hinv[b] is
 * the ncols x ncols upper block (row stride ldh, batch stride h_bstride).
 * Quantization parameters of row r, column c are
 * scale[(b*rows + r) * param_ld + colmap[c]] (same for zero).
 * In place: W <- dequantized Q; codes (int8, optional), err (fp32, optional,
 * same layout as W).  G2PTQ also reads z and updates ghinv (same layout as W);
 * GPTAQ reads p (same layout as hinv).  ncols <= 128.  G2PTQ's --approx_grad
 * ablation: wraw (same layout as W, the raw weights) and approx_beta != 0
 * subtract (w - wraw) * approx_beta from each column's error and pull the
 * next column toward its raw value by the same factor (g2ptq_utils.py:48-51,
 * 71-73); NULL / 0 otherwise (and for the other methods).
 * Replaces run_eager / _run_torch_compensation / _run_triton_compensation of
 * gptq_utils/gptq_utils.py:28-90, gptq_utils/g2ptq_utils.py:34-126 and
 * gptq_utils/gptaq_utils.py:28-100 (reference layout [B, blk, R] is the
 * transpose of this one). */
int g2q_compensate_block(int method, float* W, int64_t ldw, int64_t w_bstride,
                         int64_t batch, int64_t rows, int64_t ncols,
                         const float* hinv, int64_t ldh, int64_t h_bstride,
                         const float* scale, const float* zero, int64_t param_ld,
                         const int* colmap, int maxq,
                         int8_t* codes, float* err,
                         const float* z, float* ghinv, const float* p,
                         const float* wraw, float approx_beta, void* stream);

/* Whole block traversal of fasterquant: for each block of `blocksize`
 * columns (dynamic groups: find parameters at each group start from the
 * current W), compensate the block, then apply the trailing update
 * W[:, i2:] -= Err @ U[i1:i2, i2:] (plus the G2PTQ / GPTAQ terms).
 * W: [nl, rows, C] fp32, overwritten with the dequantized weights.
 * U: [nl, C, C] upper factors.  scale/zero: [nl*rows, ngroups] (static
 * parameters are read, dynamic ones are written).  colgroup[c]: parameter
 * column of (permuted) column c.  codes: [nl, rows, C] int8 output.
 * G2PTQ: z [nl, rows, C] read, gh [nl, rows, C] updated; with --approx_grad
 * wraw [nl, rows, C] holds the traversal's input weights (the reference's
 * W_raw snapshot, g2ptq_utils.py:270-273) and approx_beta the shrink factor
 * (NULL / 0 otherwise).  GPTAQ: p [nl, C, C].
 * precision: 0 = fp32 CUDA-core trailing update, 1 = tensor cores
 * (fp16 hi/lo operands with power-of-two row / column scales).  clip (NULL: plain min/max) selects the clip search for
 * the dynamic group parameters, its hdiag indexed by the permuted column.
 * Needs g2q_compensate_workspace_bytes bytes; *status receives
 * G2Q_ERR_BAD_SCALE on a non-positive dynamic scale.
 * Replaces GPTQ._run_compensation (gptq_utils/gptq_utils.py:165-232),
 * G2PTQ._run_compensation (gptq_utils/g2ptq_utils.py:252-347) and
 * GPTAQ._run_compensation (gptq_utils/gptaq_utils.py:193-261). */
int g2q_compensate(int method, float* W, int64_t nl, int64_t rows, int64_t C,
                   const float* U, float* scale, float* zero, int64_t ngroups,
                   const int* colgroup, int dynamic_groups, int groupsize, int bits, int sym,
                   int blocksize, int8_t* codes,
                   const float* z, float* gh, const float* p, const float* wraw,
                   float approx_beta, const g2q_clip_t* clip,
                   int precision, void* workspace, size_t workspace_bytes, int* status,
                   void* stream);
size_t g2q_compensate_workspace_bytes(int method, int64_t nl, int64_t rows, int64_t C,
                                      int precision);

/* Hessian preparation of fasterquant for `nl` layers: an all-zero H[b]
 * becomes the identity (RTN fallback); columns with H[b][c][c] == 0 get
 * H[b][c][c] = 1 and W[b][:, c] = 0 (and, when extra != NULL, extra[b][:, c]
 * = 0 with the same layout as W; when gzero != NULL and H[b] was all zero,
 * gzero[b] is cleared, rows x C).  W is [nl, rows, C].
 * Replaces gptq_utils/gptq_utils.py:272-277, gptaq_utils.py:302-308,
 * g2ptq_utils.py:394-401. */
int g2q_prepare_hessian(float* H, int64_t nl, int64_t C, float* W, int64_t rows,
                        float* extra, int64_t extra_rows, float* gzero, void* stream);

/* Stable descending argsort of key[0..n) (ties keep index order) into perm
 * (int64).  Replaces torch.argsort(..., descending=True) of the act-order
 * permutation, gptq_utils/gptq_utils.py:281-282. */
int g2q_argsort_desc(int64_t* perm, const float* key, int64_t n, void* stream);

/* key[c] = mean over nl layers of H[b][c][c]  (gptq_utils/gptq_utils.py:281). */
int g2q_mean_diag(float* key, const float* H, int64_t nl, int64_t C, void* stream);

/* dst[b][r][c] = src[b][r][perm[c]] for float (elem_bytes 4) or int8 (1).
 * With inverse != 0: dst[b][r][perm[c]] = src[b][r][c]. */
int g2q_permute_cols(void* dst, const void* src, int elem_bytes, int64_t nl, int64_t rows,
                     int64_t C, const int64_t* perm, int inverse, void* stream);

/* dst[b][i][j] = src[b][perm[i]][perm[j]]  (gptq_utils/gptq_utils.py:289). */
int g2q_permute_sym(float* dst, const float* src, int64_t nl, int64_t C,
                    const int64_t* perm, void* stream);

/* Casts n fp32 values to dst_dtype (G2Q_DTYPE_BF16/F16/F32) and counts NaNs
 * into *nan_count (device int, accumulated).  Replaces the write-back cast and
 * NaN check of gptq_utils/gptq_utils.py:346-350. */
int g2q_cast_check(void* dst, int dst_dtype, const float* src, int64_t n, int* nan_count,
                   void* stream);

/* compressed-tensors packing of int8 codes [rows, cols] into int32
 * [rows, ceil(cols / (32/bits))]: value + 2^(bits-1), 32/bits values per
 * word, first value in the lowest bits.  Replaces pack_to_int32 as called by
 * utils/compressed_tensors_utils.py:39. */
int g2q_pack_int32(int32_t* out, const int8_t* codes, int64_t rows, int64_t cols, int bits,
                   void* stream);

/* G2PTQ trust-region step size (gptq_utils/g2ptq_utils.py:459-470):
 * with GH = grad @ Hinv, qe = Qsub - Wsub, d = diag(Hinv)[c]:
 *   loss = |(qe*GH + qe^2/2) / d|,  c_ = sum_c(grad*GH) - GH^2/d
 *   c_ = max(c_, 2 alpha loss, tiny);  beta = mean_c(1 - sqrt(max(1 - 2 alpha loss / c_, 0)))
 * All of grad, GH, Qsub, Wsub are [nl, rows, C]; dinv is [nl, C];
 * beta is [nl, rows]. */
int g2q_trust_region_beta(float* beta, const float* grad, const float* GH,
                          const float* Qsub, const float* Wsub, const float* dinv,
                          int64_t nl, int64_t rows, int64_t C, float alpha, void* stream);

/* dinv[b][c] = sum_k U[b][k][c]^2 = diag(U^T U)  -- the diagonal of H^-1. */
int g2q_diag_of_utu(float* dinv, const float* U, int64_t nl, int64_t C, void* stream);

/* X[b][r][c] *= s[b*rows + r]  (row scaling, G2PTQ Z = (G U^T) * beta). */
int g2q_scale_rows(float* X, const float* s, int64_t nl, int64_t rows, int64_t C,
                   void* stream);

/* ---- G2PTQ refresh step (saliency and gradient caches, block losses) ---- */

/* out[t][g] = mean over columns g*R/G .. (g+1)*R/G - 1 of grad[t][:]^2, fp32
 * ([T, G], contiguous); grad is [T, R] with row stride ld (G2Q_DTYPE_*).
 * R % G != 0 is invalid.  Replaces SaliencyCache.grad_hook,
 * gptq_utils/g2ptq_utils.py:605-618. */
int g2q_saliency(float* out, const void* grad, int dtype, int64_t ld, int64_t T, int64_t R,
                 int G, void* stream);

/* out[i] = (first ? 0 : out[i]) + w * x[i], product and sum rounded apart.
 * One term of the weighted sum over loss types of summarize_saliency /
 * summarize_gradients, gptq_utils/g2ptq_utils.py:620-640 and 704-711. */
int g2q_scaled_accumulate(float* out, const float* x, int64_t n, float w, int first,
                          void* stream);

/* cache[i] = (first ? 0 : cache[i] * keep) + grad[i] * inv, each operation
 * rounded apart; with keep = i / (i + 1) and inv the fp32 reciprocal of
 * n_tokens * (i + 1) this is GradientCache.cache_gradient,
 * gptq_utils/g2ptq_utils.py:693-702 (torch divides by a host scalar on the
 * GPU as a multiply by its fp32 reciprocal). */
int g2q_running_mean(float* cache, const void* grad, int dtype, int64_t n, float keep,
                     float inv, int first, void* stream);

/* Block-loss forward over `rows` rows of V values (x row stride ldx; target,
 * same dtype, stride ldt, for KL and MSE; int64 labels [rows] for NLL, -100 =
 * ignored row, other out-of-range labels give a NaN row loss).  Writes
 * row_stats [rows][3] (the base-2 log-sum-exp of x and of target, the row's
 * loss) and loss[0] = the sum of the row losses in a fixed order.
 * KL replaces F.kl_div(F.log_softmax(x), F.softmax(target), "none").sum()
 * (gptq_utils/g2ptq_utils.py:992-997), NLL F.cross_entropy(x, labels, "sum")
 * (:981-985), MSE F.mse_loss(x, target, "none").mean(-1).sum() / 2
 * (:1020-1033); computed in fp32 whatever the input dtype. */
int g2q_block_loss_forward(int kind, float* loss, float* row_stats, const void* x,
                           const void* target, const int64_t* labels, int dtype, int64_t ldx,
                           int64_t ldt, int64_t rows, int64_t V, void* stream);

/* The gradient of that loss with respect to x, times *grad_scale (a device
 * float; NULL = 1), written in x's dtype with row stride ldg: KL
 * softmax(x) - softmax(target), NLL softmax(x) - onehot(label) (0 for
 * ignored rows), MSE (x - target) / V.  row_stats from the forward. */
int g2q_block_loss_backward(int kind, void* grad, int64_t ldg, const float* row_stats,
                            const void* x, const void* target, const int64_t* labels, int dtype,
                            int64_t ldx, int64_t ldt, const float* grad_scale, int64_t rows,
                            int64_t V, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* G2PTQ_B200_H */
